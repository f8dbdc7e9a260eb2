"""Qwen3-shape decode step built from the adallm_b200 kernels.

This is the hot loop of the reference runtime -- ``ModelRunner.run_model`` replaying
one CUDA graph of ``Qwen3DecoderLayer.forward`` x L (adallm/runtime/model_runner.py:307-323,
adallm/architectures/qwen3.py:1358-1371, :471-487, :512-516) -- restated over this
package's ops so it can be timed and checked on its own:

    residual-add + RMSNorm            (adallm/ops/layernorm.py:28-40)
    qkv_proj  NVFP4 (column-parallel)  (adallm/ops/linear.py:158-191)
    q/k per-head RMSNorm, RoPE         (adallm/architectures/qwen3.py:481-484)
    FP8 KV store + paged decode attn   (adallm/ops/attention.py:307-428)
    o_proj    NVFP4 (row-parallel, all-reduce)   (adallm/ops/linear.py:193-215)
    residual-add + RMSNorm, gate_up NVFP4, SiLU*up, down NVFP4 (+ all-reduce)
    final RMSNorm, lm_head (bf16, vocab-parallel) and greedy argmax

Tensor parallelism follows the reference's sharding exactly: column-parallel shards
of q / k / v and gate / up rows, row-parallel shards of the K dimension of o_proj and
down_proj, head-sharded KV cache, vocab-sharded embedding / lm_head
(adallm/ops/embed_head.py:9-66).  The reduction after the row-parallel projections (an NCCL
all-reduce in the reference) runs over NVLink peer memory: each rank's GEMM writes its
partials into every rank's inbox and the next RMSNorm sums them (``_gemm_rowpar``).

Weights are random-init NVFP4 (random e2m1 codes, e4m3 block scales and a per-matrix
fp32 scale_2, sized so every projection has roughly unit gain).  They are generated on
the device from seeded generators per full (unsharded) matrix, so every tensor-parallel
rank holds exactly its slice of the same model.
"""
from __future__ import annotations

import ctypes as C
import math
import os
import zlib
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.distributed as dist

from . import _native as N
from .nvfp4_gemm import prepack_scales, sf_bytes, workspace_bytes

# In the decode step the kernel right before attention is qk_norm_rope_store, which appends each
# sequence's new K/V row at position context_lens - 1 (slot_mapping is that position) and writes
# q; context_lens and block_tables come from the host upload or advance(), both long before.  So
# attention may read its metadata and start the older cache tiles' loads before waiting.
ATTN_META_EARLY = 1


@dataclass
class DecodeConfig:
    num_layers: int = 36
    hidden: int = 4096
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 12288
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position: int = 40960
    page_size: int = 16
    terms: int = 4
    tp_size: int = 1
    tp_rank: int = 0

    @property
    def hq(self):
        return self.num_heads // self.tp_size

    @property
    def hkv(self):
        return self.num_kv_heads // self.tp_size

    @property
    def inter(self):
        return self.intermediate // self.tp_size

    @property
    def vocab_shard(self):
        return self.vocab // self.tp_size


QWEN3_8B = DecodeConfig()


@dataclass
class NVFP4Weight:
    packed: torch.Tensor      # uint8 [N, K/2]
    scale: torch.Tensor       # fp16 [N, K/16]  (reference parameter layout)
    scale_2: torch.Tensor     # fp32 []
    sf: torch.Tensor = field(default=None)  # prepacked scale factors

    @property
    def n(self):
        return self.packed.shape[0]

    @property
    def k(self):
        return self.packed.shape[1] * 2


def stable_seed(*parts) -> int:
    """Process-independent seed (Python's str hash is salted per process)."""
    return zlib.crc32(repr(parts).encode()) & 0x7FFFFFFF


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def random_nvfp4(n: int, k: int, seed: int, device) -> tuple[torch.Tensor, torch.Tensor, float]:
    """Full [n, k] random NVFP4 matrix: uniform e2m1 codes, e4m3 block scales in
    [0.5, 2], scale_2 chosen for unit gain (E[code^2] = 8.5625 for uniform codes)."""
    g = _gen(seed, device)
    packed = torch.randint(0, 256, (n, k // 2), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
    sbits = torch.randint(0x30, 0x41, (n, k // 16), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
    scale = sbits.view(torch.float8_e4m3fn).to(torch.float16)
    scale_2 = 1.0 / (math.sqrt(k) * math.sqrt(8.5625) * 1.1)
    return packed, scale, scale_2


def sharded_nvfp4(seed: int, kind: str, layer: int, parts: list[tuple[str, int]], k_full: int, split_k: bool,
                  tp_size: int, tp_rank: int, device) -> tuple[torch.Tensor, torch.Tensor, float]:
    """This rank's shard of a (possibly fused) random NVFP4 linear, in the reference layout.

    parts: [(name, full_rows)], each generated whole from its own seed and sharded per rank,
    then concatenated like QKVParallelLinear / MergedColumnParallelLinear
    (adallm/ops/linear.py:138-191); split_k shards K like RowParallelLinear
    (adallm/ops/linear.py:193-209).  One fp32 global scale per fused linear (the loader keeps
    the last shard's, adallm/infra/loader.py:103-115; here all parts share it)."""
    packs, scales = [], []
    scale_2 = None
    for name, rows in parts:
        packed, scale, s2 = random_nvfp4(rows, k_full, stable_seed(seed, kind, layer, name), device)
        scale_2 = s2 if scale_2 is None else scale_2
        if split_k:
            kk = k_full // tp_size
            packed = packed[:, tp_rank * kk // 2:(tp_rank + 1) * kk // 2]
            scale = scale[:, tp_rank * kk // 16:(tp_rank + 1) * kk // 16]
        else:
            r = rows // tp_size
            packed = packed[tp_rank * r:(tp_rank + 1) * r]
            scale = scale[tp_rank * r:(tp_rank + 1) * r]
        packs.append(packed.contiguous())
        scales.append(scale.contiguous())
    return torch.cat(packs).contiguous(), torch.cat(scales).contiguous(), scale_2


def fill_rows(out: torch.Tensor, seed: int, name: str, row0: int, chunk: int = 4096) -> None:
    """Rows [row0, row0 + len(out)) of a random bf16 table N(0, 0.02), generated in fixed chunks so
    that a vocab shard equals the same rows of the full table on every rank."""
    rows = out.shape[0]
    for ci in range(row0 // chunk, (row0 + rows - 1) // chunk + 1):
        g = _gen(stable_seed(seed, name, ci), out.device)
        blk = (torch.randn((chunk, out.shape[1]), generator=g, device=out.device) * 0.02).to(torch.bfloat16)
        lo = max(row0, ci * chunk)
        hi = min(row0 + rows, (ci + 1) * chunk)
        out[lo - row0:hi - row0] = blk[lo - ci * chunk:hi - ci * chunk]


def vocab_parallel_pick(local_max: torch.Tensor, local_idx: torch.Tensor, tp_rank: int, vocab_shard: int,
                        tp_size: int, group=None) -> torch.Tensor:
    """Greedy token over a vocab-parallel lm_head (adallm/ops/embed_head.py:56-66 gathers the
    logits instead): all-gather each rank's (max logit, global index) and take the first global
    maximum, i.e. torch.argmax over the full vocabulary.  Returns int64 [B]."""
    pair = torch.stack([local_max.float(), (local_idx + tp_rank * vocab_shard).float()], 1)
    allp = [torch.empty_like(pair) for _ in range(tp_size)]
    dist.all_gather(allp, pair, group=group)
    vals = torch.stack([p[:, 0] for p in allp], 1)
    idx = torch.stack([p[:, 1] for p in allp], 1)
    best = vals.argmax(dim=1, keepdim=True)  # ties: the lower rank, i.e. the lower index
    return idx.gather(1, best).view(-1).to(torch.int64)


class Qwen3DecodeEngine:
    """Static-shape decode engine for batch ``max_batch`` (graph-capturable)."""

    def __init__(self, cfg: DecodeConfig, device, max_batch: int, max_ctx: int, seed: int = 0,
                 group=None, fused: bool = True):
        self.cfg = cfg
        self.fused = fused
        # each GEMM pulling the next one's weights into L2 (ADALLM_B200_L2_PREFETCH=1) measured 2%
        # slower on the Qwen3-8B step (7,671 vs 7,833 tok/s): off by default
        self.l2_prefetch = os.environ.get("ADALLM_B200_L2_PREFETCH", "0") == "1"
        self.device = torch.device(device)
        self.B = max_batch
        self.max_pages_per_seq = -(-max_ctx // cfg.page_size)
        self.group = group
        self.seed = seed
        self._init_weights()
        self._alloc_state()
        if self.tp_peer:
            self._setup_peers()

    # ------------------------------------------------------------------ weights
    def _sharded(self, kind: str, layer: int, parts: list[tuple[str, int]], k_full: int, split_k: bool) -> NVFP4Weight:
        c = self.cfg
        packed, scale, scale_2 = sharded_nvfp4(self.seed, kind, layer, parts, k_full, split_k, c.tp_size, c.tp_rank,
                                               self.device)
        w = NVFP4Weight(packed, scale, torch.tensor(scale_2, dtype=torch.float32, device=self.device))
        w.sf = prepack_scales(w.scale, w.n, w.k)
        return w

    def _init_weights(self):
        c = self.cfg
        d = self.device
        D = c.head_dim
        self.layers = []
        for li in range(c.num_layers):
            L = {}
            L["qkv"] = self._sharded("qkv", li, [("q", c.num_heads * D), ("k", c.num_kv_heads * D),
                                                 ("v", c.num_kv_heads * D)], c.hidden, False)
            L["o"] = self._sharded("o", li, [("o", c.hidden)], c.num_heads * D, True)
            L["gate_up"] = self._sharded("gu", li, [("gate", c.intermediate), ("up", c.intermediate)], c.hidden,
                                         False)
            L["down"] = self._sharded("down", li, [("down", c.hidden)], c.intermediate, True)
            L["in_norm"] = torch.ones(c.hidden, dtype=torch.bfloat16, device=d)
            L["post_norm"] = torch.ones(c.hidden, dtype=torch.bfloat16, device=d)
            L["q_norm"] = torch.ones(D, dtype=torch.bfloat16, device=d)
            L["k_norm"] = torch.ones(D, dtype=torch.bfloat16, device=d)
            self.layers.append(L)
        self.final_norm = torch.ones(c.hidden, dtype=torch.bfloat16, device=d)
        v0 = c.tp_rank * c.vocab_shard
        emb = torch.empty((c.vocab_shard, c.hidden), dtype=torch.bfloat16, device=d)
        # generated in fixed chunks so every rank's shard equals the same rows of the full table
        self._fill_rows(emb, "embed", v0)
        self.embed = emb
        lm = torch.empty((c.vocab_shard, c.hidden), dtype=torch.bfloat16, device=d)
        self._fill_rows(lm, "lm_head", v0)
        self.lm_head = lm
        from .rotary_embedding import build_cos_sin_cache
        self.cos_sin = build_cos_sin_cache(D, c.max_position, c.rope_theta, None, d).contiguous()

    def _fill_rows(self, out: torch.Tensor, name: str, row0: int):
        fill_rows(out, self.seed, name, row0)

    # ------------------------------------------------------------------ state
    def _alloc_state(self):
        c = self.cfg
        d = self.device
        B, D = self.B, c.head_dim
        bf = torch.bfloat16
        self.num_pages = B * self.max_pages_per_seq
        # [2, L, pages, page, Hkv, D] like ModelRunner.allocate_kv_cache (model_runner.py:137-169)
        self.kv_cache = torch.zeros((2, c.num_layers, self.num_pages, c.page_size, c.hkv, D),
                                    dtype=torch.float8_e4m3fn, device=d)
        # per-step inputs (static for graph capture)
        self.input_ids = torch.zeros(B, dtype=torch.int64, device=d)
        self.positions = torch.zeros(B, dtype=torch.int64, device=d)
        self.slot_mapping = torch.zeros(B, dtype=torch.int32, device=d)
        self.context_lens = torch.zeros(B, dtype=torch.int32, device=d)
        self.block_tables = torch.full((B, self.max_pages_per_seq), -1, dtype=torch.int32, device=d)
        self.next_tokens = torch.zeros(B, dtype=torch.int64, device=d)
        # activations
        H, qkv_n = c.hidden, (c.hq + 2 * c.hkv) * D
        self.hidden = torch.zeros((B, H), dtype=bf, device=d)
        self.residual = torch.zeros((B, H), dtype=bf, device=d)
        self.xnorm = torch.zeros((B, H), dtype=bf, device=d)
        self.qkv = torch.zeros((B, qkv_n), dtype=bf, device=d)
        self.q_rot = torch.zeros((B, c.hq, D), dtype=bf, device=d)
        self.attn = torch.zeros((B, c.hq, D), dtype=bf, device=d)
        self.gate_up = torch.zeros((B, 2 * c.inter), dtype=bf, device=d)
        self.act = torch.zeros((B, c.inter), dtype=bf, device=d)
        self.logits = torch.zeros((B, c.vocab_shard), dtype=bf, device=d)
        # lm_head + greedy pick (ada_lm_head_argmax), in groups of at most 64 tokens
        self.lm_group = min(B, 64)
        self.lmh_ws = torch.zeros(int(N.lib().ada_lm_head_workspace_size(self.lm_group, c.vocab_shard)),
                                  dtype=torch.uint8, device=d)
        self.local_max = torch.zeros(B, dtype=torch.float32, device=d)
        # workspaces (zeroed once; the kernels leave them ready for reuse)
        shapes = [(B, w.n, w.k) for w in self.layers[0].values() if isinstance(w, NVFP4Weight)]
        self.gemm_ws = torch.zeros(max(workspace_bytes(*s, c.terms) for s in shapes), dtype=torch.uint8, device=d)
        self.attn_ws_bytes = int(N.lib().ada_fp8_paged_decode_workspace_size(B, c.hq, self.max_pages_per_seq,
                                                                             c.page_size, D))
        # quantised GEMM operands written by the fused producers (ada_nvfp4_act_quant layout)
        self.bn = int(N.lib().ada_nvfp4_block_n(B, c.terms))
        self.m_pad = -(-B // self.bn) * self.bn

        def qbuf(k):
            sf_len = (self.m_pad // self.bn) * (k // 64) * 512 if c.terms == 1 else 16  # block scales: terms == 1
            return (torch.zeros(self.m_pad * c.terms * k // 2, dtype=torch.uint8, device=d),
                    torch.zeros(sf_len, dtype=torch.uint8, device=d),
                    torch.ones(self.m_pad, dtype=torch.float32, device=d))
        self.q_hidden = qbuf(H)
        self.q_attn = qbuf(c.hq * D)
        self.q_inter = qbuf(c.inter)
        self.gemm_only_ws = torch.zeros(max(int(N.lib().ada_nvfp4_gemm_workspace_size(*s_, c.terms))
                                            for s_ in shapes), dtype=torch.uint8, device=d)
        self.attn_ws = torch.zeros(max(self.attn_ws_bytes, 256), dtype=torch.uint8, device=d)
        # split-K partial planes (TP1 fused path): each projection leaves nplanes fp32 planes
        # [nplanes][B][n] that its consumer sums; one buffer serves all four (each is consumed
        # by the very next kernel, which completes before the next projection writes)
        self.splits = {name: int(N.lib().ada_nvfp4_gemm_splits(B, w.n, w.k, c.terms))
                       for name, w in self.layers[0].items() if isinstance(w, NVFP4Weight)}
        self.use_parts = self.fused and all(v > 0 for v in self.splits.values())
        # TP > 1: the row-parallel projections (o, down) reduce across ranks through NVLink peer
        # memory inside the GEMM epilogue + the consuming RMSNorm instead of an NCCL all-reduce
        self.tp_peer = self.use_parts and c.tp_size > 1
        plane_max = max(self.splits[name] * B * w.n for name, w in self.layers[0].items()
                        if isinstance(w, NVFP4Weight))
        self.parts = torch.zeros(plane_max if self.use_parts else 4, dtype=torch.float32, device=d)

    # ------------------------------------------------------------------ TP peer memory
    def _setup_peers(self):
        """Each rank: one peer buffer [epoch][o inbox][down inbox], mapped by every other rank
        through CUDA IPC.  Inbox of a projection kind: the partial planes of all ranks as tagged
        8-byte words [world * splits][B][hidden]; at most 8 planes in all (the consumer reads
        every one of them)."""
        c, B, W = self.cfg, self.B, self.cfg.tp_size
        lib = N.lib()
        H = c.hidden

        def al(x):
            return -(-x // 256) * 256
        self.peer_ks = {name: max(1, min(self.splits[name], 8 // W)) for name in ("o", "down")}
        self.off_inbox = {"o": 256}
        self.off_inbox["down"] = self.off_inbox["o"] + al(W * self.peer_ks["o"] * B * H * 8)
        total = self.off_inbox["down"] + al(W * self.peer_ks["down"] * B * H * 8)
        base, handle = C.c_void_p(), (C.c_char * 64)()
        N.check(lib.ada_peer_alloc(total, C.byref(base), handle), "peer alloc")
        self._peer_own = base.value
        handles = [None] * W
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        self.peer_base = []
        for r in range(W):
            if r == c.tp_rank:
                self.peer_base.append(self._peer_own)
                continue
            ptr_ = C.c_void_p()
            N.check(lib.ada_peer_open(handles[r], C.byref(ptr_)), "peer open")
            self.peer_base.append(ptr_.value)
        self.epoch_ptr = self._peer_own  # steps completed on this rank (uint32)
        self.tag_mul = 2 * c.num_layers  # tag of (layer, kind) in a step: epoch * tag_mul + 2 * layer + kind + 1
        dist.barrier(group=self.group)

    def close(self):
        """Unmap the peers' buffers and free this rank's (all ranks call it, then synchronise)."""
        if getattr(self, "_peer_own", None) is None:
            return
        lib = N.lib()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for r, b in enumerate(self.peer_base):
            if r != self.cfg.tp_rank:
                lib.ada_peer_close(b)
        dist.barrier(group=self.group)
        lib.ada_peer_free(self._peer_own)
        self._peer_own = None

    def _gemm_rowpar(self, qb, w: NVFP4Weight, name: str, li: int, stream: int, next_w: NVFP4Weight | None = None):
        """Row-parallel projection (o / down): TP1 -> local partial planes; TP > 1 -> this rank's
        partials, tagged for (step, layer, kind), into every rank's inbox of that kind."""
        if not self.tp_peer:
            return ("local",) + self._gemm_parts(qb, w, name, stream, next_w=next_w)
        c, B, W = self.cfg, self.B, self.cfg.tp_size
        xq, sfx, gx = qb
        ks, kind = self.peer_ks[name], (0 if name == "o" else 1)
        inboxes = N.ptr_array([b + self.off_inbox[name] for b in self.peer_base])
        st = N.lib().ada_nvfp4_gemm_partials_peer(xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), B, c.terms, self.bn,
                                                  w.packed.data_ptr(), w.packed.stride(0), w.sf.data_ptr(),
                                                  w.scale_2.data_ptr(), w.n, w.k, w.n, B * w.n, ks, W, c.tp_rank,
                                                  C.cast(inboxes, C.c_void_p), self.epoch_ptr, self.tag_mul,
                                                  2 * li + kind + 1, self.gemm_only_ws.data_ptr(),
                                                  self.gemm_only_ws.numel(), stream)
        N.check(st, "NVFP4 kernel (peer partials)")
        return ("peer", name, li, ks, w.n)

    # ------------------------------------------------------------------ ops
    def _linear(self, x: torch.Tensor, w: NVFP4Weight, y: torch.Tensor, stream: int, name: str | None = None):
        """act-quant + GEMM; with the split count of the partial-plane path, so both paths sum
        the same K splits in the same order (bit-identical results)."""
        c = self.cfg
        ks = self.splits.get(name, 0) if name else 0
        st = N.lib().ada_nvfp4_linear_ex(x.data_ptr(), 0, x.stride(0), x.shape[0], w.k, w.packed.data_ptr(),
                                         w.packed.stride(0), w.sf.data_ptr(), w.scale_2.data_ptr(), w.n, None,
                                         y.data_ptr(), 0, y.stride(0), c.terms, ks, self.gemm_ws.data_ptr(),
                                         self.gemm_ws.numel(), stream)
        N.check(st, "NVFP4 kernel")

    def _gemm(self, qb, w: NVFP4Weight, y: torch.Tensor, stream: int):
        c = self.cfg
        xq, sfx, gx = qb
        st = N.lib().ada_nvfp4_gemm(xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), self.B, c.terms, self.bn,
                                    w.packed.data_ptr(), w.packed.stride(0), w.sf.data_ptr(), w.scale_2.data_ptr(),
                                    w.n, w.k, None, y.data_ptr(), 0, y.stride(0), 0, self.gemm_only_ws.data_ptr(),
                                    self.gemm_only_ws.numel(), stream)
        N.check(st, "NVFP4 kernel")

    def _gemm_parts(self, qb, w: NVFP4Weight, name: str, stream: int, next_w: NVFP4Weight | None = None):
        """Partial-plane GEMM; with next_w (and L2 prefetch on) its CTAs also pull the next
        projection's packed weights and scale factors into L2 once their own loads are issued."""
        c = self.cfg
        xq, sfx, gx = qb
        ns = self.splits[name]
        nw = next_w if self.l2_prefetch else None
        st = N.lib().ada_nvfp4_gemm_partials_pf(xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), self.B, c.terms,
                                                self.bn, w.packed.data_ptr(), w.packed.stride(0), w.sf.data_ptr(),
                                                w.scale_2.data_ptr(), w.n, w.k, self.parts.data_ptr(), w.n,
                                                self.B * w.n, ns, N.ptr(nw.packed if nw else None),
                                                nw.packed.numel() if nw else 0, N.ptr(nw.sf if nw else None),
                                                nw.sf.numel() if nw else 0, self.gemm_only_ws.data_ptr(),
                                                self.gemm_only_ws.numel(), stream)
        N.check(st, "NVFP4 kernel")
        return ns, w.n  # planes, row stride

    def _rms_quant_parts(self, planes, w, qb, stream, y=None):
        """residual += sum(planes); normed = RMSNorm(residual); quantised into qb (or into y when
        qb is None).  planes: ("local", n, ld) in self.parts, or ("peer", kind, layer, splits, ld):
        all ranks' planes in this rank's inbox of that kind, once their count has arrived."""
        c = self.cfg
        H = c.hidden
        rp = self.residual.data_ptr()
        xq, sfx, gx = qb if qb is not None else (None, None, None)
        if planes[0] == "local":
            _, ns, ld = planes
            st = N.lib().ada_rmsnorm_quant_parts(self.parts.data_ptr(), ns, self.B * ld, ld, rp, H, rp, H,
                                                 w.data_ptr(), N.ptr(y), H, self.B, H, c.rms_eps, 0, 0, c.terms,
                                                 self.bn, N.ptr(xq), N.ptr(sfx), N.ptr(gx), stream)
        else:
            _, name, li, ks, ld = planes
            W, kind = c.tp_size, (0 if name == "o" else 1)
            st = N.lib().ada_rmsnorm_quant_peer(self._peer_own + self.off_inbox[name], W * ks, self.B * ld, ld, rp, H,
                                                rp, H, w.data_ptr(), N.ptr(y), H, self.B, H, c.rms_eps, 0, 0, c.terms,
                                                self.bn, N.ptr(xq), N.ptr(sfx), N.ptr(gx), self.epoch_ptr,
                                                self.tag_mul, 2 * li + kind + 1, self.gemm_only_ws.data_ptr(), stream)
        N.check(st, "rms_norm+quant")

    def _rms_quant(self, x, w, qb, stream, residual=None):
        c = self.cfg
        H = x.shape[-1]
        xq, sfx, gx = qb
        rp = residual.data_ptr() if residual is not None else None
        st = N.lib().ada_rmsnorm_quant(x.data_ptr(), H, rp, H, rp, H, w.data_ptr(), None, 0, self.B, H, c.rms_eps, 0, 0,
                                       c.terms, self.bn, xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), stream)
        N.check(st, "rms_norm+quant")

    def _rms(self, x, w, y, stream, residual=None, rows=None, hidden=None):
        c = self.cfg
        hidden = hidden or x.shape[-1]
        rows = rows or x.numel() // hidden
        if residual is None:
            st = N.lib().ada_rmsnorm(x.data_ptr(), hidden, None, 0, None, 0, w.data_ptr(), y.data_ptr(), hidden,
                                     rows, hidden, c.rms_eps, 0, 0, stream)
        else:
            st = N.lib().ada_rmsnorm(x.data_ptr(), hidden, residual.data_ptr(), hidden, residual.data_ptr(), hidden,
                                     w.data_ptr(), y.data_ptr(), hidden, rows, hidden, c.rms_eps, 0, 0, stream)
        N.check(st, "rms_norm")

    # ------------------------------------------------------------------ device error words
    def error_words(self) -> list[torch.Tensor]:
        """The int32 device words the step's kernels OR their failure codes into (sticky until
        cleared): the fused path's GEMM workspace word (GEMM pipeline waits, and at TP > 1 the
        peer-inbox waits of the consuming RMSNorm) and the standalone linear's workspace word."""
        return [self.gemm_only_ws[:4].view(torch.int32), self.gemm_ws[:4].view(torch.int32),
                self.lmh_ws[:4].view(torch.int32)]

    def check_errors(self):
        """Raise if any kernel of the steps run so far gave up a bounded wait (synchronises)."""
        code = 0
        for w in self.error_words():
            code |= int(w.item())
        N.raise_on_error_word(code, "decode step")

    def _all_reduce(self, t: torch.Tensor):
        if self.cfg.tp_size > 1:
            dist.all_reduce(t, group=self.group)

    def forward(self):
        """One decode step for the static batch: reads input_ids / positions / slot_mapping /
        context_lens / block_tables, writes next_tokens (greedy) and the KV cache."""
        c = self.cfg
        B, D = self.B, c.head_dim
        lib = N.lib()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        v0 = c.tp_rank * c.vocab_shard
        N.check(lib.ada_embedding(self.input_ids.data_ptr(), B, self.embed.data_ptr(), v0, v0 + c.vocab_shard,
                                  c.hidden, self.hidden.data_ptr(), 0, stream), "embedding")
        self._all_reduce(self.hidden)
        qn, kn = c.hq * D, c.hkv * D
        if not self.fused:
            self._layers_unfused(lib, stream)
        elif self.use_parts:
            self._layers_parts(lib, stream)
            self._lm_head(stream)
            return
        else:
            for li, L in enumerate(self.layers):
                if li == 0:
                    self.residual.copy_(self.hidden)
                    self._rms_quant(self.hidden, L["in_norm"], self.q_hidden, stream)
                else:
                    self._rms_quant(self.hidden, L["in_norm"], self.q_hidden, stream, residual=self.residual)
                self._gemm(self.q_hidden, L["qkv"], self.qkv, stream)
                kc, vc = self.kv_cache[0, li], self.kv_cache[1, li]
                N.check(lib.ada_qk_norm_rope_store(self.qkv.data_ptr(), self.qkv.stride(0), B, c.hq, c.hkv, D,
                                                   L["q_norm"].data_ptr(), L["k_norm"].data_ptr(), c.rms_eps,
                                                   self.positions.data_ptr(), self.cos_sin.data_ptr(),
                                                   self.cos_sin.shape[0], self.slot_mapping.data_ptr(),
                                                   kc.data_ptr(), vc.data_ptr(), 1.0, 1.0, self.q_rot.data_ptr(),
                                                   None, 0, stream), "qk_norm_rope_store")
                xq, sfx, gx = self.q_attn
                N.check(lib.ada_fp8_paged_decode_quant_ex(
                    self.q_rot.data_ptr(), 0, qn, D, kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1),
                    kc.stride(2), self.num_pages, self.block_tables.data_ptr(), self.block_tables.stride(0),
                    self.max_pages_per_seq, self.context_lens.data_ptr(), B, c.hq, c.hkv, D, c.page_size,
                    D ** -0.5, 1.0, 1.0, 0, None, 0, c.terms, self.bn, xq.data_ptr(), sfx.data_ptr(),
                    gx.data_ptr(), self.attn_ws.data_ptr(), self.attn_ws_bytes, ATTN_META_EARLY, stream), "attention")
                self._gemm(self.q_attn, L["o"], self.hidden, stream)
                self._all_reduce(self.hidden)
                self._rms_quant(self.hidden, L["post_norm"], self.q_hidden, stream, residual=self.residual)
                self._gemm(self.q_hidden, L["gate_up"], self.gate_up, stream)
                xq, sfx, gx = self.q_inter
                N.check(lib.ada_gated_act_quant(self.gate_up.data_ptr(), 2 * c.inter, None, 0, B, c.inter, 0, 0,
                                                c.terms, self.bn, xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(),
                                                stream), "silu_and_mul+quant")
                self._gemm(self.q_inter, L["down"], self.hidden, stream)
                self._all_reduce(self.hidden)
        self._rms(self.hidden, self.final_norm, self.xnorm, stream, residual=self.residual)
        self._lm_head(stream)

    def _layers_parts(self, lib, stream):
        """Fused step where every projection leaves split-K partial planes and the next kernel
        sums them while loading (no split-K reduction inside the GEMMs); at TP > 1 the
        row-parallel projections' planes of all ranks meet in each rank's inbox (peer memory)."""
        c = self.cfg
        B, D = self.B, c.head_dim
        qn = c.hq * D
        planes = None
        for li, L in enumerate(self.layers):
            nxt = self.layers[li + 1] if li + 1 < len(self.layers) else None
            if li == 0:
                self.residual.copy_(self.hidden)
                self._rms_quant(self.hidden, L["in_norm"], self.q_hidden, stream)
            else:
                self._rms_quant_parts(planes, L["in_norm"], self.q_hidden, stream)
            ns, ld = self._gemm_parts(self.q_hidden, L["qkv"], "qkv", stream, next_w=L["o"])
            kc, vc = self.kv_cache[0, li], self.kv_cache[1, li]
            N.check(lib.ada_qk_norm_rope_store_parts(self.parts.data_ptr(), ns, B * ld, ld, B, c.hq, c.hkv, D,
                                                     L["q_norm"].data_ptr(), L["k_norm"].data_ptr(), c.rms_eps,
                                                     self.positions.data_ptr(), self.cos_sin.data_ptr(),
                                                     self.cos_sin.shape[0], self.slot_mapping.data_ptr(),
                                                     kc.data_ptr(), vc.data_ptr(), 1.0, 1.0, self.q_rot.data_ptr(),
                                                     None, 0, stream), "qk_norm_rope_store")
            xq, sfx, gx = self.q_attn
            N.check(lib.ada_fp8_paged_decode_quant_ex(
                self.q_rot.data_ptr(), 0, qn, D, kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1),
                kc.stride(2), self.num_pages, self.block_tables.data_ptr(), self.block_tables.stride(0),
                self.max_pages_per_seq, self.context_lens.data_ptr(), B, c.hq, c.hkv, D, c.page_size,
                D ** -0.5, 1.0, 1.0, 0, None, 0, c.terms, self.bn, xq.data_ptr(), sfx.data_ptr(),
                gx.data_ptr(), self.attn_ws.data_ptr(), self.attn_ws_bytes, ATTN_META_EARLY, stream), "attention")
            planes = self._gemm_rowpar(self.q_attn, L["o"], "o", li, stream, next_w=L["gate_up"])
            self._rms_quant_parts(planes, L["post_norm"], self.q_hidden, stream)
            ns, ld = self._gemm_parts(self.q_hidden, L["gate_up"], "gate_up", stream, next_w=L["down"])
            xq, sfx, gx = self.q_inter
            N.check(lib.ada_gated_act_quant_parts(self.parts.data_ptr(), ns, B * ld, ld, None, 0, B, c.inter, 0, 0,
                                                  c.terms, self.bn, xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(),
                                                  stream), "silu_and_mul+quant")
            planes = self._gemm_rowpar(self.q_inter, L["down"], "down", li, stream,
                                       next_w=nxt["qkv"] if nxt is not None else None)
        self._rms_quant_parts(planes, self.final_norm, None, stream, y=self.xnorm)
        if self.tp_peer:  # every counter of this step has been consumed
            N.check(lib.ada_tp_epoch_advance(self.epoch_ptr, stream), "tp epoch")

    def _layers_unfused(self, lib, stream):
        """Reference-shaped sequence: every op a separate kernel (act-quant separate from the GEMM)."""
        c = self.cfg
        B, D = self.B, c.head_dim
        qn, kn = c.hq * D, c.hkv * D
        for li, L in enumerate(self.layers):
            if li == 0:
                self.residual.copy_(self.hidden)
                self._rms(self.hidden, L["in_norm"], self.xnorm, stream)
            else:
                self._rms(self.hidden, L["in_norm"], self.xnorm, stream, residual=self.residual)
            self._linear(self.xnorm, L["qkv"], self.qkv, stream, "qkv")
            kc, vc = self.kv_cache[0, li], self.kv_cache[1, li]
            # q/k RMSNorm + RoPE + FP8 KV store in one kernel (qwen3.py:481-486, attention.py:311-312)
            N.check(lib.ada_qk_norm_rope_store(self.qkv.data_ptr(), self.qkv.stride(0), B, c.hq, c.hkv, D,
                                               L["q_norm"].data_ptr(), L["k_norm"].data_ptr(), c.rms_eps,
                                               self.positions.data_ptr(), self.cos_sin.data_ptr(),
                                               self.cos_sin.shape[0], self.slot_mapping.data_ptr(), kc.data_ptr(),
                                               vc.data_ptr(), 1.0, 1.0, self.q_rot.data_ptr(), None, 0, stream),
                    "qk_norm_rope_store")
            N.check(lib.ada_fp8_paged_decode(self.q_rot.data_ptr(), 0, qn, D, kc.data_ptr(), vc.data_ptr(),
                                             kc.stride(0), kc.stride(1), kc.stride(2), self.num_pages,
                                             self.block_tables.data_ptr(), self.block_tables.stride(0),
                                             self.max_pages_per_seq, self.context_lens.data_ptr(), B, c.hq, c.hkv,
                                             D, c.page_size, D ** -0.5, 1.0, 1.0, 0, self.attn.data_ptr(), 0,
                                             self.attn_ws.data_ptr(), self.attn_ws_bytes, stream), "attention")
            self._linear(self.attn.view(B, qn), L["o"], self.hidden, stream, "o")
            self._all_reduce(self.hidden)
            self._rms(self.hidden, L["post_norm"], self.xnorm, stream, residual=self.residual)
            self._linear(self.xnorm, L["gate_up"], self.gate_up, stream, "gate_up")
            N.check(lib.ada_gated_act(self.gate_up.data_ptr(), 2 * c.inter, self.act.data_ptr(), c.inter, B, c.inter,
                                      0, 0, stream), "silu_and_mul")
            self._linear(self.act, L["down"], self.hidden, stream, "down")
            self._all_reduce(self.hidden)

    def _lm_head(self, stream):
        """logits = xnorm . lm_head^T (bf16) and this rank's greedy pick in one tensor-core pass
        (ada_lm_head_argmax); at TP > 1 the ranks' (max, index) pairs are gathered
        (vocab_parallel_pick).  The logits are kept for inspection (4.8 MB at bs16)."""
        c = self.cfg
        H, V = self.xnorm.shape[1], c.vocab_shard
        for g0 in range(0, self.B, self.lm_group):
            g1 = min(self.B, g0 + self.lm_group)
            st = N.lib().ada_lm_head_argmax(self.xnorm[g0].data_ptr(), H, g1 - g0, H, self.lm_head.data_ptr(),
                                            self.lm_head.stride(0), V, 0, self.logits[g0].data_ptr(), V,
                                            self.next_tokens[g0].data_ptr(), self.local_max[g0].data_ptr(),
                                            self.lmh_ws.data_ptr(), self.lmh_ws.numel(), stream)
            N.check(st, "lm_head")
        if c.tp_size > 1:
            self.next_tokens.copy_(vocab_parallel_pick(self.local_max, self.next_tokens, c.tp_rank, c.vocab_shard,
                                                       c.tp_size, self.group))

    # ------------------------------------------------------------------ graphs
    def advance(self):
        """Device-side bookkeeping of one generated token (the next step's inputs), the
        on-device counterpart of ModelRunner.prepare_decode (model_runner.py:278-298)."""
        page = self.cfg.page_size
        self.input_ids.copy_(self.next_tokens)
        self.positions.add_(1)
        self.context_lens.add_(1)
        pg = torch.div(self.positions, page, rounding_mode="floor").unsqueeze(1)
        blk = self.block_tables.gather(1, pg).squeeze(1).to(torch.int64)
        self.slot_mapping.copy_((blk * page + self.positions % page).to(torch.int32))

    def capture(self, with_advance: bool = False) -> torch.cuda.CUDAGraph:
        """Capture forward() (and optionally advance()) into one CUDA graph, the way the
        reference captures its decode step (model_runner.py:333-368)."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):  # warm-up outside capture (sets kernel attributes, NCCL comms)
            self.forward()
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.forward()
            if with_advance:
                self.advance()
        return g

    def kernels_per_step(self) -> int:
        """adallm_b200 kernels launched by one forward(): embedding; per layer fused: norm+quant x2,
        GEMM x4, qk-norm/rope/store, attention (one kernel for short caches, else split +
        merge+quant), SiLU*up+quant (unfused: norm x2, act-quant + GEMM x4, qk-norm/rope/store,
        attention split + merge (or one kernel), SiLU*up); final norm; argmax x2; TP peer path:
        the epoch advance."""
        attn = 1 if self.max_pages_per_seq * self.cfg.page_size <= 1024 and self.cfg.hkv <= 8 else 2
        per_layer = (8 if self.fused else 12) + attn
        return 1 + self.cfg.num_layers * per_layer + 3 + (1 if getattr(self, "tp_peer", False) else 0)

    def export_cpu_weights(self) -> dict:
        """CPU copies in the reference parameter layout (tensor-parallel size 1 only)."""
        assert self.cfg.tp_size == 1
        layers = []
        for L in self.layers:
            d = {}
            for name in ("qkv", "o", "gate_up", "down"):
                w = L[name]
                d[name] = (w.packed.cpu(), w.scale.cpu(), float(w.scale_2.item()))
            for name in ("in_norm", "post_norm", "q_norm", "k_norm"):
                d[name] = L[name].cpu()
            layers.append(d)
        return dict(layers=layers, embed=self.embed.cpu(), lm_head=self.lm_head.cpu(),
                    final_norm=self.final_norm.cpu(), cos_sin=self.cos_sin.cpu())


class DecodeSession:
    """Host-side sequence bookkeeping for a static batch, mirroring ModelRunner.prepare_decode
    (adallm/runtime/model_runner.py:278-298): every sequence owns a seeded random set of pages
    of the pool (as a block manager would hand out), and each step uploads token ids,
    positions, slot_mapping and context_lens from pinned host memory."""

    def __init__(self, engine: Qwen3DecodeEngine, seed: int = 0):
        self.e = engine
        B, P = engine.B, engine.max_pages_per_seq
        g = torch.Generator().manual_seed(seed)
        perm = torch.randperm(engine.num_pages, generator=g).to(torch.int32)
        self.block_tables = perm.view(B, P).contiguous()
        engine.block_tables.copy_(self.block_tables)
        self.lens = torch.zeros(B, dtype=torch.int64)
        pin = torch.cuda.is_available()
        self.h_ids = torch.zeros(B, dtype=torch.int64).pin_memory() if pin else torch.zeros(B, dtype=torch.int64)
        self.h_pos = torch.zeros(B, dtype=torch.int64).pin_memory() if pin else torch.zeros(B, dtype=torch.int64)
        self.h_slot = torch.zeros(B, dtype=torch.int32).pin_memory() if pin else torch.zeros(B, dtype=torch.int32)
        self.h_ctx = torch.zeros(B, dtype=torch.int32).pin_memory() if pin else torch.zeros(B, dtype=torch.int32)
        self.h_out = torch.zeros(B, dtype=torch.int64).pin_memory() if pin else torch.zeros(B, dtype=torch.int64)
        # the engine's device error words, read back with the tokens of every step
        nerr = len(engine.error_words())
        self.h_err = torch.zeros(nerr, dtype=torch.int32).pin_memory() if pin else torch.zeros(nerr, dtype=torch.int32)

    H2D_BYTES_PER_STEP = property(lambda self: self.e.B * (8 + 8 + 4 + 4))
    D2H_BYTES_PER_STEP = property(lambda self: self.e.B * 8 + 4 * self.h_err.numel())  # tokens + error words

    def prepare(self, tokens: torch.Tensor):
        """Fill the pinned input buffers for the next step (numpy views: a few microseconds)."""
        page = self.e.cfg.page_size
        pos = self.lens.numpy()
        self.h_ids.numpy()[:] = tokens.numpy() if isinstance(tokens, torch.Tensor) else tokens
        self.h_pos.numpy()[:] = pos
        blk = self.block_tables.numpy()[np.arange(pos.shape[0]), pos // page].astype(np.int64)
        self.h_slot.numpy()[:] = blk * page + pos % page
        self.h_ctx.numpy()[:] = pos + 1

    def upload(self):
        e = self.e
        e.input_ids.copy_(self.h_ids, non_blocking=True)
        e.positions.copy_(self.h_pos, non_blocking=True)
        e.slot_mapping.copy_(self.h_slot, non_blocking=True)
        e.context_lens.copy_(self.h_ctx, non_blocking=True)

    def _copy_errors(self):
        for i, w in enumerate(self.e.error_words()):
            self.h_err[i:i + 1].copy_(w, non_blocking=True)

    def _raise_on_errors(self):
        """A bounded device wait that ran out (a GEMM pipeline stage, or at TP > 1 a peer's words
        that never arrived) leaves a code in an error word; the tokens of that step are not
        trusted: raise instead of returning them."""
        code = 0
        for v in self.h_err.tolist():
            code |= int(v)
        N.raise_on_error_word(code, "decode step")

    def download(self) -> torch.Tensor:
        self.h_out.copy_(self.e.next_tokens, non_blocking=True)
        self._copy_errors()
        torch.cuda.current_stream(self.e.device).synchronize()
        self._raise_on_errors()
        return self.h_out.clone()

    def capture_step(self) -> torch.cuda.CUDAGraph:
        """One CUDA graph for a host-fed step: H2D of the pinned inputs, forward(), D2H of the
        greedy tokens into pinned memory.  step() replays it."""
        e = self.e
        s = torch.cuda.Stream(e.device)
        s.wait_stream(torch.cuda.current_stream(e.device))
        with torch.cuda.stream(s):  # warm-up outside capture
            self.upload()
            e.forward()
        torch.cuda.current_stream(e.device).wait_stream(s)
        torch.cuda.synchronize(e.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.upload()
            e.forward()
            self.h_out.copy_(e.next_tokens, non_blocking=True)
            self._copy_errors()
        self._step_graph = g
        return g

    def step(self, tokens) -> torch.Tensor:
        """prepare + replay of the captured step + wait for the tokens (capture_step() first);
        raises RuntimeError if a kernel of the step reported a failed wait."""
        self.prepare(tokens)
        self._step_graph.replay()
        torch.cuda.current_stream(self.e.device).synchronize()
        self._raise_on_errors()
        return self.h_out.clone()

    def commit(self):
        self.lens += 1
