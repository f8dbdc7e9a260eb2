"""Qwen3-MoE-shape decode step built from the adallm_b200 kernels (
Qwen3-30B-A3B shape), tensor-parallel size 1 as the reference runs MoE (qwen3.py:1383-1384).

Per decoder layer (Qwen3MoeDecoderLayer.forward, adallm/architectures/qwen3.py:1400-1412) the
attention half is the dense engine's (decode_step.py): RMSNorm + quantised operand, qkv NVFP4
GEMM into split-K partial planes, q/k-norm + RoPE + FP8 KV store from the planes, FP8 paged
decode attention with the o_proj operand quantised in its merge, o GEMM into planes.  The MLP is
the sparse MoE block (Qwen3MoeSparseMoeBlock.forward, qwen3.py:1010-1032 and the TP = 1 expert
loop :1263-1290):

    x, residual = post_attention_layernorm(o, residual)   one kernel summing the o planes
    router_logits = gate(x)                              bf16 [T, E] (FP16Linear, qwen3.py:696)
    ids, w = softmax fp32 -> top-k -> renormalise         one kernel with the router GEMM
                                                          (ada_moe_router_topk)
    h = grouped NVFP4 gate+up over the T * top_k routed rows (only the touched experts streamed)
    a = SiLU(gate) * up;  y = grouped NVFP4 down         ada_moe_experts (5 launches)
    out = sum_k w_k * y_k                                 ada_moe_combine

The reference runs the experts as top_k separate gather GEMMs per projection (gate, up and down
each, qwen3.py:1263-1290); here gate and up are one stacked [E, 2I, H] weight, each projection is
one grouped launch over all routed rows, and one routing plan serves both.  Weights are random-init NVFP4 (decode_step.py's
generator); router weights N(0, 1/H), so router logits are ~N(0, 1) as the config states.
"""
from __future__ import annotations

import os

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native as N
from .decode_step import ATTN_META_EARLY, Qwen3DecodeEngine, random_nvfp4, stable_seed
from .nvfp4_gemm import prepack_scales


@dataclass
class MoEConfig:
    """Qwen3-30B-A3B widths: 48 layers, hidden 2048, 32 query / 4 KV heads of 128, 128 experts
    with top-8 softmax routing (renormalised), expert intermediate 768, vocab 151936."""
    num_layers: int = 48
    hidden: int = 2048
    num_heads: int = 32
    num_kv_heads: int = 4
    head_dim: int = 128
    num_experts: int = 128
    top_k: int = 8
    moe_intermediate: int = 768
    norm_topk_prob: bool = True
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position: int = 40960
    page_size: int = 16
    terms: int = 4
    tp_size: int = 1
    tp_rank: int = 0
    ep_size: int = 1   # expert parallelism: rank ep_rank holds experts [ep_rank * E / ep_size, +E / ep_size)
    ep_rank: int = 0

    hq = property(lambda self: self.num_heads)
    hkv = property(lambda self: self.num_kv_heads)
    inter = property(lambda self: self.moe_intermediate)
    intermediate = property(lambda self: self.moe_intermediate)
    vocab_shard = property(lambda self: self.vocab)


QWEN3_30B_A3B = MoEConfig()


@dataclass
class Experts:
    packed: torch.Tensor    # uint8 [E, N, K/2]
    scale: torch.Tensor     # fp16 [E, N, K/16] (reference parameter layout)
    scale_2: torch.Tensor   # fp32 [E]
    sf: torch.Tensor        # prepacked scale factors of the [E * N, K/16] scale matrix

    @property
    def e(self):
        return self.packed.shape[0]

    @property
    def n(self):
        return self.packed.shape[1]

    @property
    def k(self):
        return self.packed.shape[2] * 2


class Qwen3MoeDecodeEngine(Qwen3DecodeEngine):
    """Static-shape MoE decode engine for batch ``max_batch`` (graph-capturable).

    Attention runs at tensor-parallel size 1 (as the reference's MoE).  With cfg.ep_size > 1
    (expert parallelism, beyond the reference; one process per GPU, `group` the NCCL group of the
    ep_size ranks) every rank runs the same attention and routing, holds a contiguous block of
    experts, runs the expert MLP over the rows routed to its experts only (ada_moe_experts with
    all_local = 0), sums its slots in fp32 (ada_moe_combine_ep_f32) and all-reduces
    them: one NCCL all-reduce of [batch, hidden] fp32 per layer, rounded once to bf16 afterwards, so
    the block output is the single-GPU combine's up to the order of the fp32 additions."""

    def __init__(self, cfg: MoEConfig, device, max_batch: int, max_ctx: int, seed: int = 0, group=None):
        if cfg.tp_size != 1:
            raise ValueError("the MoE decode engine runs attention at tensor-parallel size 1 (as the reference)")
        if cfg.num_experts % cfg.ep_size or not 0 <= cfg.ep_rank < cfg.ep_size:
            raise ValueError("experts must split evenly over the expert-parallel ranks")
        self.local_experts = cfg.num_experts // cfg.ep_size
        self.expert_base = cfg.ep_rank * self.local_experts
        # at EP 1 the weighted combine is the input stage of the next RMSNorm (one launch fewer per
        # layer, the same values); ADALLM_B200_MOE_FOLD_COMBINE=0 keeps the separate combine kernel
        self.fold_combine = os.environ.get("ADALLM_B200_MOE_FOLD_COMBINE", "1") != "0"
        super().__init__(cfg, device, max_batch, max_ctx, seed=seed, group=group, fused=True)
        if not self.use_parts:
            raise ValueError("MoE engine: an attention projection has no partial-plane split at this batch")
        self._alloc_moe()

    def _experts(self, name: str, layer: int, n: int, k: int) -> Experts:
        c = self.cfg
        packs, scales, s2 = [], [], []
        for e in range(self.expert_base, self.expert_base + self.local_experts):  # seeded by the global id
            p, s, g2 = random_nvfp4(n, k, stable_seed(self.seed, "expert", name, layer, e), self.device)
            packs.append(p)
            scales.append(s)
            s2.append(g2)
        packed = torch.stack(packs).contiguous()
        scale = torch.stack(scales).contiguous()
        ne = self.local_experts
        sf = prepack_scales(scale.view(ne * n, k // 16), ne * n, k)
        return Experts(packed, scale, torch.tensor(s2, dtype=torch.float32, device=self.device), sf)

    def _init_weights(self):
        c = self.cfg
        d = self.device
        D = c.head_dim
        self.layers = []
        g = torch.Generator(device=d)
        for li in range(c.num_layers):
            L = {}
            L["qkv"] = self._sharded("qkv", li, [("q", c.num_heads * D), ("k", c.num_kv_heads * D),
                                                 ("v", c.num_kv_heads * D)], c.hidden, False)
            L["o"] = self._sharded("o", li, [("o", c.hidden)], c.num_heads * D, True)
            # gate rows then up rows of every expert (the stacked gate_up of moe_block_ep)
            L["experts_gate_up"] = self._experts("gate_up", li, 2 * c.moe_intermediate, c.hidden)
            L["experts_down"] = self._experts("down", li, c.hidden, c.moe_intermediate)
            g.manual_seed(stable_seed(self.seed, "router", li))
            L["router"] = (torch.randn((c.num_experts, c.hidden), generator=g, device=d)
                           * c.hidden ** -0.5).to(torch.bfloat16)
            for name in ("in_norm", "post_norm", "q_norm", "k_norm"):
                L[name] = torch.ones(c.hidden if name in ("in_norm", "post_norm") else D, dtype=torch.bfloat16,
                                     device=d)
            self.layers.append(L)
        self.final_norm = torch.ones(c.hidden, dtype=torch.bfloat16, device=d)
        emb = torch.empty((c.vocab, c.hidden), dtype=torch.bfloat16, device=d)
        self._fill_rows(emb, "embed", 0)
        self.embed = emb
        lm = torch.empty((c.vocab, c.hidden), dtype=torch.bfloat16, device=d)
        self._fill_rows(lm, "lm_head", 0)
        self.lm_head = lm
        from .rotary_embedding import build_cos_sin_cache
        self.cos_sin = build_cos_sin_cache(D, c.max_position, c.rope_theta, None, d).contiguous()

    def _alloc_moe(self):
        c = self.cfg
        d = self.device
        B, k = self.B, c.top_k
        bf = torch.bfloat16
        rows = B * k
        self.route_ids = torch.zeros(rows, dtype=torch.int32, device=d)
        self.route_w = torch.zeros(rows, dtype=bf, device=d)
        self.y_rows = torch.zeros((rows, c.hidden), dtype=bf, device=d)
        self.moe_sum = torch.zeros((B, c.hidden), dtype=torch.float32, device=d) if c.ep_size > 1 else None
        lib = N.lib()
        gu = self.layers[0]["experts_gate_up"]
        self.ws_experts = torch.zeros(int(lib.ada_moe_experts_workspace_size(B, k, c.hidden, c.moe_intermediate,
                                                                             c.terms, gu.e)),
                                      dtype=torch.uint8, device=d)

    def error_words(self) -> list[torch.Tensor]:
        words = super().error_words()
        if hasattr(self, "ws_experts"):
            words.append(self.ws_experts[:4].view(torch.int32))
        return words

    def _experts_mlp(self, L, stream: int):
        """self.xnorm -> self.y_rows: every routed row through its (local) expert's gate_up, SiLU*up
        and down (ada_moe_experts: one routing, the gather folded into the quantiser); rows routed
        to another rank's expert are skipped."""
        c = self.cfg
        gu, dn = L["experts_gate_up"], L["experts_down"]
        st = N.lib().ada_moe_experts(self.xnorm.data_ptr(), 0, self.xnorm.stride(0), self.B, c.top_k,
                                     self.route_ids.data_ptr(), gu.e, self.expert_base, int(c.ep_size == 1),
                                     gu.packed.data_ptr(), gu.packed.stride(1), gu.sf.data_ptr(), gu.scale_2.data_ptr(),
                                     dn.packed.data_ptr(), dn.packed.stride(1), dn.sf.data_ptr(), dn.scale_2.data_ptr(),
                                     c.moe_intermediate, c.hidden, 0, self.y_rows.data_ptr(), self.y_rows.stride(0),
                                     c.terms, self.ws_experts.data_ptr(), self.ws_experts.numel(), stream)
        N.check(st, "MoE expert MLP")

    def _moe_block(self, L, stream: int):
        """self.xnorm -> self.hidden: router, top-k, grouped experts, weighted combine."""
        c = self.cfg
        lib = N.lib()
        B = self.B
        N.check(lib.ada_moe_router_topk(self.xnorm.data_ptr(), 0, self.xnorm.stride(0), B, L["router"].data_ptr(),
                                        L["router"].stride(0), c.hidden, c.num_experts, c.top_k,
                                        int(c.norm_topk_prob), self.route_ids.data_ptr(), self.route_w.data_ptr(),
                                        self.ws_experts.data_ptr(), stream), "moe router + route")
        self._experts_mlp(L, stream)
        if c.ep_size == 1 and self.fold_combine:
            return  # the weighted combine is the input stage of the next RMSNorm (ada_rmsnorm_quant_combine)
        if c.ep_size == 1:
            N.check(lib.ada_moe_combine(self.y_rows.data_ptr(), 0, self.y_rows.stride(0), self.route_w.data_ptr(), B,
                                        c.top_k, c.hidden, self.hidden.data_ptr(), self.hidden.stride(0), stream),
                    "moe combine")
        else:  # this rank's slots in fp32, the fp32 sum over the ranks, one rounding
            N.check(lib.ada_moe_combine_ep_f32(self.y_rows.data_ptr(), 0, self.y_rows.stride(0),
                                               self.route_w.data_ptr(), self.route_ids.data_ptr(), self.expert_base,
                                               self.local_experts, B, c.top_k, c.hidden, self.moe_sum.data_ptr(),
                                               self.moe_sum.stride(0), stream), "moe combine (expert-parallel)")
            dist.all_reduce(self.moe_sum, group=self.group)
            self.hidden.copy_(self.moe_sum)

    def forward(self):
        c = self.cfg
        B, D = self.B, c.head_dim
        lib = N.lib()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        N.check(lib.ada_embedding(self.input_ids.data_ptr(), B, self.embed.data_ptr(), 0, c.vocab, c.hidden,
                                  self.hidden.data_ptr(), 0, stream), "embedding")
        qn = c.hq * D
        H = c.hidden
        fold = c.ep_size == 1 and self.fold_combine
        for li, L in enumerate(self.layers):
            xq, sfx, gx = self.q_hidden
            if li == 0:
                self.residual.copy_(self.hidden)
                res = None
            else:
                res = self.residual.data_ptr()
            if li > 0 and fold:  # the previous layer's combine + residual add + RMSNorm + quantiser
                N.check(lib.ada_rmsnorm_quant_combine(self.y_rows.data_ptr(), self.y_rows.stride(0),
                                                      self.route_w.data_ptr(), c.top_k, res, H, res, H,
                                                      L["in_norm"].data_ptr(), None, 0, B, H, c.rms_eps, 0, 0,
                                                      c.terms, self.bn, xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(),
                                                      stream), "moe combine + rms_norm + quant")
            else:
                N.check(lib.ada_rmsnorm_quant(self.hidden.data_ptr(), H, res, H, res, H, L["in_norm"].data_ptr(),
                                              None, 0, B, H, c.rms_eps, 0, 0, c.terms, self.bn, xq.data_ptr(),
                                              sfx.data_ptr(), gx.data_ptr(), stream), "rms_norm+quant")
            ns, ld = self._gemm_parts(self.q_hidden, L["qkv"], "qkv", stream)
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
            ns, ld = self._gemm_parts(self.q_attn, L["o"], "o", stream)
            # x, residual = post_attention_layernorm(o, residual): plain bf16 rows for the router and experts
            rp = self.residual.data_ptr()
            N.check(lib.ada_rmsnorm_quant_parts(self.parts.data_ptr(), ns, B * ld, ld, rp, H, rp, H,
                                                L["post_norm"].data_ptr(), self.xnorm.data_ptr(), H, B, H, c.rms_eps,
                                                0, 0, c.terms, self.bn, None, None, None, stream), "rms_norm")
            self._moe_block(L, stream)
        if fold:
            rp = self.residual.data_ptr()
            N.check(lib.ada_rmsnorm_quant_combine(self.y_rows.data_ptr(), self.y_rows.stride(0),
                                                  self.route_w.data_ptr(), c.top_k, rp, H, rp, H,
                                                  self.final_norm.data_ptr(), self.xnorm.data_ptr(), H, B, H,
                                                  c.rms_eps, 0, 0, c.terms, self.bn, None, None, None, stream),
                    "moe combine + rms_norm")
        else:
            N.check(lib.ada_rmsnorm(self.hidden.data_ptr(), H, self.residual.data_ptr(), H, self.residual.data_ptr(),
                                    H, self.final_norm.data_ptr(), self.xnorm.data_ptr(), H, B, H, c.rms_eps, 0, 0,
                                    stream), "rms_norm")
        self._lm_head(stream)

    def kernels_per_step(self) -> int:
        """Embedding; per layer: RMSNorm+quant, qkv GEMM, q/k-norm+RoPE+store, attention (one kernel
        for short caches, else split + merge+quant), o GEMM, RMSNorm from planes, router GEMM +
        top-k, the
        expert MLP (routing, gathering quantiser, gate_up GEMM, SiLU*up+quant, down GEMM), combine;
        final RMSNorm; lm_head + pick (the expert-parallel all-reduce is NCCL's)."""
        attn = 1 if self.max_pages_per_seq * self.cfg.page_size <= 1024 and self.cfg.hkv <= 8 else 2
        fold = self.cfg.ep_size == 1 and self.fold_combine  # the combine folded into the next RMSNorm
        return 1 + self.cfg.num_layers * (12 + attn - (1 if fold else 0)) + 3

    def export_cpu_weights(self) -> dict:
        if self.cfg.ep_size != 1:
            raise ValueError("CPU weights are exported from an engine holding every expert (ep_size 1)")
        layers = []
        for L in self.layers:
            d = {}
            for name in ("qkv", "o"):
                w = L[name]
                d[name] = (w.packed.cpu(), w.scale.cpu(), float(w.scale_2.item()))
            for name in ("experts_gate_up", "experts_down"):
                w = L[name]
                d[name] = (w.packed.cpu(), w.scale.cpu(), w.scale_2.cpu())
            for name in ("router", "in_norm", "post_norm", "q_norm", "k_norm"):
                d[name] = L[name].cpu()
            layers.append(d)
        return dict(layers=layers, embed=self.embed.cpu(), lm_head=self.lm_head.cpu(),
                    final_norm=self.final_norm.cpu(), cos_sin=self.cos_sin.cpu())
