"""The reference's Qwen3 decoder layer at decode time on this package's fused kernels.

install() routes adallm.architectures.qwen3.Qwen3DecoderLayer.forward (qwen3.py:1358-1371) here
for decode steps.  Same inputs, parameters, KV cache and forward context as the reference layer,
nine kernels instead of the ~17 of the per-op path:

  input RMSNorm (+ residual add) + activation quantiser     ada_rmsnorm_quant
  qkv projection -> split-K partial planes                  ada_nvfp4_gemm_partials
  q/k RMSNorm + RoPE + FP8 KV store, from the planes        ada_qk_norm_rope_store_parts
  paged decode attention + o_proj operand quantiser         ada_fp8_paged_decode_quant_ex
  o projection -> partial planes                            ada_nvfp4_gemm_partials
  post-attention RMSNorm (+ residual add), from the planes  ada_rmsnorm_quant_parts
  gate_up projection -> partial planes                      ada_nvfp4_gemm_partials
  SiLU(gate) * up + quantiser, from the planes              ada_gated_act_quant_parts
  down projection -> hidden states                          ada_nvfp4_gemm

Every consumer of partial planes sums them in split order and rounds the sum to the model dtype
before its own arithmetic, so the layer computes what the per-op path computes, up to the K-split
order of the GEMMs' fp32 sums.  A step the fused path does not cover returns None and the caller
runs the reference's forward over the per-op replacements: prefill, tensor parallelism, a q/k
bias (no q/k norms), a sliding window, weights that are not NVFP4, shapes outside the kernels'
limits, and a CUDA-graph capture whose batch size was never run eagerly (the working buffers are
sized outside capture: the reference's capture_cudagraph runs each batch size once before it
captures it, model_runner.py:348-352).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as N
from . import nvfp4_gemm

# attention launch flag: context lengths, block tables and every cached K/V row but the newest
# were written at least two kernels earlier (the runner's input copies; the newest row comes from
# the q/k-norm + RoPE + store kernel just before)
_ATTN_META_EARLY = 1

CALLS = 0  # decode steps of a layer that took the fused path (graph captures count once)


@dataclass
class _Linear:
    packed: torch.Tensor
    scale: torch.Tensor
    scale_2: torch.Tensor
    n: int
    k: int

    @property
    def sf(self) -> torch.Tensor:
        return nvfp4_gemm._cached_sf(self.scale, self.n, self.k)


@dataclass
class _Spec:
    hidden: int
    hq: int
    hkv: int
    head_dim: int
    inter: int
    qkv: _Linear
    o: _Linear
    gate_up: _Linear
    down: _Linear


def _nvfp4(mod) -> _Linear | None:
    w = getattr(mod, "weight", None)
    s = getattr(mod, "weight_scale", None)
    s2 = getattr(mod, "weight_scale_2", None)
    if getattr(mod, "bias", None) is not None or not all(isinstance(t, torch.Tensor) for t in (w, s, s2)):
        return None
    if w.dtype != torch.uint8 or w.dim() != 2 or s.dim() != 2 or not w.is_cuda or not s.is_cuda:
        return None
    n, k = w.shape[0], w.shape[1] * 2
    if s.shape[0] != n or s.shape[1] * 16 != k or n % 128 or k % 256 or s2.numel() != 1 or s2.dtype != torch.float32:
        return None
    return _Linear(w, s, s2, n, k)


def _spec(layer) -> _Spec | None:
    """The layer's shapes and NVFP4 weights when the fused path covers it (cached on the layer)."""
    cached = getattr(layer, "_ada_fused_spec", None)
    if cached is not None:
        return cached
    spec = None
    try:
        attn, mlp = layer.self_attn, layer.mlp
        ok = (getattr(attn, "num_heads", 0) == getattr(attn, "total_num_heads", -1)  # TP 1
              and not getattr(attn, "qkv_bias", True) and hasattr(attn, "q_norm") and hasattr(attn, "k_norm")
              and getattr(attn.attn, "sliding_window", None) in (None, 0)
              and type(mlp.act_fn).__name__ == "SiluAndMul")
        lins = [_nvfp4(m) for m in (attn.qkv_proj, attn.o_proj, mlp.gate_up_proj, mlp.down_proj)]
        if ok and all(lins):
            qkv, o, gu, dn = lins
            hidden, d, hq, hkv = layer.input_layernorm.weight.shape[0], attn.head_dim, attn.num_heads, attn.num_kv_heads
            inter = gu.n // 2
            cs = attn.rotary_emb.cos_sin_cache
            if (qkv.k == hidden and qkv.n == (hq + 2 * hkv) * d and o.k == hq * d and o.n == hidden
                    and gu.k == hidden and dn.k == inter and dn.n == hidden and hidden % 256 == 0
                    and inter % 256 == 0 and (hq * d) % 256 == 0 and d == 128 and hq % hkv == 0
                    and cs.dtype == torch.float32 and cs.is_contiguous() and cs.shape[-1] == d):
                spec = _Spec(hidden, hq, hkv, d, inter, qkv, o, gu, dn)
    except Exception:
        spec = None
    if spec is not None:  # a layer not covered now (e.g. weights not yet on the GPU) is asked again
        try:
            layer._ada_fused_spec = spec
        except Exception:
            pass
    return spec


class _NotReady(Exception):
    pass


class _Buffers:
    """Grow-only working memory of one device, shared by every layer (they run in stream order):
    the three quantised GEMM operands, the partial planes, the rotated queries and the GEMM and
    attention workspaces.  Allocated only outside CUDA-graph capture."""

    def __init__(self, device):
        self.device = device
        self.flat: dict[str, torch.Tensor] = {}
        self.splits: dict[tuple, int] = {}

    def get(self, name: str, numel: int, dtype: torch.dtype) -> torch.Tensor:
        t = self.flat.get(name)
        if t is None or t.numel() < numel or t.dtype != dtype:
            if torch.cuda.is_current_stream_capturing():
                raise _NotReady(name)
            t = torch.zeros(max(numel, 64), dtype=dtype, device=self.device)
            self.flat[name] = t
        return t

    def nsplits(self, m: int, n: int, k: int, terms: int) -> int:
        key = (m, n, k, terms)
        ns = self.splits.get(key)
        if ns is None:
            ns = int(N.lib().ada_nvfp4_gemm_splits(m, n, k, terms))
            self.splits[key] = ns
        return ns


_BUFS: dict[int, _Buffers] = {}


def _buffers(device: torch.device) -> _Buffers:
    b = _BUFS.get(device.index)
    if b is None:
        b = _BUFS[device.index] = _Buffers(device)
    return b


def decode_forward(layer, positions: torch.Tensor, hidden_states: torch.Tensor, residual: torch.Tensor | None,
                   ctx) -> tuple[torch.Tensor, torch.Tensor] | None:
    """One decode step of a Qwen3DecoderLayer: (hidden_states, residual) as the reference's
    forward returns them, or None when the fused path does not cover this call."""
    if ctx is None or ctx.is_prefill or ctx.block_tables is None or ctx.context_lens is None \
            or ctx.slot_mapping is None:
        return None
    x = hidden_states
    if x.dim() != 2 or x.dtype not in (torch.bfloat16, torch.float16) or not x.is_cuda or not x.is_contiguous():
        return None
    if residual is not None and (residual.shape != x.shape or residual.dtype != x.dtype
                                 or not residual.is_contiguous()):
        return None
    spec = _spec(layer)
    if spec is None:
        return None
    B, H = x.shape
    attn = layer.self_attn
    kc, vc = attn.attn.k_cache, attn.attn.v_cache
    bt, cl, sm = ctx.block_tables, ctx.context_lens, ctx.slot_mapping
    if (B == 0 or H != spec.hidden or kc.dtype != torch.float8_e4m3fn or vc.dtype != torch.float8_e4m3fn
            or kc.dim() != 4 or kc.shape[2] != spec.hkv or kc.shape[3] != spec.head_dim or kc.stride() != vc.stride()
            or positions.dtype != torch.int64 or positions.numel() != B or sm.dtype != torch.int32
            or sm.numel() != B or cl.dtype != torch.int32 or cl.numel() != B or bt.dtype != torch.int32
            or bt.dim() != 2 or bt.shape[0] != B or bt.stride(1) != 1):
        return None
    lib = N.lib()
    terms = nvfp4_gemm.DEFAULT_TERMS
    dt = N.DT[x.dtype]
    D, hq, hkv, inter = spec.head_dim, spec.hq, spec.hkv, spec.inter
    qn = hq * D
    bn = int(lib.ada_nvfp4_block_n(B, terms))
    m_pad = -(-B // bn) * bn
    page, max_pages = kc.shape[1], bt.shape[1]
    bufs = _buffers(x.device)
    try:
        ops = {}
        for name, k in (("h", H), ("a", qn), ("i", inter)):
            sf_len = (m_pad // bn) * (k // 64) * 512 if terms == 1 else 16
            ops[name] = (bufs.get("xq_" + name, m_pad * terms * k // 2, torch.uint8),
                         bufs.get("sfx_" + name, sf_len, torch.uint8),
                         bufs.get("gx_" + name, m_pad, torch.float32))
        ns = {lin: bufs.nsplits(B, w.n, w.k, terms) for lin, w in
              (("qkv", spec.qkv), ("o", spec.o), ("gate_up", spec.gate_up))}
        planes = bufs.get("planes", max(ns[name] * B * w.n for name, w in
                                        (("qkv", spec.qkv), ("o", spec.o), ("gate_up", spec.gate_up))), torch.float32)
        q_rot = bufs.get("q_rot_" + str(dt), B * qn, x.dtype)
        gemm_ws = bufs.get("gemm_ws", 256, torch.uint8)
        attn_bytes = max(int(lib.ada_fp8_paged_decode_workspace_size(B, hq, max_pages, page, D)), 256)
        attn_ws = bufs.get("attn_ws", attn_bytes, torch.uint8)
    except _NotReady:
        return None
    if min(ns.values()) < 1:
        return None
    s = N.stream_ptr(x.device)
    ln_in, ln_post = layer.input_layernorm, layer.post_attention_layernorm
    qkv, o, gu, dn = spec.qkv, spec.o, spec.gate_up, spec.down

    def gemm_parts(op, w: _Linear, nsp: int):
        xq, sfx, gx = op
        N.check(lib.ada_nvfp4_gemm_partials(xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), B, terms, bn,
                                            w.packed.data_ptr(), w.packed.stride(0), w.sf.data_ptr(),
                                            w.scale_2.data_ptr(), w.n, w.k, planes.data_ptr(), w.n, B * w.n, nsp,
                                            gemm_ws.data_ptr(), gemm_ws.numel(), s), "NVFP4 kernel (partials)")

    # input RMSNorm: residual is the layer input at the first layer, else x + residual (new tensor)
    xq, sfx, gx = ops["h"]
    if residual is None:
        res = x
        N.check(lib.ada_rmsnorm_quant(x.data_ptr(), H, None, 0, None, 0, ln_in.weight.data_ptr(), None, 0, B, H,
                                      float(ln_in.eps), 0, dt, terms, bn, xq.data_ptr(), sfx.data_ptr(),
                                      gx.data_ptr(), s), "rms_norm+quant")
    else:
        res = torch.empty_like(x)
        N.check(lib.ada_rmsnorm_quant(x.data_ptr(), H, residual.data_ptr(), H, res.data_ptr(), H,
                                      ln_in.weight.data_ptr(), None, 0, B, H, float(ln_in.eps), 0, dt, terms, bn,
                                      xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), s), "rms_norm+quant")
    # attention half
    gemm_parts(ops["h"], qkv, ns["qkv"])
    cs = attn.rotary_emb.cos_sin_cache
    N.check(lib.ada_qk_norm_rope_store_parts(planes.data_ptr(), ns["qkv"], B * qkv.n, qkv.n, B, hq, hkv, D,
                                             attn.q_norm.weight.data_ptr(), attn.k_norm.weight.data_ptr(),
                                             float(attn.q_norm.eps), positions.data_ptr(), cs.data_ptr(), cs.shape[0],
                                             sm.data_ptr(), kc.data_ptr(), vc.data_ptr(), 1.0, 1.0, q_rot.data_ptr(),
                                             None, dt, s), "qk_norm_rope_store")
    xq, sfx, gx = ops["a"]
    N.check(lib.ada_fp8_paged_decode_quant_ex(
        q_rot.data_ptr(), dt, qn, D, kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1), kc.stride(2),
        kc.shape[0], bt.data_ptr(), bt.stride(0), max_pages, cl.data_ptr(), B, hq, hkv, D, page,
        float(attn.attn.scale), 1.0, 1.0, 0, None, 0, terms, bn, xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(),
        attn_ws.data_ptr(), attn_ws.numel(), _ATTN_META_EARLY, s), "attention")
    gemm_parts(ops["a"], o, ns["o"])
    # residual + o (rounded) -> the new residual (in place on this call's own residual tensor; at
    # the first layer the residual is the layer input, which stays untouched), post RMSNorm
    res_out = torch.empty_like(x) if res is x else res
    xq, sfx, gx = ops["h"]
    N.check(lib.ada_rmsnorm_quant_parts(planes.data_ptr(), ns["o"], B * H, H, res.data_ptr(), H, res_out.data_ptr(),
                                        H, ln_post.weight.data_ptr(), None, 0, B, H, float(ln_post.eps), 0, dt,
                                        terms, bn, xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), s), "rms_norm+quant")
    res = res_out
    # MLP half
    gemm_parts(ops["h"], gu, ns["gate_up"])
    xq, sfx, gx = ops["i"]
    N.check(lib.ada_gated_act_quant_parts(planes.data_ptr(), ns["gate_up"], B * gu.n, gu.n, None, 0, B, inter, 0, dt,
                                          terms, bn, xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), s),
            "silu_and_mul+quant")
    out = torch.empty_like(x)
    N.check(lib.ada_nvfp4_gemm(xq.data_ptr(), sfx.data_ptr(), gx.data_ptr(), B, terms, bn, dn.packed.data_ptr(),
                               dn.packed.stride(0), dn.sf.data_ptr(), dn.scale_2.data_ptr(), dn.n, dn.k, None,
                               out.data_ptr(), dt, H, 0, gemm_ws.data_ptr(), gemm_ws.numel(), s), "NVFP4 kernel")
    global CALLS
    CALLS += 1
    return out, res
