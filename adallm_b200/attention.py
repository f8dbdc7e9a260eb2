"""FP8 paged decode attention and FP8 KV-cache store (B200 kernels).

Mirrors the reference interface in adallm/ops/attention.py:
  * store_kvcache(key, value, k_cache, v_cache, slot_mapping)   (:236-251)
  * Attention(num_heads, head_dim, scale, num_kv_heads, sliding_window).forward(q, k, v)
    decode branch (:307-428), reading per-step metadata from the forward context
  * paged_prefill: the prefix-cache prefill branch (:335-358), which the reference runs as
    _gather_kv_from_blocks (:254-286) + flash_attn_varlen_func(causal=True, window=(W, 0));
    here one kernel reads the e4m3 pages in place through the block table.
A prefill without a prefix cache (no block table: the reference attends over the fresh
bf16 K/V with flash-attn) is not part of this package: ``Attention.forward`` raises for it
when used standalone, and ``adallm_b200.install`` keeps the reference's branch for it.
"""
from __future__ import annotations

import torch
from torch import nn

from . import _native as N
from .context import get_context


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor, k_scale: float = 1.0, v_scale: float = 1.0) -> None:
    """k_cache.view(-1, Hkv*D)[slot] = e4m3(key / k_scale) for every slot != -1 (in place)."""
    N.require_cuda(key, value, k_cache, v_cache, slot_mapping, what="store_kvcache")
    n, hkv, d = key.shape
    if key.stride(-1) != 1 or value.stride(-1) != 1 or key.stride(1) != d or value.stride(1) != d:
        raise ValueError("store_kvcache expects [T, Hkv, D] rows with contiguous heads")
    if slot_mapping.numel() != n:
        raise ValueError("slot_mapping must have one entry per token")
    if k_cache.dtype != torch.float8_e4m3fn or v_cache.dtype != torch.float8_e4m3fn:
        raise ValueError("adallm_b200 stores the KV cache as float8_e4m3fn")
    if k_cache.stride(1) != hkv * d or v_cache.stride(1) != hkv * d or k_cache.stride(-1) != 1:
        raise ValueError("KV cache must be laid out [num_pages, page, Hkv, D] with contiguous slots")
    if key.dtype not in N.DT or value.dtype != key.dtype:
        raise ValueError("key/value must be bf16 or fp16")
    slots = slot_mapping if slot_mapping.dtype == torch.int32 else slot_mapping.to(torch.int32)
    st = N.lib().ada_store_kvcache_fp8(key.data_ptr(), value.data_ptr(), N.DT[key.dtype], n, hkv, d,
                                       key.stride(0), value.stride(0), slots.data_ptr(), k_cache.data_ptr(),
                                       v_cache.data_ptr(), hkv * d, float(k_scale), float(v_scale),
                                       N.stream_ptr(key.device))
    N.check(st, "store_kvcache")


def paged_decode_workspace_bytes(batch: int, num_heads: int, max_pages: int, page_size: int, head_dim: int) -> int:
    return int(N.lib().ada_fp8_paged_decode_workspace_size(batch, num_heads, max_pages, page_size, head_dim))


def paged_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                 context_lens: torch.Tensor, scale: float, window: int = 0, k_scale: float = 1.0,
                 v_scale: float = 1.0, out: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention of one query token per sequence against the e4m3 paged cache.

    q [B, Hq, D] bf16/fp16; k_cache/v_cache [num_pages, page, Hkv, D] e4m3;
    block_tables int32 [B, max_pages] (-1 padded); context_lens int32 [B].
    Returns [B, Hq, D] in q.dtype (the reference returns fp16 cast back to q.dtype)."""
    N.require_cuda(q, k_cache, v_cache, block_tables, context_lens, what="paged_decode")
    b, hq, d = q.shape
    _, page, hkv, _ = k_cache.shape
    if q.dtype not in N.DT:
        raise ValueError("q must be bf16 or fp16")
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k_cache.stride() != v_cache.stride() or k_cache.stride(-1) != 1:
        raise ValueError("k_cache and v_cache must share a [pages, page, Hkv, D] layout")
    if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
        raise ValueError("block_tables and context_lens must be int32")
    max_pages = block_tables.shape[1]
    if out is None:
        out = torch.empty((b, hq, d), dtype=q.dtype, device=q.device)
    need = paged_decode_workspace_bytes(b, hq, max_pages, page, d)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    st = N.lib().ada_fp8_paged_decode(
        q.data_ptr(), N.DT[q.dtype], q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(),
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), k_cache.shape[0], block_tables.data_ptr(),
        block_tables.stride(0),
        max_pages, context_lens.data_ptr(), b, hq, hkv, d, page, float(scale), float(k_scale), float(v_scale),
        int(window), out.data_ptr(), N.DT[out.dtype], workspace.data_ptr(), need, N.stream_ptr(q.device))
    N.check(st, "FP8 KV decode kernel")
    return out


def paged_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                  cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor, max_seqlen_q: int, scale: float,
                  window: int = 0, k_scale: float = 1.0, v_scale: float = 1.0, out: torch.Tensor | None = None,
                  err: torch.Tensor | None = None) -> torch.Tensor:
    """Causal prefill attention of the new tokens against the e4m3 paged cache.

    q [total_q, Hq, D] bf16/fp16 (sequence b: rows cu_seqlens_q[b]..cu_seqlens_q[b+1]);
    k_cache/v_cache [num_pages, page, Hkv, D] e4m3 holding every sequence's cached prefix and
    new tokens (store_kvcache runs first); block_tables int32 [B, max_pages] (-1 padded);
    cu_seqlens_q / cu_seqlens_k int32 [B + 1] (the reference's forward-context fields);
    max_seqlen_q must be at least every sequence's new-token count (the grid is sized by it).
    window W > 0: query i sees keys [i + off - W, i + off], off = len_k - len_q.
    Returns [total_q, Hq, D] in q.dtype (the reference returns fp16 cast back to q.dtype).
    err: optional int32 [1] device word; 0x70 is OR-ed in if a tile wait ran out."""
    N.require_cuda(q, k_cache, v_cache, block_tables, cu_seqlens_q, cu_seqlens_k, what="paged_prefill")
    total_q, hq, d = q.shape
    _, page, hkv, _ = k_cache.shape
    if q.dtype not in N.DT:
        raise ValueError("q must be bf16 or fp16")
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k_cache.stride() != v_cache.stride() or k_cache.stride(-1) != 1:
        raise ValueError("k_cache and v_cache must share a [pages, page, Hkv, D] layout")
    if k_cache.dtype != torch.float8_e4m3fn or v_cache.dtype != torch.float8_e4m3fn:
        raise ValueError("the paged prefill reads a float8_e4m3fn cache")
    for t, name in ((block_tables, "block_tables"), (cu_seqlens_q, "cu_seqlens_q"), (cu_seqlens_k, "cu_seqlens_k")):
        if t.dtype != torch.int32:
            raise ValueError(f"{name} must be int32")
    batch = cu_seqlens_q.numel() - 1
    if cu_seqlens_k.numel() != batch + 1 or block_tables.shape[0] < batch:
        raise ValueError("cu_seqlens_q, cu_seqlens_k and block_tables must describe the same sequences")
    if out is None:
        out = torch.empty((total_q, hq, d), dtype=q.dtype, device=q.device)
    if total_q == 0 or batch == 0:
        return out
    st = N.lib().ada_fp8_paged_prefill(
        q.data_ptr(), N.DT[q.dtype], q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(),
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), k_cache.shape[0], block_tables.data_ptr(),
        block_tables.stride(0), block_tables.shape[1], cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), batch,
        int(max_seqlen_q), hq, hkv, d, page, float(scale), float(k_scale), float(v_scale), int(window),
        out.data_ptr(), N.DT[out.dtype], out.stride(0), out.stride(1),
        err.data_ptr() if err is not None else None, N.stream_ptr(q.device))
    N.check(st, "FP8 paged prefill attention")
    return out


class Attention(nn.Module):
    """Drop-in for adallm.ops.attention.Attention (decode branch).

    KV cache views k_cache / v_cache are attached by the runner exactly as the
    reference's ModelRunner.allocate_kv_cache does (adallm/runtime/model_runner.py:154-169)."""

    def __init__(self, num_heads, head_dim, scale, num_kv_heads, sliding_window: int | None = None):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.sliding_window = sliding_window
        self.k_scale = 1.0
        self.v_scale = 1.0
        self.k_cache = self.v_cache = torch.tensor([])

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        context = get_context()
        if context.is_prefill and context.block_tables is None:
            raise NotImplementedError("adallm_b200 runs the prefix-cache prefill and the decode branch; a prefill "
                                      "without a block table stays on the reference path")
        if self.k_cache.numel() and self.v_cache.numel():
            store_kvcache(k, v, self.k_cache, self.v_cache, context.slot_mapping, self.k_scale, self.v_scale)
        window = self.sliding_window if (self.sliding_window is not None and self.sliding_window > 0) else 0
        if context.is_prefill:
            try:
                return paged_prefill(q.view(-1, self.num_heads, self.head_dim), self.k_cache, self.v_cache,
                                     context.block_tables, context.cu_seqlens_q, context.cu_seqlens_k,
                                     context.max_seqlen_q, self.scale, window, self.k_scale, self.v_scale)
            except Exception as exc:
                if torch.cuda.is_current_stream_capturing() or isinstance(exc, ValueError):
                    raise
                raise RuntimeError("FP8 paged prefill kernel failed; no fallback is allowed in this runtime.") from exc
        try:
            return paged_decode(q.view(-1, self.num_heads, self.head_dim), self.k_cache, self.v_cache,
                                context.block_tables, context.context_lens, self.scale, window,
                                self.k_scale, self.v_scale)
        except Exception as exc:
            if torch.cuda.is_current_stream_capturing():
                raise
            if isinstance(exc, ValueError):
                raise
            raise RuntimeError("FP8 KV decode kernel failed; no fallback is allowed in this runtime.") from exc
