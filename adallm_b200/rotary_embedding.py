"""Rotary embedding on the B200 kernel (adallm_b200 C ABI ``ada_rope``).

Same constructor, cache and forward contract as the reference
(adallm/ops/rotary_embedding.py:17-90): an fp32 cos/sin cache
[max_position, 1, head_size] = [cos | sin] with optional linear scaling,
NeoX rotate-half applied in fp32 and cast back, new q / k returned.
"""
from __future__ import annotations

from functools import lru_cache

import torch
from torch import nn

from . import _native as N


def build_cos_sin_cache(head_size: int, max_position: int, base: float, rope_scaling: dict | None = None,
                        device=None) -> torch.Tensor:
    """fp32 [max_position, 1, head_size]; same arithmetic as rotary_embedding.py:26-43."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_size, 2, dtype=torch.float) / head_size))
    t = torch.arange(max_position, dtype=torch.float)
    if rope_scaling is not None:
        rope_type = rope_scaling.get("rope_type", rope_scaling.get("type", "linear"))
        if rope_type != "linear":
            raise ValueError(f"Unsupported rope_scaling type: {rope_type}")
        t = t / float(rope_scaling.get("factor", 1.0))
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1)
    return cache if device is None else cache.to(device)


def apply_rope(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor, cos_sin_cache: torch.Tensor,
               q_out: torch.Tensor | None = None, k_out: torch.Tensor | None = None):
    N.require_cuda(positions, query, key, cos_sin_cache, what="rotary_embedding")
    if query.dtype not in N.DT or key.dtype != query.dtype:
        raise ValueError("rotary embedding expects bf16/fp16 q and k")
    d = cos_sin_cache.shape[-1]
    t = positions.numel()
    q3 = query.view(t, -1, d) if query.is_contiguous() else query.reshape(t, -1, d)
    k3 = key.view(t, -1, d) if key.is_contiguous() else key.reshape(t, -1, d)
    if q3.stride(1) != d or k3.stride(1) != d or q3.stride(2) != 1 or k3.stride(2) != 1:
        q3, k3 = q3.contiguous(), k3.contiguous()
    if cos_sin_cache.dtype != torch.float32 or not cos_sin_cache.is_contiguous():
        raise ValueError("cos_sin_cache must be contiguous fp32")
    pos = positions if positions.dtype == torch.int64 else positions.to(torch.int64)
    qo = q_out if q_out is not None else torch.empty(q3.shape, dtype=query.dtype, device=query.device)
    ko = k_out if k_out is not None else torch.empty(k3.shape, dtype=key.dtype, device=key.device)
    st = N.lib().ada_rope(pos.data_ptr(), q3.data_ptr(), q3.stride(0), k3.data_ptr(), k3.stride(0), qo.data_ptr(),
                          ko.data_ptr(), t, q3.shape[1], k3.shape[1], d, cos_sin_cache.data_ptr(),
                          cos_sin_cache.shape[0], N.DT[query.dtype], N.stream_ptr(query.device))
    N.check(st, "rotary_embedding")
    return qo.view(query.shape), ko.view(key.shape)


class RotaryEmbedding(nn.Module):
    """Drop-in for adallm.ops.rotary_embedding.RotaryEmbedding."""

    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int, base: float,
                 rope_scaling: dict | None = None) -> None:
        super().__init__()
        self.head_size = head_size
        assert rotary_dim == head_size
        self.register_buffer("cos_sin_cache", build_cos_sin_cache(head_size, max_position_embeddings, base,
                                                                  rope_scaling), persistent=False)

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor):
        return apply_rope(positions, query, key, self.cos_sin_cache)


@lru_cache(1)
def _get_rope_cached(head_size, rotary_dim, max_position, base, rope_scaling_key):
    rope_scaling = dict(rope_scaling_key) if rope_scaling_key is not None else None
    return RotaryEmbedding(head_size, rotary_dim, max_position, base, rope_scaling=rope_scaling)


def get_rope(head_size: int, rotary_dim: int, max_position: int, base: float, rope_scaling: dict | None = None):
    key = None if rope_scaling is None else tuple(sorted(rope_scaling.items()))
    return _get_rope_cached(head_size, rotary_dim, max_position, base, key)
