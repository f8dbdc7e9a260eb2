"""RMSNorm / GemmaRMSNorm on the B200 kernel (adallm_b200 C ABI ``ada_rmsnorm``).

Same constructor and forward contract as the reference's modules
(adallm/ops/layernorm.py:5-50 and :53-102): ``forward(x)`` returns the
normalised tensor; ``forward(x, residual)`` returns ``(normalised, x + residual)``.
Works on [..., hidden] inputs, including the per-head q/k norms
([T, heads, head_dim], adallm/architectures/qwen3.py:481-483).
"""
from __future__ import annotations

import torch
from torch import nn

from . import _native as N


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
             gemma: bool = False, out: torch.Tensor | None = None, residual_out: torch.Tensor | None = None):
    N.require_cuda(x, weight, residual, what="rms_norm")
    if x.dtype not in N.DT or weight.dtype != x.dtype:
        raise ValueError("rms_norm expects bf16/fp16 input and weight of the same dtype")
    hidden = x.shape[-1]
    x2 = x.reshape(-1, hidden)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    rows = x2.shape[0]
    y = out if out is not None else torch.empty(x.shape, dtype=x.dtype, device=x.device)
    y2 = y.view(-1, hidden)
    if residual is not None:
        r2 = residual.reshape(-1, hidden)
        if r2.stride(-1) != 1:
            r2 = r2.contiguous()
        ro = residual_out if residual_out is not None else torch.empty(residual.shape, dtype=x.dtype, device=x.device)
        ro2 = ro.view(-1, hidden)
        st = N.lib().ada_rmsnorm(x2.data_ptr(), x2.stride(0), r2.data_ptr(), r2.stride(0), ro2.data_ptr(),
                                 ro2.stride(0), weight.data_ptr(), y2.data_ptr(), y2.stride(0), rows, hidden,
                                 float(eps), int(gemma), N.DT[x.dtype], N.stream_ptr(x.device))
        N.check(st, "rms_norm")
        return y, ro
    st = N.lib().ada_rmsnorm(x2.data_ptr(), x2.stride(0), None, 0, None, 0, weight.data_ptr(), y2.data_ptr(),
                             y2.stride(0), rows, hidden, float(eps), int(gemma), N.DT[x.dtype],
                             N.stream_ptr(x.device))
    N.check(st, "rms_norm")
    return y


class RMSNorm(nn.Module):
    """Drop-in for adallm.ops.layernorm.RMSNorm."""

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        return rms_norm(x, self.weight, self.eps, residual, gemma=False)


class GemmaRMSNorm(nn.Module):
    """Drop-in for adallm.ops.layernorm.GemmaRMSNorm (weight stored as w, applied as 1 + w)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.zeros(hidden_size))

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        return rms_norm(x, self.weight, self.eps, residual, gemma=True)
