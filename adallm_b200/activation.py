"""Gated activations on the B200 kernel (adallm_b200 C ABI ``ada_gated_act``).
Drop-ins for SiluAndMul / GeluAndMul(tanh) (adallm/ops/activation.py:6-26)."""
from __future__ import annotations

import torch
from torch import nn

from . import _native as N


def gated_act(x: torch.Tensor, act: int, out: torch.Tensor | None = None) -> torch.Tensor:
    N.require_cuda(x, what="gated activation")
    if x.dtype not in N.DT:
        raise ValueError("gated activation expects bf16/fp16")
    inter = x.shape[-1] // 2
    x2 = x.reshape(-1, 2 * inter)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    y = out if out is not None else torch.empty(x.shape[:-1] + (inter,), dtype=x.dtype, device=x.device)
    y2 = y.view(-1, inter)
    st = N.lib().ada_gated_act(x2.data_ptr(), x2.stride(0), y2.data_ptr(), y2.stride(0), x2.shape[0], inter, act,
                               N.DT[x.dtype], N.stream_ptr(x.device))
    N.check(st, "gated activation")
    return y


class SiluAndMul(nn.Module):
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return gated_act(x, 0)


class GeluAndMul(nn.Module):
    def __init__(self, approximate: str = "tanh"):
        super().__init__()
        if approximate != "tanh":
            raise ValueError("only the tanh approximation is implemented (the reference's default)")
        self.approximate = approximate

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return gated_act(x, 1)
