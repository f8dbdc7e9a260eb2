"""Mixture-of-experts block pieces on the B200 kernels, restating Qwen3MoeSparseMoeBlock.forward
(adallm/architectures/qwen3.py:1026-1032 and the expert loop after it):

    ids, w = route_topk(router_logits, top_k, norm_topk_prob)   # softmax fp32, top-k, renormalise
    h = nvfp4_linear_gather(x.repeat_interleave(top_k, 0), ...)  # grouped NVFP4 GEMM per routed row
    out = combine(h, w, top_k)                                   # sum of the k expert rows, weighted
"""
from __future__ import annotations

import torch

from . import _native as N


def route_topk(router_logits: torch.Tensor, top_k: int, norm_topk_prob: bool = True):
    """(expert ids int32 [T, top_k], routing weights [T, top_k] in the logits' dtype)."""
    N.require_cuda(router_logits, what="route_topk")
    lg = router_logits if router_logits.dtype in (torch.bfloat16, torch.float16) else router_logits.to(torch.bfloat16)
    if lg.stride(-1) != 1:
        lg = lg.contiguous()
    t, e = lg.shape
    ids = torch.empty((t, top_k), dtype=torch.int32, device=lg.device)
    w = torch.empty((t, top_k), dtype=lg.dtype, device=lg.device)
    st = N.lib().ada_moe_route_topk(lg.data_ptr(), N.DT[lg.dtype], lg.stride(0), t, e, top_k, int(norm_topk_prob),
                                    ids.data_ptr(), w.data_ptr(), N.stream_ptr(lg.device))
    N.check(st, "moe route")
    return ids, w


def combine(expert_out: torch.Tensor, weights: torch.Tensor, top_k: int) -> torch.Tensor:
    """[T * top_k, H] expert rows (row t*top_k + j = token t's j-th expert) -> [T, H]."""
    N.require_cuda(expert_out, weights, what="moe combine")
    y = expert_out if expert_out.stride(-1) == 1 else expert_out.contiguous()
    rows, h = y.shape
    t = rows // top_k
    w = weights.to(y.dtype).reshape(-1).contiguous()
    out = torch.empty((t, h), dtype=y.dtype, device=y.device)
    st = N.lib().ada_moe_combine(y.data_ptr(), N.DT[y.dtype], y.stride(0), w.data_ptr(), t, top_k, h, out.data_ptr(),
                                 out.stride(0), N.stream_ptr(y.device))
    N.check(st, "moe combine")
    return out
