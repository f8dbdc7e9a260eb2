"""Mixture-of-experts block pieces on the B200 kernels, restating Qwen3MoeSparseMoeBlock.forward
(adallm/architectures/qwen3.py:1026-1032 and the expert loop after it):

    ids, w = route_topk(router_logits, top_k, norm_topk_prob)   # softmax fp32, top-k, renormalise
    h = nvfp4_linear_gather(x.repeat_interleave(top_k, 0), ...)  # grouped NVFP4 GEMM per routed row
    out = combine(h, w, top_k)                                   # sum of the k expert rows, weighted

Expert parallelism (beyond the reference, which runs MoE at TP = 1 only, qwen3.py:1383): each
rank holds a contiguous block of experts (expert_shard), moe_block_ep computes that block's
share and sums the ranks' shares with one all-reduce.
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


def combine(expert_out: torch.Tensor, weights: torch.Tensor, top_k: int, expert_ids: torch.Tensor | None = None,
            expert_base: int = 0, num_local: int | None = None, fp32: bool = False) -> torch.Tensor:
    """[T * top_k, H] expert rows (row t*top_k + j = token t's j-th expert) -> [T, H].

    With expert_ids (expert parallelism) only the slots whose expert is in
    [expert_base, expert_base + num_local) are summed: this rank's share of the block output,
    returned unrounded in fp32 when fp32 is set (sum the ranks' shares in fp32, then round once)."""
    N.require_cuda(expert_out, weights, what="moe combine")
    y = expert_out if expert_out.stride(-1) == 1 else expert_out.contiguous()
    rows, h = y.shape
    t = rows // top_k
    w = weights.to(y.dtype).reshape(-1).contiguous()
    if fp32 and expert_ids is None:
        raise ValueError("fp32 output is the expert-parallel share; pass expert_ids")
    out = torch.empty((t, h), dtype=torch.float32 if fp32 else y.dtype, device=y.device)
    if expert_ids is None:
        st = N.lib().ada_moe_combine(y.data_ptr(), N.DT[y.dtype], y.stride(0), w.data_ptr(), t, top_k, h,
                                     out.data_ptr(), out.stride(0), N.stream_ptr(y.device))
    else:
        ids = expert_ids.to(device=y.device, dtype=torch.int32).reshape(-1).contiguous()
        if ids.numel() != t * top_k or num_local is None:
            raise ValueError("expert_ids must have top_k entries per token, and num_local must be given")
        fn = N.lib().ada_moe_combine_ep_f32 if fp32 else N.lib().ada_moe_combine_ep
        st = fn(y.data_ptr(), N.DT[y.dtype], y.stride(0), w.data_ptr(), ids.data_ptr(), int(expert_base),
                int(num_local), t, top_k, h, out.data_ptr(), out.stride(0), N.stream_ptr(y.device))
    N.check(st, "moe combine")
    return out


def expert_shard(num_experts: int, world: int, rank: int) -> tuple[int, int]:
    """(first expert, expert count) of `rank` when num_experts are split over `world` ranks in
    contiguous, equal blocks (num_experts must divide evenly)."""
    if world <= 0 or not 0 <= rank < world or num_experts % world:
        raise ValueError("experts must split evenly over the ranks")
    per = num_experts // world
    return rank * per, per


def moe_block_ep(x: torch.Tensor, router_logits: torch.Tensor, top_k: int, norm_topk_prob: bool,
                 gate_up: tuple, down: tuple, expert_base: int, group=None) -> torch.Tensor:
    """One MoE block with this rank's experts: route (the same on every rank), the grouped gate+up
    GEMM over the rows routed here, SiLU(gate) * up, the grouped down GEMM, the weighted sum of the
    local slots, then (with a process group) the sum over the ranks: fp32 shares, one fp32
    all-reduce, one rounding to x's dtype.

    x [T, H]; router_logits [T, E_total]; gate_up = (packed [E, 2I, H/2], scale [E, 2I, H/16],
    scale_2 [E]) with gate rows first; down = (packed [E, H, I/2], scale [E, H, I/16], scale_2 [E]);
    E = this rank's experts, starting at expert_base."""
    from .activation import gated_act
    from .nvfp4_gemm import nvfp4_linear_gather
    ids, w = route_topk(router_logits, top_k, norm_topk_prob)
    flat = ids.reshape(-1)
    xr = x.repeat_interleave(top_k, 0)
    h = nvfp4_linear_gather(xr, gate_up[0], gate_up[1], gate_up[2], flat, 16, expert_base=expert_base)
    # rows routed to other ranks hold stale values; the down GEMM and the combine never read them
    a = gated_act(h, 0)
    y = nvfp4_linear_gather(a, down[0], down[1], down[2], flat, 16, expert_base=expert_base)
    share = combine(y, w, top_k, expert_ids=ids, expert_base=expert_base, num_local=gate_up[0].shape[0],
                    fp32=group is not None)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(share, group=group)
        share = share.to(x.dtype)
    return share
