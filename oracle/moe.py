"""MoE routing restated on the CPU (test infrastructure only).

Qwen3MoeSparseMoeBlock.forward, adallm/architectures/qwen3.py:1026-1032:
    routing_weights = softmax(router_logits, dim=1, dtype=float32)
    routing_weights, selected_experts = topk(routing_weights, top_k)
    if norm_topk_prob: routing_weights /= routing_weights.sum(-1, keepdim=True)
    routing_weights = routing_weights.to(hidden_states.dtype)
"""
from __future__ import annotations

import torch


def route_topk(router_logits: torch.Tensor, top_k: int, norm_topk_prob: bool = True, dtype=None):
    """(expert ids int64 [T, top_k] in descending weight order, weights [T, top_k] in `dtype`
    (default: the logits' dtype)).  Equal weights are ordered by the lower expert (torch.topk
    leaves their order unspecified; a stable descending sort fixes it)."""
    w = torch.softmax(router_logits.float(), dim=1, dtype=torch.float32)
    w, ids = torch.sort(w, dim=-1, descending=True, stable=True)
    w, ids = w[:, :top_k], ids[:, :top_k]
    if norm_topk_prob:
        w = w / w.sum(dim=-1, keepdim=True)
    return ids, w.to(dtype or router_logits.dtype)
