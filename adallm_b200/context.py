"""Per-step attention metadata, the same contract as the reference's global
forward context (adallm/infra/context.py:5-45): ``slot_mapping``,
``context_lens``, ``block_tables`` and ``is_prefill``.  When adallm_b200 is
installed into the reference runtime, ``get_context`` reads the reference's
own context instead (see ``adallm_b200.install``)."""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class Context:
    is_prefill: bool = False
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None


_CONTEXT = Context()
_PROVIDER = None


def get_context() -> Context:
    if _PROVIDER is not None:
        return _PROVIDER()
    return _CONTEXT


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0,
                slot_mapping=None, context_lens=None, block_tables=None) -> None:
    global _CONTEXT
    _CONTEXT = Context(is_prefill, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, slot_mapping,
                       context_lens, block_tables)


def reset_context() -> None:
    global _CONTEXT
    _CONTEXT = Context()


def use_context_provider(fn) -> None:
    """Route get_context() to another runtime's context getter (None restores the local one)."""
    global _PROVIDER
    _PROVIDER = fn
