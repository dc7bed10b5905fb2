"""Attention metadata side channel, field for field the reference's.

nano-vLLM passes the hot path's metadata through a module-level Context
(nanovllm/utils/context.py:5-27) that ModelRunner fills before each forward
(model_runner.py:129-188) and that Attention.forward reads.  This mirror has
the same eight fields and functions, so tests and the benchmark can drive
`Attention` without the reference installed; `integrate.install()` points
`Attention` at the reference's own context instead.
"""
from dataclasses import dataclass

import torch


@dataclass(slots=True)
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


def get_context() -> Context:
    return _CONTEXT


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0,
                slot_mapping=None, context_lens=None, block_tables=None):
    global _CONTEXT
    _CONTEXT = Context(is_prefill, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, slot_mapping,
                       context_lens, block_tables)


def reset_context():
    global _CONTEXT
    _CONTEXT = Context()
