"""Per-step context, mirroring the reference's nanovllm/utils/context.py.

The GDN layer reads ``cu_seqlens_q``, ``max_seqlen_q``, ``linear_state_ids``
and ``lens_q`` from it (qwen3_5.py:869-881).  The dataclass keeps every field
of the reference's Context, in the same order, so ``set_context`` calls
written for the reference work unchanged.  When the layer is installed into
the reference engine (:func:`layer.install`), it reads the engine's own
context instead of this one.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(slots=True)
class Context:
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    num_decode_tokens: int = 0
    flashinfer_decode: object | None = None
    flashinfer_prefill: object | None = None
    draft_slot_mapping: torch.Tensor | None = None
    draft_block_tables: torch.Tensor | None = None
    # per-sequence recurrent-state slot ids, int64 [bs] on the device
    linear_state_ids: torch.Tensor | None = None
    # host copy of the per-sequence query lengths (avoids a device sync)
    lens_q: list[int] | None = None
    vision_embeds: tuple = ()


_CONTEXT = Context()


def get_context() -> Context:
    return _CONTEXT


def set_context(cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0,
                slot_mapping=None, block_tables=None, num_decode_tokens=0,
                flashinfer_decode=None, flashinfer_prefill=None,
                draft_slot_mapping=None, draft_block_tables=None,
                linear_state_ids=None, lens_q=None, vision_embeds=()):
    global _CONTEXT
    _CONTEXT = Context(cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                       slot_mapping, block_tables, num_decode_tokens,
                       flashinfer_decode, flashinfer_prefill,
                       draft_slot_mapping, draft_block_tables,
                       linear_state_ids, lens_q, vision_embeds)


def reset_context():
    global _CONTEXT
    _CONTEXT = Context()
