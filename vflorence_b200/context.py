"""Per-step metadata read by the attention custom ops (mirror of vflorence/utils/context.py:1-30).

One forward at a time: the context is a module global set once per decode step, as in the
reference. The engine puts device tensors in it, and its ``cross_staged`` entries carry the
grouped ``query_start_loc`` of the beams (see ``attention.stage_cross``). The reference's own
form - host tensors built by its ``ModelRunner._prepare`` and 5-tuple cross staging - is also
taken: the ops upload host metadata inside the call.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(slots=True)
class Context:
    context_lens: torch.Tensor | None = None     # int32 [B] (device, or host in the reference's form)
    block_tables: torch.Tensor | None = None     # int32 [B, max_blocks], zero padded
    slot_mapping: torch.Tensor | None = None     # int64 [B]
    query_start_loc: torch.Tensor | None = None  # int32 [B + 1]
    self_metadata: torch.Tensor | None = None    # host plan (paged_ops.get_scheduler_metadata)
    isa: str | None = None
    cross_staged: list | None = None             # per layer: (k, v, table, lens, metadata[, qsl])
    # beam search: runs of consecutive rows at one position (the beams of a request) attend as
    # one group with per-row block tables (self_metadata is then a row-tables plan)
    self_groups: torch.Tensor | None = None      # int32 [G + 1], device: row offsets of the groups
    self_group_lens: torch.Tensor | None = None  # int32 [G], device: each group's context length
    # whether self_metadata takes the fused KV append (asked once per step, not once per layer)
    self_append: bool | None = None


_CONTEXT: Context | None = None


def get_context() -> Context:
    """The active step's Context (None outside a forward)."""
    return _CONTEXT


def set_context(**fields) -> None:
    """Set the global Context for the current forward; no arguments resets it."""
    global _CONTEXT
    _CONTEXT = Context(**fields)
