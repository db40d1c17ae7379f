"""Device chunk selection and compact history plans.

``select_context_chunks`` is the drop-in for diffspec/runtime.py:348-414
(same arguments, same ``DiffSpecSelection`` result, same ``ValueError``s) and
``select_rows`` is its batched, host-sync-free form used by the retrieval hook.
``build_history_plan`` replaces the per-row host loop ``_history_plan_host``
(diffspec/runtime.py:1713-1735) and the plan upload of
``_rebuild_working_cache_batched`` (:1737-1765).

Tie rule: equal scores are ranked by ascending chunk index, so the selection
is a pure function of the scores (torch.topk does not specify tie order).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib

__all__ = [
    "DiffSpecSelection",
    "select_context_chunks",
    "select_rows",
    "build_history_plan",
    "history_budget",
]


@dataclass(frozen=True)
class DiffSpecSelection:
    chunk_indices: torch.Tensor
    token_indices: torch.Tensor
    chunk_scores: torch.Tensor


def history_budget(token_budget: int, max_tree_depth: int, chunk_size: int) -> int:
    """``(token_budget - depth - 1) // C * C`` (diffspec/runtime.py:627-635)."""
    return (token_budget - max_tree_depth - 1) // chunk_size * chunk_size


def select_context_chunks(
    chunk_scores: torch.Tensor,
    seq_len: int,
    chunk_size: int,
    token_budget: int,
) -> DiffSpecSelection:
    """Select top scoring chunks while always retaining the newest chunk."""
    # diffspec/runtime.py:355-367
    if chunk_scores.ndim != 1:
        raise ValueError("chunk_scores must be one-dimensional")
    if seq_len < 0:
        raise ValueError("seq_len must be non-negative")
    if token_budget < chunk_size or token_budget % chunk_size != 0:
        raise ValueError("token_budget must be a positive chunk-size multiple")
    num_chunks = (seq_len + chunk_size - 1) // chunk_size
    if num_chunks != chunk_scores.numel():
        raise ValueError("chunk score count does not match sequence length")
    device = _lib.require_cuda(chunk_scores)
    if num_chunks == 0:
        empty = torch.empty(0, dtype=torch.long, device=device)
        return DiffSpecSelection(empty, empty, chunk_scores)
    max_chunks = token_budget // chunk_size
    count = min(num_chunks, max_chunks)
    seq = torch.tensor([seq_len], dtype=torch.int32).to(device, non_blocking=True)
    chunk_idx, token_idx, scores = select_rows(
        chunk_scores.reshape(1, 1, -1).to(torch.float32),
        seq,
        chunk_size=chunk_size,
        token_budget=token_budget,
        normalize_heads=0,
        with_outputs=True,
    )
    n_tokens = (count - 1) * chunk_size + (seq_len - (num_chunks - 1) * chunk_size)
    return DiffSpecSelection(
        chunk_indices=chunk_idx[0, :count],
        token_indices=token_idx[0, :n_tokens],
        chunk_scores=scores[0, :count].to(chunk_scores.dtype),
    )


def select_rows(
    parts: torch.Tensor,
    seq_lens: torch.Tensor,
    *,
    chunk_size: int,
    token_budget: int,
    normalize_heads: int,
    row_slots: torch.Tensor | None = None,
    sel_chunks: torch.Tensor | None = None,
    sel_count: torch.Tensor | None = None,
    with_outputs: bool = False,
):
    """Batched selection over ``parts [rows, P, N]`` (summed over P in order).

    With ``normalize_heads > 0`` the summed mass is divided by the chunk's
    valid token count and ``normalize_heads`` first (the head mean of
    diffspec/kernels.py:150).  When ``sel_chunks``/``sel_count`` are given,
    rows whose ``row_slots`` entry is >= 0 overwrite that slot's selection.
    Returns ``(chunk_indices, token_indices, chunk_scores)`` (-1 padded) when
    ``with_outputs``; nothing is copied to the host.
    """
    device = _lib.require_cuda(parts, seq_lens)
    if parts.ndim != 3 or parts.dtype != torch.float32 or parts.stride(2) != 1:
        raise ValueError("parts must be fp32 [rows, parts, chunks] with unit chunk stride")
    if token_budget < chunk_size or token_budget % chunk_size != 0:
        raise ValueError("token_budget must be a positive chunk-size multiple")
    rows, num_parts, max_chunks = parts.shape
    s = token_budget // chunk_size
    seq_lens = seq_lens.to(torch.int32).contiguous()
    outs = (None, None, None)
    if with_outputs:
        outs = (
            torch.empty((rows, s), dtype=torch.int64, device=device),
            torch.empty((rows, s * chunk_size), dtype=torch.int64, device=device),
            torch.empty((rows, s), dtype=torch.float32, device=device),
        )
    if row_slots is not None:
        row_slots = row_slots.to(torch.int32).contiguous()
    _lib.call(
        "dsb_select_context_chunks",
        _lib.ptr(parts),
        parts.stride(0),
        parts.stride(1),
        num_parts,
        int(normalize_heads),
        _lib.ptr(seq_lens),
        _lib.ptr(row_slots),
        rows,
        max_chunks,
        chunk_size,
        token_budget,
        _lib.ptr(sel_chunks),
        sel_chunks.shape[1] if sel_chunks is not None else 0,
        _lib.ptr(sel_count),
        sel_count.shape[0] if sel_count is not None else 0,
        _lib.ptr(outs[0]),
        _lib.ptr(outs[1]),
        _lib.ptr(outs[2]),
        _lib.ptr(_lib.error_flag(device)),
        _lib.stream_ptr(device),
    )
    return outs if with_outputs else None


def build_history_plan(
    row_slots: torch.Tensor,
    committed_lens: torch.Tensor,
    sel_chunks: torch.Tensor,
    sel_count: torch.Tensor,
    *,
    chunk_size: int,
    history_budget: int,
    working_budget: int,
    plan: torch.Tensor | None = None,
    history_lens: torch.Tensor | None = None,
    working_lens: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Plan rows ``[slot, history_len, tail_start, prefix_len, prefix_drop, chunks...]``.

    ``history_end = max(0, committed_len - 1)`` excludes the root being
    replayed; ``sel_count[slot] < 0`` means the slot has no retrieval yet
    (most recent ``history_budget`` tokens).  Returns ``(plan, history_lens)``.
    """
    device = _lib.require_cuda(row_slots, committed_lens, sel_chunks, sel_count)
    rows = row_slots.shape[0]
    width = 5 + working_budget // chunk_size
    if plan is None:
        plan = torch.empty((rows, width), dtype=torch.int64, device=device)
    if history_lens is None:
        history_lens = torch.empty(rows, dtype=torch.int32, device=device)
    if plan.shape != (rows, width) or plan.dtype != torch.int64 or not plan.is_contiguous():
        raise ValueError("plan must be contiguous int64 [rows, 5 + working_budget // chunk_size]")
    _lib.call(
        "dsb_build_history_plan",
        _lib.ptr(row_slots),
        _lib.ptr(committed_lens),
        rows,
        _lib.ptr(sel_chunks),
        sel_chunks.shape[1],
        _lib.ptr(sel_count),
        sel_count.shape[0],
        chunk_size,
        history_budget,
        width,
        _lib.ptr(plan),
        _lib.ptr(history_lens),
        _lib.ptr(working_lens),
        _lib.ptr(_lib.error_flag(device)),
        _lib.stream_ptr(device),
    )
    return plan, history_lens
