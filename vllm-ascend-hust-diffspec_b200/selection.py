"""Device chunk selection and compact history plans.

``select_context_chunks`` is the drop-in for diffspec/runtime.py:348-414
(same arguments, same ``DiffSpecSelection`` result, same ``ValueError``s) and
``select_rows`` is its batched, host-sync-free form used by the retrieval hook.
``build_history_plan`` replaces the per-row host loop ``_history_plan_host``
(diffspec/runtime.py:1713-1735) and the plan upload of
``_rebuild_working_cache_batched`` (:1737-1765).

Tie rule: equal scores are ranked by ascending chunk index, so the selection
is a pure function of the scores (torch.topk does not specify tie order).

Rolling recent window: ``recent_window`` (tokens, a chunk-size multiple; None
= one chunk, the reference) sets the length of the plan's rolling tail.  The
window mode (more than one chunk) has no reference counterpart: the newest
``recent_window / C`` chunks are then left out of the ranking, since the tail
holds them, and ``(token_budget - recent_window) / C`` ranked chunks plus the
newest are kept.
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


def _check_window(recent_window: int | None, chunk_size: int, budget: int) -> int:
    """The window in tokens (chunk_size when None), validated."""
    if recent_window is None:
        return chunk_size
    if recent_window < chunk_size or recent_window % chunk_size or recent_window > budget:
        raise ValueError("recent_window must be a chunk-size multiple in [chunk_size, budget]")
    return int(recent_window)


def select_context_chunks(
    chunk_scores: torch.Tensor,
    seq_len: int,
    chunk_size: int,
    token_budget: int,
    *,
    recent_window: int | None = None,
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
    window = _check_window(recent_window, chunk_size, token_budget)
    device = _lib.require_cuda(chunk_scores)
    if num_chunks == 0:
        empty = torch.empty(0, dtype=torch.long, device=device)
        return DiffSpecSelection(empty, empty, chunk_scores)
    max_chunks = token_budget // chunk_size
    count = num_chunks if num_chunks <= max_chunks else max_chunks - window // chunk_size + 1
    seq = torch.tensor([seq_len], dtype=torch.int32).to(device, non_blocking=True)
    chunk_idx, token_idx, scores = select_rows(
        chunk_scores.reshape(1, 1, -1).to(torch.float32),
        seq,
        chunk_size=chunk_size,
        token_budget=token_budget,
        normalize_heads=0,
        with_outputs=True,
        recent_window=window,
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
    recent_window: int | None = None,
):
    """Batched selection over ``parts [rows, P, N]`` (summed over P in order),
    or over ``parts [world, rows, P / world, N]`` — the all-gathered per-rank
    parts of head-sharded ranks, read in place (part p of a row is rank
    p // (P / world)'s local part p % (P / world)).

    With ``normalize_heads > 0`` the summed mass is divided by the chunk's
    valid token count and ``normalize_heads`` first (the head mean of
    diffspec/kernels.py:150).  When ``sel_chunks``/``sel_count`` are given,
    rows whose ``row_slots`` entry is >= 0 overwrite that slot's selection.
    Returns ``(chunk_indices, token_indices, chunk_scores)`` (-1 padded) when
    ``with_outputs``; nothing is copied to the host.
    """
    device = _lib.require_cuda(parts, seq_lens)
    if parts.ndim not in (3, 4) or parts.dtype != torch.float32 or parts.stride(-1) != 1:
        raise ValueError("parts must be fp32 [rows, parts, chunks] (or [world, rows, parts, "
                         "chunks]) with unit chunk stride")
    if token_budget < chunk_size or token_budget % chunk_size != 0:
        raise ValueError("token_budget must be a positive chunk-size multiple")
    window = _check_window(recent_window, chunk_size, token_budget)
    if parts.ndim == 4:
        world, rows, per_group, max_chunks = parts.shape
        num_parts, group_stride = world * per_group, parts.stride(0)
        row_stride, part_stride = parts.stride(1), parts.stride(2)
    else:
        rows, num_parts, max_chunks = parts.shape
        per_group, group_stride = num_parts, 0
        row_stride, part_stride = parts.stride(0), parts.stride(1)
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
        row_stride,
        part_stride,
        num_parts,
        per_group,
        group_stride,
        int(normalize_heads),
        _lib.ptr(seq_lens),
        _lib.ptr(row_slots),
        rows,
        max_chunks,
        chunk_size,
        token_budget,
        window,
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
    recent_window: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Plan rows ``[slot, history_len, tail_start, prefix_len, prefix_drop, chunks...]``.

    ``history_end = max(0, committed_len - 1)`` excludes the root being
    replayed; ``sel_count[slot] < 0`` means the slot has no retrieval yet
    (most recent ``history_budget`` tokens).  The rolling tail holds the last
    ``min(recent_window, history_budget)`` history tokens (one chunk when
    None, the reference).  Returns ``(plan, history_lens)``.
    """
    window = _check_window(recent_window, chunk_size, history_budget)
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
        window,
        width,
        _lib.ptr(plan),
        _lib.ptr(history_lens),
        _lib.ptr(working_lens),
        _lib.ptr(_lib.error_flag(device)),
        _lib.stream_ptr(device),
    )
    return plan, history_lens
