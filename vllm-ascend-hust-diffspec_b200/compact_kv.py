"""Fused raw KV gather and local-position RoPE (drop-in for ``diffspec.compact_kv``).

``rebuild_compact_kv_from_plan`` keeps the signature, plan contract and
``ValueError`` conditions of diffspec/compact_kv.py:136-242; the kernel is the
sm_100a ``rope_bulk_kernel`` in ``libdiffspec_b200.so``.
``rebuild_working_cache`` is the reference's whole
``_rebuild_working_cache_batched`` (diffspec/runtime.py:1737-1765: host plan,
plan upload, rebuild) as one launch that computes the plan on the device.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["rebuild_compact_kv_from_plan", "rebuild_working_cache"]


def _validate_compact_inputs(
    raw_key: torch.Tensor,
    raw_value: torch.Tensor,
    working_key: torch.Tensor,
    working_value: torch.Tensor,
    plan: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    *,
    max_width: int,
    rotary_dim: int,
) -> None:
    """The checks of diffspec/compact_kv.py:136-181, in the same order."""
    if raw_key.ndim != 4 or raw_key.shape != raw_value.shape:
        raise ValueError("raw key/value must have matching 4-D shapes")
    if working_key.ndim != 4 or working_key.shape != working_value.shape:
        raise ValueError("working key/value must have matching 4-D shapes")
    slots, max_model_len, heads, head_dim = raw_key.shape
    if (
        working_key.shape[0] != slots
        or working_key.shape[1] != heads
        or working_key.shape[3] != head_dim
    ):
        raise ValueError("working cache slot, head and head dimensions must match raw KV")
    if min(max_model_len, heads, head_dim) <= 0:
        raise ValueError("raw sequence, head and head dimensions must be positive")
    if plan.ndim != 2 or plan.dtype != torch.int64:
        raise ValueError("KV plan must be a contiguous 2-D int64 tensor")
    if plan.shape[0] > slots or not 0 <= max_width <= working_key.shape[2]:
        raise ValueError("KV plan exceeds the working cache batch or token capacity")
    if rotary_dim < 0 or rotary_dim > head_dim or rotary_dim % 2:
        raise ValueError("rotary_dim must be even and between zero and head_dim")
    if (
        cos_sin_cache.ndim != 2
        or cos_sin_cache.shape[0] < max_width
        or cos_sin_cache.shape[1] < rotary_dim
        or cos_sin_cache.stride(1) != 1
    ):
        raise ValueError("cos/sin cache must contain all local positions and rotary dimensions")
    caches = (raw_key, raw_value, working_key, working_value)
    if any(not cache.is_contiguous() for cache in (*caches, plan)):
        raise ValueError("raw KV, working KV and plan must be contiguous")
    if any(cache.dtype != raw_key.dtype for cache in caches):
        raise ValueError("all KV caches must have the same dtype")
    if raw_key.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise ValueError("KV caches must use BF16, FP16 or FP32")
    if any(tensor.device != raw_key.device for tensor in (*caches, plan, cos_sin_cache)):
        raise ValueError("KV caches, plan and cos/sin cache must share a device")


def rebuild_compact_kv_from_plan(
    raw_key: torch.Tensor,
    raw_value: torch.Tensor,
    working_key: torch.Tensor,
    working_value: torch.Tensor,
    plan: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    *,
    chunk_size: int,
    max_width: int,
    rotary_dim: int,
    is_neox_style: bool,
) -> None:
    """Rebuild compact KV from fixed-capacity per-request chunk plans.

    A plan row contains ``[slot, history_len, tail_start, prefix_len,
    prefix_drop, chunk_ids...]`` (width ``5 + working_budget // chunk_size``).
    For local position ``p < history_len`` the source position is
    ``chunk_ids[(p + prefix_drop) // C] * C + (p + prefix_drop) % C`` when
    ``p < prefix_len`` and ``tail_start + p - prefix_len`` otherwise; K is
    rotated at ``p`` (fp32 math), V and K dims past ``rotary_dim`` are copied.
    Slots must be distinct across rows; positions past ``history_len`` are left
    untouched; ``max_width`` bounds the launch and nothing is copied to the
    host.  Device-side index errors are recorded in the library's error flag
    instead of faulting.
    """
    _validate_compact_inputs(
        raw_key, raw_value, working_key, working_value, plan, cos_sin_cache,
        max_width=max_width, rotary_dim=rotary_dim,
    )
    if chunk_size <= 0 or plan.shape[1] != 5 + working_key.shape[2] // chunk_size:
        raise ValueError("plan width must be 5 + working_budget // chunk_size")
    if not plan.shape[0] or not max_width:
        return
    device = _lib.require_cuda(raw_key, plan)
    slots, max_model_len, heads, head_dim = raw_key.shape
    _lib.call(
        "dsb_rebuild_compact_kv_from_plan",
        _lib.ptr(raw_key),
        _lib.ptr(raw_value),
        _lib.ptr(working_key),
        _lib.ptr(working_value),
        _lib.ptr(plan),
        plan.shape[0],
        plan.shape[1],
        _lib.ptr(cos_sin_cache),
        _lib.dtype_code(cos_sin_cache.dtype),
        cos_sin_cache.stride(0),
        cos_sin_cache.shape[0],
        slots,
        max_model_len,
        heads,
        head_dim,
        working_key.shape[2],
        chunk_size,
        max_width,
        rotary_dim,
        int(bool(is_neox_style)),
        _lib.dtype_code(raw_key.dtype),
        _lib.ptr(_lib.error_flag(device)),
        _lib.stream_ptr(device),
    )


def rebuild_working_cache(
    raw_key: torch.Tensor,
    raw_value: torch.Tensor,
    working_key: torch.Tensor,
    working_value: torch.Tensor,
    row_slots: torch.Tensor,
    committed_lens: torch.Tensor,
    sel_chunks: torch.Tensor,
    sel_count: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    *,
    chunk_size: int,
    history_budget: int,
    rotary_dim: int,
    is_neox_style: bool,
    plan: torch.Tensor | None = None,
    history_lens: torch.Tensor | None = None,
    working_lens: torch.Tensor | None = None,
    recent_window: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """History plan + working-cache rebuild of every row in one launch.

    Row ``r`` uses slot ``row_slots[r]`` with committed length
    ``committed_lens[r]`` (the root included; history ends before it) and the
    slot's selection ``sel_chunks[slot, :sel_count[slot]]`` (count < 0: no
    retrieval yet).  The plan rows, ``history_lens`` and ``working_lens`` come
    out exactly as ``selection.build_history_plan`` computes them, and the
    working cache exactly as ``rebuild_compact_kv_from_plan`` of that plan
    leaves it.  ``recent_window`` is the rolling tail's length
    (``selection.build_history_plan``; one chunk when None).  Returns
    ``(plan, history_lens)``.
    """
    working_budget = working_key.shape[2]
    rows = row_slots.shape[0]
    if chunk_size <= 0:
        raise ValueError("plan width must be 5 + working_budget // chunk_size")
    width = 5 + working_budget // chunk_size
    device = _lib.require_cuda(raw_key, row_slots, committed_lens, sel_chunks, sel_count)
    if plan is None:
        plan = torch.empty((rows, width), dtype=torch.int64, device=device)
    if history_lens is None:
        history_lens = torch.empty(rows, dtype=torch.int32, device=device)
    _validate_compact_inputs(
        raw_key, raw_value, working_key, working_value, plan, cos_sin_cache,
        max_width=history_budget, rotary_dim=rotary_dim,
    )
    if plan.shape != (rows, width):
        raise ValueError("plan must be contiguous int64 [rows, 5 + working_budget // chunk_size]")
    for t in (row_slots, committed_lens, sel_chunks, sel_count, history_lens):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError("slots, lengths and selection state must be contiguous int32")
    if working_lens is not None and (working_lens.dtype != torch.int32 or not working_lens.is_contiguous()):
        raise ValueError("working_lens must be contiguous int32")
    if rows == 0:
        return plan, history_lens
    slots, max_model_len, heads, head_dim = raw_key.shape
    _lib.call(
        "dsb_rebuild_working_cache",
        _lib.ptr(raw_key),
        _lib.ptr(raw_value),
        _lib.ptr(working_key),
        _lib.ptr(working_value),
        _lib.ptr(row_slots),
        _lib.ptr(committed_lens),
        rows,
        _lib.ptr(sel_chunks),
        sel_chunks.shape[1],
        _lib.ptr(sel_count),
        slots,
        chunk_size,
        history_budget,
        0 if recent_window is None else int(recent_window),
        width,
        _lib.ptr(plan),
        _lib.ptr(history_lens),
        _lib.ptr(working_lens),
        _lib.ptr(cos_sin_cache),
        _lib.dtype_code(cos_sin_cache.dtype),
        cos_sin_cache.stride(0),
        cos_sin_cache.shape[0],
        max_model_len,
        heads,
        head_dim,
        working_budget,
        rotary_dim,
        int(bool(is_neox_style)),
        _lib.dtype_code(raw_key.dtype),
        _lib.ptr(_lib.error_flag(device)),
        _lib.stream_ptr(device),
    )
    return plan, history_lens
