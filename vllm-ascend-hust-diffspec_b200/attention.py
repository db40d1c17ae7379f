"""GQA draft decode attention over the compact working cache.

Replaces the closed ``torch_npu.npu_fused_infer_attention_score`` call of
``_forward_linear_attention_npu`` (diffspec/runtime.py:2079-2134) and the
index_copy / index_select around it: one sm_100a kernel stores the step's new
K/V at each request's local position and attends over positions
``0..position`` of its slot, reading slots through an index vector so
reordered batches copy nothing.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["AttentionWorkspace", "draft_decode_attention"]


class AttentionWorkspace:
    """Split-KV scratch and merge tickets, reused across calls on one device.

    The merge tickets are left at zero by every call, so one workspace may
    serve any number of calls issued in order on a stream; calls that can run
    concurrently on the GPU need separate workspaces.
    """

    def __init__(self, device: torch.device):
        self.device = device
        self.scratch = torch.empty(0, dtype=torch.float32, device=device)
        self.counters = torch.zeros(0, dtype=torch.int32, device=device)

    def ensure(self, scratch_floats: int, counters: int) -> None:
        if self.scratch.numel() < scratch_floats:
            self.scratch = torch.empty(scratch_floats, dtype=torch.float32, device=self.device)
        if self.counters.numel() < counters:
            self.counters = torch.zeros(counters, dtype=torch.int32, device=self.device)


_workspaces: dict[int, AttentionWorkspace] = {}


def _default_workspace(device: torch.device) -> AttentionWorkspace:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None:
        ws = AttentionWorkspace(torch.device("cuda", idx))
        _workspaces[idx] = ws
    return ws


def draft_decode_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    working_key: torch.Tensor,
    working_value: torch.Tensor,
    slots: torch.Tensor,
    positions: torch.Tensor,
    scale: float,
    output: torch.Tensor | None = None,
    *,
    rows: int | None = None,
    position_offset: int = 0,
    num_splits: int | None = None,
    workspace: AttentionWorkspace | None = None,
) -> torch.Tensor:
    """Write K/V at ``p = positions + position_offset``, attend over ``0..p``.

    ``query [n, Hq, D]``, ``key/value [n, Hk, D]``, working caches
    ``[S, Hk, W, D]``, ``slots``/``positions`` int32 ``[rows]``.  Output rows
    ``>= rows`` (graph padding) are zeroed, as the reference's
    ``output.zero_()`` does.
    """
    if query.ndim != 3 or key.ndim != 3 or value.shape != key.shape:
        raise ValueError("query must be [n, Hq, D] and key/value [n, Hk, D]")
    if working_key.ndim != 4 or working_key.shape != working_value.shape:
        raise ValueError("working key/value must have matching 4-D shapes")
    num_slots, num_kv_heads, working_budget, head_dim = working_key.shape
    n, num_query_heads, qd = query.shape
    if qd != head_dim or key.shape[1:] != (num_kv_heads, head_dim):
        raise ValueError("query/key/value head layout does not match the working cache")
    if num_query_heads % num_kv_heads:
        raise ValueError("query heads must be divisible by KV heads")
    if not (query.dtype == key.dtype == value.dtype == working_key.dtype == working_value.dtype):
        raise ValueError("query, key, value and working caches must share a dtype")
    if not (working_key.is_contiguous() and working_value.is_contiguous()):
        raise ValueError("working caches must be contiguous")
    rows = slots.shape[0] if rows is None else rows
    if rows > n or slots.shape[0] < rows or positions.shape[0] < rows:
        raise ValueError("slots/positions must cover the real rows and rows <= n")
    device = _lib.require_cuda(query, key, value, working_key, slots, positions)
    if output is None:
        output = torch.empty_like(query)
    elif output.shape[1:] != query.shape[1:] or output.dtype != query.dtype or not output.is_contiguous():
        raise ValueError("output must be contiguous [n_out, Hq, D] in the query dtype")
    out_rows = output.shape[0]
    if out_rows < rows:
        raise ValueError("output has fewer rows than the batch")
    query = query.contiguous()
    key = key.contiguous()
    value = value.contiguous()
    slots = slots.to(torch.int32).contiguous()
    positions = positions.to(torch.int32).contiguous()
    lib = _lib.load()
    if num_splits is None:
        num_splits = lib.dsb_draft_attention_default_splits(
            rows, num_kv_heads, working_budget, _lib.sm_count(device)
        )
    ws = workspace if workspace is not None else _default_workspace(device)
    ws.ensure(
        lib.dsb_draft_attention_scratch_floats(rows, num_query_heads, num_kv_heads, head_dim, num_splits),
        rows * num_kv_heads,
    )
    _lib.call(
        "dsb_draft_decode_attention",
        _lib.ptr(query),
        _lib.ptr(key),
        _lib.ptr(value),
        _lib.ptr(working_key),
        _lib.ptr(working_value),
        _lib.ptr(slots),
        _lib.ptr(positions),
        int(position_offset),
        rows,
        out_rows,
        num_slots,
        num_query_heads,
        num_kv_heads,
        head_dim,
        working_budget,
        float(scale),
        _lib.dtype_code(query.dtype),
        _lib.ptr(output),
        _lib.ptr(ws.scratch),
        ws.scratch.numel(),
        _lib.ptr(ws.counters),
        num_splits,
        _lib.ptr(_lib.error_flag(device)),
        _lib.stream_ptr(device),
    )
    return output
