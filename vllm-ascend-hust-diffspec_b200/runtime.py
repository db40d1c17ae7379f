"""DiffSpec draft-context runtime on B200: the retrieval hook, the per-cycle
compact-cache rebuild and the draft attention, with device-resident state.

Mirrors the hot-path subset of ``DiffSpecDraftCache``
(diffspec/runtime.py:596-2134) for linear (non-tree) Eagle3 proposals:

* ``accept_target_queries`` — the retrieval hook (:1170-1334): committed-query
  pick, rejected-suffix exclusion, chunk scores over the target's paged K,
  the head-sharded exchange and the top-k selection, all on the device.  The
  reference's ``counts.to("cpu")`` sync (:1248) and per-request Python loop
  (:1298-1308) are gone: rows with nothing committed are masked in-kernel.
* ``prepare_compact_prefill`` / ``rebuild`` — ``_history_plan_host`` +
  ``rebuild_compact_kv_from_plan`` (:1683-1765) as one launch that computes
  the plan on the device (no D2H of selections, no host plan upload).
* ``forward_attention`` — the draft attention (:2024-2134) over the working
  cache through a slot vector (no copy for reordered slots).
* ``write_raw`` / ``populate_prefill`` — canonical pre-RoPE KV (:1336-1347,
  :1602-1618); ``capture_raw_kv`` / ``graph_safe_rope_positions`` — the draft
  step's KV sink returning local RoPE positions in a persistent buffer
  (:1767-1877), one launch; ``project_and_write_raw`` — the draft layer's K/V
  projection with the raw write in its epilogue.

Host-visible counters that depend on device data (retrievals run, rows with
nothing committed) live on the device and are read only by
``retrieval_status()``.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from . import _lib
from .attention import AttentionWorkspace, draft_decode_attention
from .compact_kv import rebuild_working_cache
from .kernels import kv_projection_write_raw, paged_chunk_head_scores, paged_decode_attention_lse
from .parallel import gather_head_scores
from .selection import (
    DiffSpecSelection,
    select_context_chunks,
    select_rows,
)

__all__ = [
    "DraftPeriodGraph",
    "DiffSpecSettings",
    "DiffSpecSelection",
    "DiffSpecRuntimeMetrics",
    "DiffSpecDraftCache",
    "causal_row_lengths",
    "chunk_attention_scores",
    "select_context_chunks",
]


@dataclass(frozen=True)
class DiffSpecSettings:
    """Same fields and order as diffspec/runtime.py:18-41."""

    chunk_size: int
    token_budget: int
    retrieval_interval: int
    max_tree_nodes: int
    max_tree_depth: int
    tree_threshold: float
    adaptive_profile: bool


@dataclass
class DiffSpecRuntimeMetrics:
    """Host counters of diffspec/runtime.py:66-116 that need no device data."""

    retrieval_attempts: int = 0
    retrieval_skipped_prefill: int = 0
    retrieval_skipped_no_snapshot: int = 0
    retrieval_skipped_interval: int = 0
    retrieval_launches: int = 0
    retrieval_seconds: float = 0.0


def chunk_attention_scores(
    query: torch.Tensor,
    keys: torch.Tensor,
    chunk_size: int,
    softmax_lse: torch.Tensor | None = None,
    scale: float | None = None,
) -> torch.Tensor:
    """Dense form of the retrieval scores (diffspec/runtime.py:281-345).

    ``query [Hq, D]``, ``keys [T, Hk, D]`` (CUDA) -> ``[ceil(T / C)]`` fp32.
    Runs the paged kernel with the dense keys as one page.
    """
    from .kernels import paged_chunk_attention_scores

    if query.ndim != 2 or keys.ndim != 3:
        raise ValueError("query must be 2-D and keys must be 3-D")
    num_query_heads, head_dim = query.shape
    num_tokens, num_kv_heads, key_head_dim = keys.shape
    if head_dim != key_head_dim:
        raise ValueError("query and key head dimensions must match")
    if num_query_heads % num_kv_heads != 0:
        raise ValueError("query heads must be divisible by KV heads")
    if chunk_size <= 0:
        raise ValueError("chunk_size must be positive")
    device = _lib.require_cuda(query, keys)
    if num_tokens == 0:
        return torch.empty(0, dtype=torch.float32, device=device)
    lse = None if softmax_lse is None else softmax_lse.reshape(1, -1)
    if lse is not None and lse.numel() != num_query_heads:
        raise ValueError("softmax_lse must contain one value per query head")
    scores = paged_chunk_attention_scores(
        query.to(keys.dtype).unsqueeze(0),
        keys.unsqueeze(0),
        lse,
        torch.zeros((1, 1), dtype=torch.int32, device=device),
        torch.tensor([num_tokens], dtype=torch.int32).to(device),
        chunk_size=chunk_size,
        max_seq_len=num_tokens,
        scale=scale if scale is not None else head_dim**-0.5,
    )
    return scores[0]


class _Staging:
    """Device buffer for small per-call int32 vectors from host lists.

    Uploads go through a ring of preallocated pinned host buffers; each slot
    records an event after its asynchronous copy and is reused only once that
    event has completed, so no host synchronisation happens in steady state
    and no pinned memory is allocated per call.  Slot i owns its own region of
    the device buffer, so an upload never overwrites the values of the
    SLOTS - 1 uploads before it, which kernels queued earlier may still read.
    """

    SLOTS = 8

    def __init__(self, device: torch.device, capacity: int):
        self.device = device
        self._alloc(max(1, capacity // self.SLOTS))

    def _alloc(self, per: int) -> None:
        self.per = (per + 1) // 2 * 2  # int32 values per slot (even: uploads start 8-byte aligned)
        self.dev = torch.empty(self.SLOTS * per, dtype=torch.int32, device=self.device)
        self.host = [torch.empty(per, dtype=torch.int32).pin_memory() for _ in range(self.SLOTS)]
        self.events: list[torch.cuda.Event | None] = [None] * self.SLOTS
        self.next = 0

    def upload(self, *lists: list[int]) -> list[torch.Tensor]:
        flat = [v for x in lists for v in x]
        n = len(flat)
        if n > self.per:
            # every queued copy and the kernels before it must be done with
            # the old buffers before they are dropped
            torch.cuda.current_stream(self.device).synchronize()
            self._alloc(2 * n)
        slot = self.next
        self.next = (slot + 1) % self.SLOTS
        ev = self.events[slot]
        if ev is not None:
            ev.synchronize()  # the copy that last used this slot has run
        host = self.host[slot]
        if n:
            host[:n] = torch.tensor(flat, dtype=torch.int32)
        dev = self.dev[slot * self.per: slot * self.per + n]
        dev.copy_(host[:n], non_blocking=True)
        if ev is None:
            ev = torch.cuda.Event()
            self.events[slot] = ev
        ev.record(torch.cuda.current_stream(self.device))
        views, off = [], 0
        for x in lists:
            views.append(dev[off:off + len(x)])
            off += len(x)
        return views


def causal_row_lengths(query_ends: list[int], seq_lens: list[int]) -> tuple[list[int], list[int]]:
    """Visible token count and block-table row of every query row of a
    target pass: request i owns rows ``[query_ends[i-1], query_ends[i])`` (a
    verify span or a prompt) and its j-th of s rows sees the first
    ``seq_lens[i] - (s - 1 - j)`` tokens (causal; at least 0)."""
    if len(query_ends) > len(seq_lens):
        raise ValueError("one seq_lens entry per request span")
    visible, table_rows, start = [], [], 0
    for i, end in enumerate(query_ends):
        span = end - start
        if span < 0:
            raise ValueError("actual_seq_lengths_q must be non-decreasing")
        for j in range(span):
            visible.append(max(0, seq_lens[i] - (span - 1 - j)))
            table_rows.append(i)
        start = end
    return visible, table_rows


class DiffSpecDraftCache:
    """Canonical raw KV and compact attention state for one-layer Eagle3 drafts."""

    def __init__(
        self,
        settings: DiffSpecSettings,
        *,
        max_num_reqs: int,
        max_model_len: int,
        num_kv_heads: int,
        head_dim: int,
        target_num_layers: int,
        dtype: torch.dtype,
        device: torch.device,
        rotary_embedding: Any = None,
        cos_sin_cache: torch.Tensor | None = None,
        rotary_dim: int | None = None,
        is_neox_style: bool = True,
        target_tensor_parallel_size: int = 1,
        process_group: Any = None,
        recent_window: int | None = None,
    ) -> None:
        if target_tensor_parallel_size < 1:
            raise ValueError("Target tensor parallel size must be positive")
        self.settings = settings
        self.max_num_reqs = max_num_reqs
        self.max_model_len = max_model_len
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.target_last_layer = target_num_layers - 1
        self.target_tensor_parallel_size = target_tensor_parallel_size
        self.process_group = process_group
        self.dtype = dtype
        self.device = torch.device(device)
        # diffspec/runtime.py:627-637
        self.history_budget = (
            (settings.token_budget - settings.max_tree_depth - 1)
            // settings.chunk_size
            * settings.chunk_size
        )
        if self.history_budget <= 0:
            raise ValueError("DiffSpec token budget is too small for tree tokens")
        # Rolling recent window (tokens): one chunk is the reference; a longer
        # window (a chunk multiple up to the history budget) is the window
        # mode of selection.select_context_chunks / build_history_plan.
        window = settings.chunk_size if recent_window is None else int(recent_window)
        if (window < settings.chunk_size or window % settings.chunk_size
                or window > self.history_budget):
            raise ValueError("recent_window must be a chunk-size multiple in "
                             "[chunk_size, history_budget]")
        self.recent_window = window
        if rotary_embedding is not None:
            cos_sin_cache = rotary_embedding.cos_sin_cache
            rotary_dim = rotary_embedding.rotary_dim
            is_neox_style = rotary_embedding.is_neox_style
        if cos_sin_cache is None:
            raise ValueError("a RoPE cos/sin cache (or rotary embedding) is required")
        self.cos_sin_cache = cos_sin_cache.to(self.device).contiguous()
        self.rotary_dim = head_dim if rotary_dim is None else rotary_dim
        self.is_neox_style = is_neox_style

        cache_shape = (max_num_reqs, max_model_len, num_kv_heads, head_dim)
        self.raw_key = torch.empty(cache_shape, dtype=dtype, device=self.device)
        self.raw_value = torch.empty_like(self.raw_key)
        working_shape = (max_num_reqs, num_kv_heads, settings.token_budget, head_dim)
        self.working_key = torch.empty(working_shape, dtype=dtype, device=self.device)
        self.working_value = torch.empty_like(self.working_key)

        self.max_selected_chunks = self.history_budget // settings.chunk_size
        self.sel_chunks = torch.zeros(
            (max_num_reqs, self.max_selected_chunks), dtype=torch.int32, device=self.device
        )
        self.sel_count = torch.full((max_num_reqs,), -1, dtype=torch.int32, device=self.device)
        self.working_lens = torch.zeros(max_num_reqs, dtype=torch.int32, device=self.device)
        self._status = torch.zeros(2, dtype=torch.int32, device=self.device)
        self._plan = torch.zeros(
            (max_num_reqs, 5 + settings.token_budget // settings.chunk_size),
            dtype=torch.int64, device=self.device,
        )
        self._history_lens = torch.zeros(max_num_reqs, dtype=torch.int32, device=self.device)
        self._staging = _Staging(self.device, _Staging.SLOTS * (4 * max_num_reqs + 16))
        self._attn_workspace = AttentionWorkspace(self.device)
        self.metrics = DiffSpecRuntimeMetrics()

        if max_num_reqs > 4096:
            raise ValueError("max_num_reqs must be at most 4096 (the device slot table's limit)")
        # Slot table on the device: the key of the request owning each slot,
        # -1 when free.  The host only interns request ids as keys that are
        # never reused (a request that leaves and comes back is a new one, as
        # in the reference, whose released ids lose their slot).
        self._slot_keys = torch.full((max_num_reqs,), -1, dtype=torch.int64, device=self.device)
        self._request_keys: dict[str, int] = {}
        self._next_key = 0
        self._num_active = 0
        self._active_slots_dev: torch.Tensor | None = None
        self._retrieval_cycle = 0
        self._cycle_open = False
        self._draft_step = 0
        self._pending_rows = 0
        self._attn_fast = None  # per-cycle prepared arguments of the draft attention call
        self._rebuild_fast = None  # prepared arguments of the plan + rebuild call
        self._active_ids: list[str] | None = None
        self._position_buffers: dict[torch.dtype, torch.Tensor] = {}
        self._positions_written: dict[torch.dtype, int] = {}
        self._target: dict[str, Any] | None = None
        self.target_is_prefill = True

    # ------------------------------------------------------------ slots
    def set_active_requests(self, request_ids: list[str]) -> None:
        """Keep canonical rows stable across batch reorder and cancellation
        (diffspec/runtime.py:755-778), with the slot table on the device.

        One ``dsb_assign_request_slots`` launch releases the slots of the
        requests that left the batch (their selection and working length
        reset), gives the new requests the lowest free slots in batch order
        and writes the batch's slot vector; the host reads nothing back.  A
        batch of more distinct requests than slots raises RuntimeError after
        the same releases and assignments as the reference's loop (the
        distinct count alone decides it: every kept request already holds a
        slot, so the new ones fit exactly when the batch does)."""
        if self._active_ids is not None and request_ids == self._active_ids:
            return  # same batch in the same order: slots unchanged
        ids = list(request_ids)
        keys: dict[str, int] = {}
        for request_id in ids:
            if request_id not in keys:
                key = self._request_keys.get(request_id)
                if key is None:
                    key = self._next_key
                    self._next_key += 1
                keys[request_id] = key
        n = len(ids)
        if n > 4096:
            raise RuntimeError("DiffSpec canonical request slots are exhausted")
        exhausted = len(keys) > self.max_num_reqs
        slots = torch.empty(n, dtype=torch.int32, device=self.device)
        # int64 keys travel as int32 pairs through the staging ring (every
        # upload starts 8-byte aligned)
        batch_keys = np.asarray([keys[r] for r in ids], dtype=np.int64)
        (pairs,) = self._staging.upload(batch_keys.view(np.int32).tolist())
        _lib.call(
            "dsb_assign_request_slots",
            _lib.ptr(self._slot_keys), self.max_num_reqs, _lib.ptr(pairs.view(torch.int64)), n,
            _lib.ptr(slots), _lib.ptr(self.sel_count), _lib.ptr(self.working_lens), None,
            _lib.ptr(_lib.error_flag(self.device)), _lib.stream_ptr(self.device),
        )
        # the table now holds keys of this batch only
        self._request_keys = keys
        if exhausted:
            self._active_ids = None
            raise RuntimeError("DiffSpec canonical request slots are exhausted")
        self._active_ids = ids
        self._num_active = n
        self._active_slots_dev = slots

    def active_slots(self) -> list[int]:
        """The batch's canonical slots, in batch order (reads the device)."""
        if self._active_slots_dev is None:
            return []
        return [int(x) for x in self._active_slots_dev.tolist()]

    def begin_cycle(self, request_ids: list[str]) -> None:
        self.set_active_requests(request_ids)
        self._cycle_open = True
        self._draft_step = 0
        self._attn_fast = None

    def end_cycle(self) -> None:
        self._cycle_open = False
        self._pending_rows = 0
        self._attn_fast = None

    # ------------------------------------------------------------ retrieval
    def begin_target_forward(self, request_ids: list[str]) -> None:
        """Discard a stale target snapshot before a new verifier pass."""
        self.set_active_requests(request_ids)
        self._target = None
        self.target_is_prefill = True

    def capture_target_attention(
        self,
        query: torch.Tensor,
        softmax_lse: torch.Tensor | None,
        key_cache: torch.Tensor | None,
        metadata: Any,
        scale: float,
    ) -> None:
        """Save the last target layer's attention inputs (runtime.py:841-878).

        ``metadata`` provides ``actual_seq_lengths_q`` (cumulative query ends),
        ``seq_lens_list`` and ``block_tables`` as in vLLM-Ascend.
        """
        if softmax_lse is None or key_cache is None:
            return
        query_ends = list(getattr(metadata, "actual_seq_lengths_q", ()))
        seq_lens = list(getattr(metadata, "seq_lens_list", ()))
        block_tables = getattr(metadata, "block_tables", None)
        if not query_ends or not seq_lens or block_tables is None:
            return
        is_prefill = bool(getattr(metadata, "num_prefills", 1))
        lse = softmax_lse.reshape(query.shape[0], query.shape[1])
        if is_prefill:  # keep only each request's last query (runtime.py:862-872)
            idx = torch.tensor([e - 1 for e in query_ends], dtype=torch.long).to(query.device)
            query = query.index_select(0, idx)
            lse = lse.index_select(0, idx)
            query_ends = list(range(1, len(query_ends) + 1))
        self._target = dict(
            query=query.detach(), lse=lse.detach(), key_cache=key_cache,
            block_tables=block_tables[: len(seq_lens)], query_ends=query_ends,
            seq_lens=seq_lens, scale=scale,
        )
        self.target_is_prefill = is_prefill

    def run_target_attention(
        self,
        query: torch.Tensor,
        key_cache: torch.Tensor,
        value_cache: torch.Tensor,
        metadata: Any,
        scale: float,
    ) -> torch.Tensor:
        """The target verifier's attention with its softmax LSE, captured for
        retrieval: the B200 counterpart of the FIA call with softmax_lse_flag
        whose LSE capture_target_attention keeps (diffspec/ascend_patch.py:
        191-240, runtime.py:841-878).

        ``query [n, Hq, D]`` holds each request's span of query rows in order
        (``metadata.actual_seq_lengths_q``: cumulative ends); the j-th of a
        span of s rows sees the first ``seq_lens_list[i] - (s - 1 - j)``
        tokens of block-table row i (causal, for verify spans and prompts
        alike).  Runs ``paged_decode_attention_lse`` once, stores the query,
        LSE, cache and table through :meth:`capture_target_attention`, and
        returns the attention output ``[n, Hq, D]``.
        """
        query_ends = [int(e) for e in metadata.actual_seq_lengths_q]
        seq_lens = [int(x) for x in metadata.seq_lens_list]
        if query_ends and query_ends[-1] != query.shape[0]:
            raise ValueError("query rows must match actual_seq_lengths_q")
        visible, table_rows = causal_row_lengths(query_ends, seq_lens)
        lens = torch.tensor(visible, dtype=torch.int32).to(self.device)
        rows = torch.tensor(table_rows, dtype=torch.int32).to(self.device)
        out, lse = paged_decode_attention_lse(
            query, key_cache, value_cache, metadata.block_tables, lens, scale=scale,
            max_seq_len=max(seq_lens, default=0), table_rows=rows,
        )
        self.capture_target_attention(query, lse, key_cache, metadata, scale)
        return out

    def accept_target_queries(self, valid_sampled_token_count: torch.Tensor, *, is_prefill: bool) -> None:
        """Retrieve context with the last committed target query per request
        (diffspec/runtime.py:1170-1334)."""
        self.metrics.retrieval_attempts += 1
        if self._target is None:
            self.metrics.retrieval_skipped_no_snapshot += 1
            return
        if is_prefill:
            self.metrics.retrieval_skipped_prefill += 1
            return
        self._retrieval_cycle += 1
        if self._retrieval_cycle % self.settings.retrieval_interval:
            self.metrics.retrieval_skipped_interval += 1
            return
        batch = self._num_active
        t = self._target
        if (
            valid_sampled_token_count.numel() < batch
            or len(t["query_ends"]) < batch
            or len(t["seq_lens"]) < batch
            or t["block_tables"].shape[0] < batch
        ):
            self.metrics.retrieval_skipped_no_snapshot += 1
            return
        self.retrieve(
            t["query"], t["lse"], t["key_cache"], t["block_tables"][:batch],
            t["query_ends"][:batch], t["seq_lens"][:batch],
            valid_sampled_token_count[:batch], t["scale"],
        )

    def retrieve(
        self,
        query: torch.Tensor,
        softmax_lse: torch.Tensor,
        key_cache: torch.Tensor,
        block_tables: torch.Tensor,
        query_ends: list[int],
        target_seq_lens: list[int],
        counts: torch.Tensor,
        scale: float,
    ) -> None:
        """Device retrieval for the active batch: pick -> score -> exchange -> select."""
        if not self._num_active:
            return
        ends_d, seqs_d = self._staging.upload(query_ends, target_seq_lens)
        self.retrieve_device(query, softmax_lse, key_cache, block_tables, ends_d, seqs_d,
                             max(target_seq_lens), counts, scale)

    def retrieve_device(
        self,
        query: torch.Tensor,
        softmax_lse: torch.Tensor,
        key_cache: torch.Tensor,
        block_tables: torch.Tensor,
        query_ends: torch.Tensor,
        target_seq_lens: torch.Tensor,
        max_seq_len: int,
        counts: torch.Tensor,
        scale: float,
    ) -> None:
        """:meth:`retrieve` with the query ends and target lengths already on
        the device (int32 ``[rows]``) and ``max_seq_len`` bounding the
        lengths: no host data is read, so the call can be captured in a CUDA
        graph whose replays see new values in those tensors."""
        started = time.perf_counter()
        rows = self._num_active
        if rows == 0:
            return
        ends_d, seqs_d = query_ends, target_seq_lens
        if ends_d.dtype != torch.int32 or seqs_d.dtype != torch.int32:
            raise ValueError("query_ends and target_seq_lens must be int32 device tensors")
        q_index = torch.empty(rows, dtype=torch.int32, device=self.device)
        r_len = torch.empty_like(q_index)
        r_slot = torch.empty_like(q_index)
        counts = counts.reshape(-1)
        if counts.dtype not in (torch.int32, torch.int64):
            counts = counts.to(torch.int64)
        counts = counts.contiguous()
        _lib.call(
            "dsb_prepare_retrieval_rows",
            _lib.ptr(ends_d), _lib.ptr(seqs_d), _lib.ptr(counts),
            int(counts.dtype == torch.int64), _lib.ptr(self._active_slots_dev), rows,
            _lib.ptr(q_index), _lib.ptr(r_len), _lib.ptr(r_slot), _lib.ptr(self._status),
            _lib.stream_ptr(self.device),
        )
        max_len = int(max_seq_len)
        parts = paged_chunk_head_scores(
            query, key_cache, softmax_lse, block_tables, r_len,
            chunk_size=self.settings.chunk_size, max_seq_len=max_len, scale=scale,
            query_index=q_index,
        )
        total_heads = query.shape[1]
        if self.target_tensor_parallel_size > 1:
            parts = gather_head_scores(parts, self.process_group)
            total_heads *= self.target_tensor_parallel_size
        select_rows(
            parts, r_len, chunk_size=self.settings.chunk_size, token_budget=self.history_budget,
            normalize_heads=total_heads, row_slots=r_slot, sel_chunks=self.sel_chunks,
            sel_count=self.sel_count, recent_window=self.recent_window,
        )
        self.metrics.retrieval_launches += 1
        self.metrics.retrieval_seconds += time.perf_counter() - started

    def set_chunk_scores(self, slot: int, chunk_scores: torch.Tensor, seq_len: int) -> DiffSpecSelection:
        """Select from a score vector and store it for ``slot`` (runtime.py:1554-1567)."""
        selection = select_context_chunks(chunk_scores, seq_len, self.settings.chunk_size,
                                          self.history_budget, recent_window=self.recent_window)
        n = selection.chunk_indices.numel()
        if n:
            self.sel_chunks[slot, :n].copy_(selection.chunk_indices.to(torch.int32))
        self.sel_count[slot] = n
        return selection

    def clear_selection(self, slot: int) -> None:
        self.sel_count[slot] = -1

    def retrieval_status(self) -> dict[str, float | int]:
        """Counters of diffspec/runtime.py:1184-1190 (reads two device ints)."""
        done, no_commit = (int(v) for v in self._status.tolist())
        m = self.metrics
        return dict(
            retrieval_count=done,
            retrieval_attempts=m.retrieval_attempts,
            retrieval_skipped_prefill=m.retrieval_skipped_prefill,
            retrieval_skipped_no_snapshot=m.retrieval_skipped_no_snapshot,
            retrieval_skipped_interval=m.retrieval_skipped_interval,
            retrieval_skipped_no_committed_tokens=no_commit,
            retrieval_ms=m.retrieval_seconds / max(m.retrieval_launches, 1) * 1e3,
            retrieval_cycle=self._retrieval_cycle,
            selected_slots=int((self.sel_count >= 0).sum().item()),
            target_tensor_parallel_size=self.target_tensor_parallel_size,
        )

    # ------------------------------------------------------------ draft cycle
    def write_raw(self, slots: torch.Tensor, positions: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> None:
        """raw[slots[i], positions[i]] = key/value[i] (runtime.py:1602-1618)."""
        n = key.shape[0]
        key = key.reshape(n, -1).contiguous()
        value = value.reshape(n, -1).contiguous()
        _lib.call(
            "dsb_write_raw_kv",
            _lib.ptr(key), _lib.ptr(value), _lib.ptr(self.raw_key), _lib.ptr(self.raw_value),
            _lib.ptr(slots.to(torch.int32).contiguous()),
            _lib.ptr(positions.to(torch.int64).contiguous()), n, self.max_num_reqs,
            self.max_model_len, self.num_kv_heads, self.head_dim, _lib.dtype_code(self.dtype),
            _lib.ptr(_lib.error_flag(self.device)), _lib.stream_ptr(self.device),
        )

    def project_and_write_raw(self, slots: torch.Tensor, positions: torch.Tensor,
                              hidden: torch.Tensor, weight: torch.Tensor,
                              out: torch.Tensor | None = None) -> torch.Tensor:
        """The draft layer's K/V projection (``hidden @ weight.T``, weight rows K
        then V) with the raw-cache write of write_raw in the same launch; returns
        the projected ``[tokens, 2 * Hk * D]`` rows (pre-RoPE)."""
        return kv_projection_write_raw(hidden, weight, slots, positions, self.raw_key,
                                       self.raw_value, out)

    @staticmethod
    def _request_indices(metadata: Any, num_tokens: int) -> list[int]:
        """Batch row of each token of a pass (runtime.py:1580-1595): request i
        owns tokens ``[ends[i-1], ends[i])`` of ``actual_seq_lengths_q`` (or of
        ``query_start_loc``); tokens past the last end stay with the last row."""
        query_ends = getattr(metadata, "actual_seq_lengths_q", None)
        if query_ends:
            starts = [0, *[int(e) for e in query_ends]]
        else:
            starts = [int(x) for x in metadata.query_start_loc.to("cpu").tolist()]
        rows, r = [], 0
        for t in range(num_tokens):
            while r + 1 < len(starts) - 1 and t >= starts[r + 1]:
                r += 1
            rows.append(r)
        return rows

    def _canonical_slots(self, batch_rows: list[int]) -> torch.Tensor:
        """Device slot of each token from its batch row (``dsb_rows_to_slots``)."""
        if not self._num_active:
            raise RuntimeError("DiffSpec request slots have not been initialized")
        if batch_rows and (min(batch_rows) < 0 or max(batch_rows) >= self._num_active):
            raise IndexError("list index out of range")
        (rows_d,) = self._staging.upload(batch_rows)
        slots = torch.empty(len(batch_rows), dtype=torch.int32, device=self.device)
        _lib.call("dsb_rows_to_slots", _lib.ptr(self._active_slots_dev), self._num_active,
                  _lib.ptr(rows_d), len(batch_rows), _lib.ptr(slots),
                  _lib.ptr(_lib.error_flag(self.device)), _lib.stream_ptr(self.device))
        return slots

    def populate_prefill(self, absolute_positions: torch.Tensor, key: torch.Tensor,
                         value: torch.Tensor, metadata: Any) -> None:
        """Canonical raw KV of a cache-only draft projection (runtime.py:1336-1347):
        token t of the pass belongs to the batch row ``metadata`` gives it and
        is written at ``[slot, absolute_positions[t]]``."""
        slots_d = self._canonical_slots(self._request_indices(metadata, key.shape[0]))
        self.write_raw(slots_d, absolute_positions, key, value)

    def capture_raw_kv(self, layer_index: int, absolute_positions: torch.Tensor,
                       key: torch.Tensor, value: torch.Tensor,
                       metadata: Any = None) -> torch.Tensor | None:
        """The draft layer's KV sink (runtime.py:1797-1877, linear proposals).

        Inside a draft cycle the first ``len(active requests)`` rows are the
        requests (later rows are graph padding and write nothing): their
        pre-RoPE K/V go to the raw cache at their absolute positions, and the
        method returns the step's local RoPE positions — history length +
        draft step for those rows, 0 for padding rows — in a persistent
        cache-owned buffer shaped like ``absolute_positions`` (see
        :meth:`graph_safe_rope_positions`).  One launch does both.  The
        step's :meth:`forward_attention` then stores its K/V at the same
        positions.  If the cycle has no rebuilt history yet, ``metadata``'s
        ``seq_lens_list`` drives the rebuild first (the reference's step-0
        path).  Outside a cycle (prefill) the rows map to requests through
        ``metadata`` as in :meth:`populate_prefill` and nothing is returned.
        """
        if layer_index != 0:
            raise ValueError("DiffSpec draft cache only supports one layer")
        if not self._cycle_open:
            if metadata is None:
                return None
            self.populate_prefill(absolute_positions.reshape(-1), key, value, metadata)
            return None
        rows = self._num_active
        flat = absolute_positions.reshape(-1)
        if key.shape[0] < rows or flat.numel() < rows:
            raise RuntimeError("DiffSpec draft tensors omit active request rows")
        if self._pending_rows == 0:
            seq_lens = list(getattr(metadata, "seq_lens_list", ()) or ())
            if not seq_lens:
                return None
            self.rebuild(seq_lens)
        if self._draft_step + 1 > self.settings.token_budget - self.history_budget:
            raise RuntimeError("DiffSpec working cache exhausted")
        if flat.dtype not in (torch.int32, torch.int64):
            raise ValueError("absolute positions must be int32 or int64")
        out = self._position_buffer(flat.dtype, flat.numel())
        k = key.reshape(key.shape[0], -1)
        v = value.reshape(value.shape[0], -1)
        if k.stride(1) != 1 or v.stride(1) != 1 or k.stride(0) != v.stride(0):
            k, v = k.contiguous(), v.contiguous()
        _lib.call(
            "dsb_capture_raw_kv",
            _lib.ptr(k), _lib.ptr(v), k.stride(0), _lib.ptr(self.raw_key), _lib.ptr(self.raw_value),
            _lib.ptr(self._active_slots_dev), _lib.ptr(flat.contiguous()),
            int(flat.dtype == torch.int64), rows, flat.numel(), self.max_num_reqs,
            self.max_model_len, self.num_kv_heads, self.head_dim, _lib.dtype_code(self.dtype),
            _lib.ptr(self._history_lens), self._draft_step, self.settings.token_budget,
            _lib.ptr(out), _lib.ptr(self.working_lens), _lib.ptr(_lib.error_flag(self.device)),
            _lib.stream_ptr(self.device),
        )
        return out.view_as(absolute_positions)

    def _position_buffer(self, dtype: torch.dtype, count: int) -> torch.Tensor:
        """``count`` entries of the persistent position buffer of ``dtype``
        (runtime.py:1767-1794): one allocation of max_num_reqs *
        max_model_len entries per dtype, so the address a captured graph
        holds stays valid; entries past ``count`` that the previous call
        wrote are cleared, the rest of the tail is zero from allocation."""
        buf = self._position_buffers.get(dtype)
        if buf is None:
            buf = torch.zeros(self.max_num_reqs * self.max_model_len, dtype=dtype, device=self.device)
            self._position_buffers[dtype] = buf
        if count > buf.numel():
            raise RuntimeError("DiffSpec RoPE input exceeds its persistent buffer")
        prev = self._positions_written.get(dtype, 0)
        if count < prev:
            buf[count:prev].zero_()
        self._positions_written[dtype] = count
        return buf[:count]

    def graph_safe_rope_positions(self, absolute_positions: torch.Tensor,
                                  local_positions: torch.Tensor | None) -> torch.Tensor:
        """A cache-owned, stable RoPE position input (runtime.py:1767-1794):
        ``local_positions`` when given (e.g. what :meth:`capture_raw_kv`
        returned, which already lives in the buffer), else the absolute
        positions, copied into the persistent buffer of their dtype."""
        src = absolute_positions if local_positions is None else local_positions
        out = self._position_buffer(absolute_positions.dtype, absolute_positions.numel())
        if src.data_ptr() != out.data_ptr():
            out.copy_(src.reshape(-1))
        return out.view_as(absolute_positions)

    def rebuild(self, committed_seq_lens: list[int] | torch.Tensor) -> torch.Tensor:
        """Plan + fused gather/RoPE rebuild of every active row's working cache.

        ``committed_seq_lens`` (host list or device tensor) are the committed
        lengths including the root; history ends just before the root.
        Returns the device int32 ``history_len`` per row, which is also the
        root's local position.
        """
        rows = self._num_active
        if rows == 0:
            return self._history_lens[:0]
        if isinstance(committed_seq_lens, torch.Tensor):
            committed = committed_seq_lens.to(device=self.device, dtype=torch.int32).reshape(-1)[:rows]
        else:
            (committed,) = self._staging.upload(list(committed_seq_lens)[:rows])
        plan = self._plan[:rows]
        hl = self._history_lens[:rows]
        cs = self._cos_sin()
        fast = self._rebuild_fast
        # Every buffer the prepared call below holds a pointer to: rebinding
        # any of them (the caches, the selection state, the slot vector or
        # the cos/sin table) sends the next call through validation again.
        sig = (rows, self._active_slots_dev.data_ptr(), self.raw_key.data_ptr(),
               self.raw_value.data_ptr(), self.working_key.data_ptr(),
               self.working_value.data_ptr(), self.sel_chunks.data_ptr(),
               self.sel_count.data_ptr(), self.working_lens.data_ptr(), plan.data_ptr(),
               hl.data_ptr(), self.raw_key.shape, self.working_key.shape,
               self.sel_chunks.shape, cs.data_ptr(), cs.dtype, cs.shape, cs.stride(0))
        if (fast is not None and fast[0] == sig and committed.dtype == torch.int32
                and committed.is_contiguous() and committed.device == self.device):
            # Same batch, caches and table as a validated call: only the
            # committed lengths change.
            _lib.check(fast[1](*fast[2], committed.data_ptr(), *fast[3], _lib.stream_ptr(self.device)),
                       "dsb_rebuild_working_cache")
        else:
            rebuild_working_cache(
                self.raw_key, self.raw_value, self.working_key, self.working_value,
                self._active_slots_dev, committed, self.sel_chunks, self.sel_count, cs,
                chunk_size=self.settings.chunk_size, history_budget=self.history_budget,
                rotary_dim=self.rotary_dim, is_neox_style=self.is_neox_style, plan=plan,
                history_lens=hl, working_lens=self.working_lens, recent_window=self.recent_window,
            )
            lib = _lib.load()
            head = (self.raw_key.data_ptr(), self.raw_value.data_ptr(), self.working_key.data_ptr(),
                    self.working_value.data_ptr(), self._active_slots_dev.data_ptr())
            tail = (rows, self.sel_chunks.data_ptr(), self.sel_chunks.shape[1],
                    self.sel_count.data_ptr(), self.raw_key.shape[0], self.settings.chunk_size,
                    self.history_budget, self.recent_window, plan.shape[1], plan.data_ptr(),
                    hl.data_ptr(),
                    self.working_lens.data_ptr(), cs.data_ptr(), _lib.dtype_code(cs.dtype),
                    cs.stride(0), cs.shape[0], self.raw_key.shape[1], self.num_kv_heads,
                    self.head_dim, self.working_key.shape[2], self.rotary_dim,
                    int(bool(self.is_neox_style)), _lib.dtype_code(self.raw_key.dtype),
                    _lib.error_flag(self.device).data_ptr())
            self._rebuild_fast = (sig, lib.dsb_rebuild_working_cache, head, tail)
        self._pending_rows = rows
        self._draft_step = 0
        self._attn_fast = None
        return hl

    def prepare_compact_prefill(self, metadata: Any, num_tokens: int, *,
                                committed_seq_lens: list[int] | None = None) -> None:
        """runtime.py:1349-1371: rebuild history at the committed roots."""
        seq_lens = committed_seq_lens if committed_seq_lens is not None else list(
            getattr(metadata, "seq_lens_list", ()))
        if seq_lens is None or len(seq_lens) == 0:
            raise RuntimeError("DiffSpec compact prefill requires sequence lengths")
        self.rebuild(list(seq_lens)[:num_tokens])

    def local_positions(self) -> torch.Tensor:
        """Device local RoPE positions of the current draft step."""
        return self._history_lens[: self._pending_rows] + self._draft_step

    def forward_attention(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                          scale: float, output: torch.Tensor) -> torch.Tensor:
        """One draft step: store K/V at each row's local position and attend
        (runtime.py:2024-2134).  Output rows past the batch are zeroed."""
        rows = self._pending_rows
        if rows == 0:
            raise RuntimeError("DiffSpec attention called without prepared state")
        if self._draft_step + 1 > self.settings.token_budget - self.history_budget:
            raise RuntimeError("DiffSpec working cache exhausted")
        fast = self._attn_fast
        sig = (query.shape, key.shape, value.shape, output.shape, query.dtype, key.dtype,
               value.dtype, output.dtype, query.device, key.device, value.device, output.device,
               float(scale), self.working_key.data_ptr(), self.working_value.data_ptr(),
               self._active_slots_dev.data_ptr(), self._history_lens.data_ptr())
        if (fast is not None and fast[0] == sig and query.is_contiguous() and key.is_contiguous()
                and value.is_contiguous() and output.is_contiguous()):
            # The later steps of a cycle repeat the first step's validated call
            # with new q/k/v/output addresses and the next position offset.
            fn, head, tail = fast[1], fast[2], fast[3]
            _lib.check(
                fn(query.data_ptr(), key.data_ptr(), value.data_ptr(), *head, self._draft_step,
                   *tail[0], output.data_ptr(), *tail[1], _lib.stream_ptr(self.device)),
                "dsb_draft_decode_attention",
            )
        else:
            draft_decode_attention(
                query, key, value, self.working_key, self.working_value,
                self._active_slots_dev, self._history_lens[:rows], scale, output,
                rows=rows, position_offset=self._draft_step, workspace=self._attn_workspace,
            )
            self._attn_fast = self._prepare_attention_fast(sig, query, output, rows, scale)
        self._draft_step += 1
        return output

    def _prepare_attention_fast(self, sig, query, output, rows, scale):
        """Arguments of the C call that stay fixed for the rest of the cycle
        (working caches, slots, history lengths, split scratch), captured after
        draft_decode_attention validated and ran the cycle's first step."""
        if not (query.is_contiguous() and output.is_contiguous()):
            return None
        lib = _lib.load()
        ws = self._attn_workspace
        splits = lib.dsb_draft_attention_default_splits(
            rows, self.num_kv_heads, self.working_key.shape[2], _lib.sm_count(self.device))
        hist = self._history_lens[:rows]
        head = (self.working_key.data_ptr(), self.working_value.data_ptr(),
                self._active_slots_dev.data_ptr(), hist.data_ptr())
        tail = ((rows, output.shape[0], self.working_key.shape[0], query.shape[1],
                 self.num_kv_heads, self.head_dim, self.working_key.shape[2], float(scale),
                 _lib.dtype_code(query.dtype)),
                (ws.scratch.data_ptr(), ws.scratch.numel(), ws.counters.data_ptr(), splits,
                 _lib.error_flag(self.device).data_ptr()))
        return (sig, lib.dsb_draft_decode_attention, head, tail)

    def _cos_sin(self) -> torch.Tensor:
        cs = self.cos_sin_cache
        if cs.dtype != self.dtype and cs.dtype != torch.float32:
            cs = cs.to(self.dtype)
        return cs


class DraftPeriodGraph:
    """One retrieval period of a :class:`DiffSpecDraftCache`, captured once
    as a CUDA graph and replayed per period, host copies included.

    A period is what the runtime's methods do between two retrievals: the
    retrieval hook on the verify pass of the period's first cycle
    (:meth:`DiffSpecDraftCache.retrieve_device`), then
    ``retrieval_interval`` draft cycles, each a plan + rebuild at that
    cycle's committed lengths and ``max_tree_depth`` draft attention steps
    (:meth:`~DiffSpecDraftCache.rebuild`,
    :meth:`~DiffSpecDraftCache.forward_attention`).  Replaying the graph
    replaces those Python calls (about twenty per period), which is the
    reference's per-cycle host work (diffspec/runtime.py:1170-1334,
    1683-1765, 2024-2134) reduced to one launch.

    Inputs are written by the caller into pinned host buffers (``inputs``):
    per cycle the verify pass's query rows, LSE, accepted counts, query ends,
    target lengths and the committed lengths, and per draft step its q/k/v.
    The graph copies the inputs to the device on a side stream in the order
    the period consumes them, as one copy for the first verify block (it
    gates the retrieval) and one per cycle for the rest (the copies of later
    cycles run while earlier cycles compute), and copies every step's
    attention output back into
    ``outputs`` on a second side stream as soon as that step is done.  After
    :meth:`replay` returns, the caller synchronizes (or waits on
    :attr:`done`) before reading ``outputs`` or rewriting ``inputs``.

    The batch (request ids, hence slots), the target's paged K and block
    table, ``max_seq_len`` and the shapes are fixed at capture; lengths,
    counts and every tensor's contents may change between replays.  Host-side
    counters of the cache (``metrics``) do not advance on replay.  Building
    the graph runs one period eagerly on placeholder inputs (zero queries,
    nothing accepted, history length 0), which touches only row 0 of the
    active slots' working caches; the first replay rebuilds them.
    """

    def __init__(self, cache: "DiffSpecDraftCache", request_ids: list[str], *,
                 key_cache: torch.Tensor, block_tables: torch.Tensor,
                 query_rows_per_request: int, num_query_heads: int, max_seq_len: int,
                 scale: float):
        self.cache = cache
        s = cache.settings
        self.interval, self.depth = s.retrieval_interval, s.max_tree_depth
        n = len(request_ids)
        if n == 0:
            raise ValueError("a period graph needs at least one request")
        dev, dt = cache.device, cache.dtype
        hq, hk, d = num_query_heads, cache.num_kv_heads, cache.head_dim
        rq = n * query_rows_per_request
        self.request_ids = list(request_ids)
        self.scale = float(scale)
        self.max_seq_len = int(max_seq_len)
        self.key_cache, self.block_tables = key_cache, block_tables

        # One pinned host buffer and its device twin, packed in the order the
        # period consumes them: [verify block of cycle c][q/k/v of its steps]...
        verify = [("query", (rq, hq, d), dt), ("lse", (rq, hq), torch.float32),
                  ("counts", (n,), torch.int64), ("query_ends", (n,), torch.int32),
                  ("seq_lens", (n,), torch.int32), ("committed", (n,), torch.int32)]
        step = [("q", (n, hq, d), dt), ("k", (n, hk, d), dt), ("v", (n, hk, d), dt)]
        layout, off = [], 0

        def place(spec):
            nonlocal off
            block, start = [], off
            for name, shape, dtype in spec:
                esize = torch.empty((), dtype=dtype).element_size()
                off = (off + 15) // 16 * 16
                nbytes = esize * int(torch.Size(shape).numel())
                block.append((name, shape, dtype, off, nbytes))
                off += nbytes
            return block, start, off

        for c in range(self.interval):
            layout.append(("verify", c, None, *place(verify)))
            for j in range(self.depth):
                layout.append(("step", c, j, *place(step)))
        total = (off + 15) // 16 * 16
        self._host_in = torch.zeros(total, dtype=torch.uint8).pin_memory()
        self._dev_in = torch.zeros(total, dtype=torch.uint8, device=dev)

        def views(buf, block):
            return {name: buf[o:o + nb].view(dtype).view(shape)
                    for name, shape, dtype, o, nb in block}

        self.inputs = {"verify": [None] * self.interval,
                       "step": [[None] * self.depth for _ in range(self.interval)]}
        self._dev = {"verify": [None] * self.interval,
                     "step": [[None] * self.depth for _ in range(self.interval)]}
        # Copies, in order: the first verify block (it gates the retrieval),
        # then one contiguous range per cycle ending with its last step block.
        self._copies = []  # (key, start, end)
        for kind, c, j, block, start, end in layout:
            hv, dv = views(self._host_in, block), views(self._dev_in, block)
            if kind == "verify":
                self.inputs["verify"][c], self._dev["verify"][c] = hv, dv
                if c == 0:
                    self._copies.append(("retrieve", start, end))
                    cycle_start = end
                else:
                    cycle_start = start
            else:
                self.inputs["step"][c][j], self._dev["step"][c][j] = hv, dv
                if j == self.depth - 1:
                    self._copies.append((c, cycle_start, end))
        self.outputs = torch.zeros((self.interval, self.depth, n, hq, d), dtype=dt).pin_memory()
        self._dev_out = torch.zeros((self.interval, self.depth, n, hq, d), dtype=dt, device=dev)
        self.h2d_bytes = int(total)
        self.d2h_bytes = int(self.outputs.numel() * self.outputs.element_size())
        for c in range(self.interval):  # placeholders that keep the first (eager) run in range
            v = self.inputs["verify"][c]
            ends = torch.arange(1, n + 1, dtype=torch.int32) * query_rows_per_request
            v["query_ends"].copy_(ends)
            v["seq_lens"].fill_(min(self.max_seq_len, cache.max_model_len))
            v["committed"].fill_(1)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.done: torch.cuda.Event | None = None
        self._capture()

    def _period(self, main, h2d, d2h) -> None:
        """Enqueue one period: copies on ``h2d`` / ``d2h``, kernels on ``main``."""
        cache = self.cache
        ready = {}
        h2d.wait_stream(main)
        with torch.cuda.stream(h2d):
            for key, start, end in self._copies:
                self._dev_in[start:end].copy_(self._host_in[start:end], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(h2d)
                ready[key] = ev
        d2h.wait_stream(main)
        with torch.cuda.stream(main):
            v0 = self._dev["verify"][0]
            main.wait_event(ready["retrieve"])
            cache.set_active_requests(self.request_ids)
            cache.retrieve_device(v0["query"], v0["lse"], self.key_cache, self.block_tables,
                                  v0["query_ends"], v0["seq_lens"], self.max_seq_len,
                                  v0["counts"], self.scale)
            for c in range(self.interval):
                # One wait per cycle, for the copy that holds its verify
                # block and every step's q/k/v: the kernels of the cycle then
                # follow one another with no copy dependency in between
                # (which would also cut the programmatic launch overlap
                # between them).
                main.wait_event(ready[c])
                cache.begin_cycle(self.request_ids)
                cache.rebuild(self._dev["verify"][c]["committed"])
                for j in range(self.depth):
                    st = self._dev["step"][c][j]
                    cache.forward_attention(st["q"], st["k"], st["v"], self.scale,
                                            self._dev_out[c, j])
                    out_ready = torch.cuda.Event()
                    out_ready.record(main)
                    d2h.wait_event(out_ready)
                    with torch.cuda.stream(d2h):
                        self.outputs[c, j].copy_(self._dev_out[c, j], non_blocking=True)
                cache.end_cycle()
        main.wait_stream(h2d)
        main.wait_stream(d2h)

    def _capture(self) -> None:
        dev = self.cache.device
        main, h2d, d2h = (torch.cuda.Stream(dev) for _ in range(3))
        main.wait_stream(torch.cuda.current_stream(dev))
        self._period(main, h2d, d2h)  # eager run: workspaces, prepared calls
        torch.cuda.current_stream(dev).wait_stream(main)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=main):
            self._period(main, h2d, d2h)
        torch.cuda.synchronize(dev)
        self.done = torch.cuda.Event()

    def replay(self) -> None:
        """Run one period on the current stream (asynchronous): copy the
        pinned inputs in, retrieve, rebuild and attend, copy the outputs
        out.  :attr:`done` is recorded after it."""
        self.graph.replay()
        self.done.record(torch.cuda.current_stream(self.cache.device))

