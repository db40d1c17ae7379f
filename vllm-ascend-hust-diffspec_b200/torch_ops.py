"""The operator surface registered as PyTorch custom ops (``torch.ops.diffspec_b200.*``).

The reference runs inside vLLM's PIECEWISE ``torch.compile`` graphs and
registers its draft-KV sink as a custom op so the compiled graph holds it as
an opaque node (diffspec/vllm_patch.py:130-162, ``direct_register_custom_op``
with a fake implementation, split at that op).  The same holds here for every
entry point of the path: each op below is a ``torch.library.custom_op`` whose
real implementation is the package function over ``libdiffspec_b200.so`` and
whose fake implementation gives output shapes and dtypes for tracing, with
the in-place working-cache writes declared in ``mutates_args`` so functional
graphs order them correctly.

==========================================  =========================================
op                                          reference
==========================================  =========================================
``paged_chunk_attention_scores``            diffspec/kernels.py:95-150
``gather_raw_kv_with_local_rope``           diffspec/kernels.py:153-210
``rebuild_compact_kv_from_plan``            diffspec/compact_kv.py:184-242
``rebuild_working_cache``                   diffspec/runtime.py:1737-1765 (plan + rebuild)
``draft_decode_attention``                  diffspec/runtime.py:2079-2134 (the FIA call)
``capture_raw_kv``                          diffspec/vllm_patch.py:132-147 (the KV sink)
==========================================  =========================================

``capture_raw_kv`` acts on the runtime registered with :func:`set_active_runtime`
(the reference looks its runtime up the same way, ``_active_runtime()``); with
none registered it returns a copy of the positions, as the reference does.
"""

from __future__ import annotations

import torch

from . import attention as _attention
from . import compact_kv as _compact_kv
from . import kernels as _kernels

__all__ = ["set_active_runtime", "active_runtime", "NAMESPACE"]

NAMESPACE = "diffspec_b200"
_active = None


def set_active_runtime(runtime) -> None:
    """The DiffSpecDraftCache that ``capture_raw_kv`` writes to (None: none)."""
    global _active
    _active = runtime


def active_runtime():
    return _active


# ---------------------------------------------------------------- retrieval scores
@torch.library.custom_op(f"{NAMESPACE}::paged_chunk_attention_scores", mutates_args=())
def paged_chunk_attention_scores(query: torch.Tensor, key_cache: torch.Tensor,
                                 softmax_lse: torch.Tensor | None, block_table: torch.Tensor,
                                 seq_lens: torch.Tensor, chunk_size: int, max_seq_len: int,
                                 scale: float) -> torch.Tensor:
    return _kernels.paged_chunk_attention_scores(
        query, key_cache, softmax_lse, block_table, seq_lens, chunk_size=chunk_size,
        max_seq_len=max_seq_len, scale=scale)


@paged_chunk_attention_scores.register_fake
def _(query, key_cache, softmax_lse, block_table, seq_lens, chunk_size, max_seq_len, scale):
    chunks = (max_seq_len + chunk_size - 1) // chunk_size
    return query.new_empty((query.shape[0], chunks), dtype=torch.float32)


# ---------------------------------------------------------------- paged gather + RoPE
@torch.library.custom_op(f"{NAMESPACE}::gather_raw_kv_with_local_rope", mutates_args=())
def gather_raw_kv_with_local_rope(raw_key_cache: torch.Tensor, raw_value_cache: torch.Tensor,
                                  block_table: torch.Tensor, selected_token_indices: torch.Tensor,
                                  cos_sin_cache: torch.Tensor, rope_dim: int,
                                  is_neox_style: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    return _kernels.gather_raw_kv_with_local_rope(
        raw_key_cache, raw_value_cache, block_table, selected_token_indices, cos_sin_cache,
        rope_dim=rope_dim, is_neox_style=is_neox_style)


@gather_raw_kv_with_local_rope.register_fake
def _(raw_key_cache, raw_value_cache, block_table, selected_token_indices, cos_sin_cache, rope_dim,
      is_neox_style=True):
    b, w = selected_token_indices.shape
    shape = (b, w, raw_key_cache.shape[2], raw_key_cache.shape[3])
    return raw_key_cache.new_empty(shape), raw_value_cache.new_empty(shape)


# ---------------------------------------------------------------- compact rebuild
@torch.library.custom_op(f"{NAMESPACE}::rebuild_compact_kv_from_plan",
                         mutates_args=("working_key", "working_value"))
def rebuild_compact_kv_from_plan(raw_key: torch.Tensor, raw_value: torch.Tensor,
                                 working_key: torch.Tensor, working_value: torch.Tensor,
                                 plan: torch.Tensor, cos_sin_cache: torch.Tensor, chunk_size: int,
                                 max_width: int, rotary_dim: int, is_neox_style: bool) -> None:
    _compact_kv.rebuild_compact_kv_from_plan(
        raw_key, raw_value, working_key, working_value, plan, cos_sin_cache,
        chunk_size=chunk_size, max_width=max_width, rotary_dim=rotary_dim,
        is_neox_style=is_neox_style)


@rebuild_compact_kv_from_plan.register_fake
def _(raw_key, raw_value, working_key, working_value, plan, cos_sin_cache, chunk_size, max_width,
      rotary_dim, is_neox_style):
    return None


@torch.library.custom_op(f"{NAMESPACE}::rebuild_working_cache",
                         mutates_args=("working_key", "working_value", "plan", "history_lens",
                                       "working_lens"))
def rebuild_working_cache(raw_key: torch.Tensor, raw_value: torch.Tensor,
                          working_key: torch.Tensor, working_value: torch.Tensor,
                          row_slots: torch.Tensor, committed_lens: torch.Tensor,
                          sel_chunks: torch.Tensor, sel_count: torch.Tensor,
                          cos_sin_cache: torch.Tensor, plan: torch.Tensor,
                          history_lens: torch.Tensor, working_lens: torch.Tensor,
                          chunk_size: int, history_budget: int, rotary_dim: int,
                          is_neox_style: bool, recent_window: int = 0) -> None:
    _compact_kv.rebuild_working_cache(
        raw_key, raw_value, working_key, working_value, row_slots, committed_lens, sel_chunks,
        sel_count, cos_sin_cache, chunk_size=chunk_size, history_budget=history_budget,
        rotary_dim=rotary_dim, is_neox_style=is_neox_style, plan=plan, history_lens=history_lens,
        working_lens=working_lens, recent_window=recent_window or None)


@rebuild_working_cache.register_fake
def _(raw_key, raw_value, working_key, working_value, row_slots, committed_lens, sel_chunks,
      sel_count, cos_sin_cache, plan, history_lens, working_lens, chunk_size, history_budget,
      rotary_dim, is_neox_style, recent_window=0):
    return None


# ---------------------------------------------------------------- draft attention
@torch.library.custom_op(f"{NAMESPACE}::draft_decode_attention",
                         mutates_args=("working_key", "working_value", "output"))
def draft_decode_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                           working_key: torch.Tensor, working_value: torch.Tensor,
                           slots: torch.Tensor, positions: torch.Tensor, scale: float,
                           output: torch.Tensor, rows: int, position_offset: int = 0) -> None:
    _attention.draft_decode_attention(query, key, value, working_key, working_value, slots,
                                      positions, scale, output, rows=rows,
                                      position_offset=position_offset)


@draft_decode_attention.register_fake
def _(query, key, value, working_key, working_value, slots, positions, scale, output, rows,
      position_offset=0):
    return None


# ---------------------------------------------------------------- the KV sink
@torch.library.custom_op(f"{NAMESPACE}::capture_raw_kv", mutates_args=())
def capture_raw_kv(positions: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   layer_index: int) -> torch.Tensor:
    runtime = _active
    if runtime is None:
        return positions.clone()
    local = runtime.capture_raw_kv(layer_index, positions, key, value)
    # a view of the runtime's persistent position buffer: a stable address
    # for graph replays (it aliases no input of the op)
    return runtime.graph_safe_rope_positions(positions, local)


@capture_raw_kv.register_fake
def _(positions, key, value, layer_index):
    return torch.empty_like(positions)
