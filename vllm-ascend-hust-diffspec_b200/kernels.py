"""Retrieval scoring and paged gather+RoPE ops (drop-in for ``diffspec.kernels``).

Same names, positional order, keyword-only arguments and ``ValueError``
conditions as ``diffspec/kernels.py`` of vllm-ascend-hust-diffspec 0.3.0; the
work runs in hand-written sm_100a kernels behind ``libdiffspec_b200.so``.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = [
    "paged_chunk_attention_scores",
    "paged_chunk_head_scores",
    "paged_chunk_stats",
    "stats_to_head_scores",
    "finalize_chunk_scores",
    "gather_raw_kv_with_local_rope",
    "kv_projection_write_raw",
    "qkv_projection_write_raw",
    "paged_decode_attention_lse",
]


def _validate_scores(query, key_cache, softmax_lse, block_table, seq_lens, query_index=None):
    """diffspec/kernels.py:107-120; with ``query_index`` the batch is the
    number of mapped rows and query/LSE may hold more token rows."""
    if query.ndim != 3:
        raise ValueError("query must have shape [batch, query_heads, head_dim]")
    if key_cache.ndim != 4:
        raise ValueError("key_cache must have shape [blocks, block_size, kv_heads, head_dim]")
    query_rows, num_query_heads, head_dim = query.shape
    batch_size = query_rows if query_index is None else query_index.numel()
    _, block_size, num_kv_heads, key_head_dim = key_cache.shape
    if head_dim != key_head_dim:
        raise ValueError("query and key head dimensions must match")
    if num_query_heads % num_kv_heads != 0:
        raise ValueError("query heads must be divisible by KV heads")
    if softmax_lse is not None and softmax_lse.numel() != query_rows * num_query_heads:
        raise ValueError("softmax_lse must contain one value per query head")
    if query.dtype != key_cache.dtype:
        raise ValueError("query and key_cache must share a dtype")
    if block_table.ndim != 2 or block_table.shape[0] < batch_size:
        raise ValueError("block_table must have one row per request")
    if seq_lens.numel() < batch_size:
        raise ValueError("seq_lens must have one entry per request")


def _prep_index(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    return t


def _batch(query, query_index):
    return query.shape[0] if query_index is None else query_index.numel()


def paged_chunk_head_scores(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    softmax_lse: torch.Tensor | None,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    *,
    chunk_size: int,
    max_seq_len: int,
    scale: float,
    query_index: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Per-(request, kv head, chunk) attention mass ``[B, Hk, ceil(max_seq_len/C)]``.

    ``out[b, g, c] = sum_{h in group g} sum_{t in chunk c, t < seq_lens[b]}
    exp(scale * q[b, h] . k[b, t, g] - lse[b, h])``, the unnormalised per-head
    sums of diffspec/kernels.py:71-83 grouped by kv head.  With
    ``softmax_lse=None`` the log-sum-exp over each request's whole sequence is
    computed on the device first (diffspec/runtime.py:321-322).
    """
    _validate_scores(query, key_cache, softmax_lse, block_table, seq_lens, query_index)
    if chunk_size <= 0:
        raise ValueError("chunk_size must be positive")
    device = _lib.require_cuda(query, key_cache, block_table, seq_lens)
    _, num_query_heads, head_dim = query.shape
    batch_size = _batch(query, query_index)
    num_blocks, block_size, num_kv_heads, _ = key_cache.shape
    max_chunks = (max_seq_len + chunk_size - 1) // chunk_size
    if out is None:
        out = torch.empty((batch_size, num_kv_heads, max_chunks), dtype=torch.float32, device=device)
    elif out.shape != (batch_size, num_kv_heads, max_chunks) or out.dtype != torch.float32:
        raise ValueError("out must be fp32 [batch, kv_heads, max_chunks]")
    if batch_size == 0 or max_chunks == 0:
        return out
    query = query.contiguous()
    key_cache = key_cache.contiguous()
    block_table = _prep_index(block_table)
    if block_table.stride(1) != 1:
        block_table = block_table.contiguous()
    seq_lens = _prep_index(seq_lens).contiguous()
    if query_index is not None:
        query_index = _prep_index(query_index).contiguous()
    dtype = _lib.dtype_code(key_cache.dtype)
    stream = _lib.stream_ptr(device)
    flag = _lib.error_flag(device)
    common = (
        _lib.ptr(block_table),
        block_table.stride(0),
        block_table.shape[1],
        _lib.ptr(seq_lens),
        batch_size,
        num_query_heads,
        num_kv_heads,
        head_dim,
        block_size,
        num_blocks,
        chunk_size,
        max_chunks,
        float(scale),
        dtype,
    )
    if softmax_lse is not None:
        lse = softmax_lse.reshape(-1, num_query_heads).to(torch.float32).contiguous()
        _lib.call(
            "dsb_paged_chunk_head_scores",
            _lib.ptr(query),
            _lib.ptr(lse),
            _lib.ptr(query_index),
            query.shape[0],
            _lib.ptr(key_cache),
            *common,
            _lib.ptr(out),
            _lib.ptr(flag),
            stream,
        )
        return out
    cmax, csum = paged_chunk_stats(
        query, key_cache, block_table, seq_lens, chunk_size=chunk_size, max_seq_len=max_seq_len,
        scale=scale, query_index=query_index,
    )
    stats_to_head_scores(cmax, csum, seq_lens, num_kv_heads, chunk_size=chunk_size, out=out)
    return out


def paged_chunk_stats(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    *,
    chunk_size: int,
    max_seq_len: int,
    scale: float,
    query_index: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-(request, query head, chunk) ``(max, sum)`` of the chunk's logits.

    ``max`` is in log2 units (``log2(e) * scale * q.k``); ``sum`` is the sum of
    ``exp(logit - max_logit)`` over the chunk's valid tokens.
    """
    _validate_scores(query, key_cache, None, block_table, seq_lens, query_index)
    device = _lib.require_cuda(query, key_cache, block_table, seq_lens)
    _, num_query_heads, head_dim = query.shape
    batch_size = _batch(query, query_index)
    num_blocks, block_size, num_kv_heads, _ = key_cache.shape
    max_chunks = (max_seq_len + chunk_size - 1) // chunk_size
    cmax = torch.empty((batch_size, num_query_heads, max_chunks), dtype=torch.float32, device=device)
    csum = torch.empty_like(cmax)
    if batch_size == 0 or max_chunks == 0:
        return cmax, csum
    query = query.contiguous()
    key_cache = key_cache.contiguous()
    block_table = _prep_index(block_table)
    if block_table.stride(1) != 1:
        block_table = block_table.contiguous()
    seq_lens = _prep_index(seq_lens).contiguous()
    if query_index is not None:
        query_index = _prep_index(query_index).contiguous()
    _lib.call(
        "dsb_paged_chunk_stats",
        _lib.ptr(query),
        _lib.ptr(query_index),
        query.shape[0],
        _lib.ptr(key_cache),
        _lib.ptr(block_table),
        block_table.stride(0),
        block_table.shape[1],
        _lib.ptr(seq_lens),
        batch_size,
        num_query_heads,
        num_kv_heads,
        head_dim,
        block_size,
        num_blocks,
        chunk_size,
        max_chunks,
        float(scale),
        _lib.dtype_code(key_cache.dtype),
        _lib.ptr(cmax),
        _lib.ptr(csum),
        _lib.ptr(_lib.error_flag(device)),
        _lib.stream_ptr(device),
    )
    return cmax, csum


def stats_to_head_scores(
    chunk_max: torch.Tensor,
    chunk_sum: torch.Tensor,
    seq_lens: torch.Tensor,
    num_kv_heads: int,
    *,
    chunk_size: int,
    out: torch.Tensor | None = None,
    lse_out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Fold chunk statistics into per-kv-head mass with the sequence-wide LSE."""
    device = _lib.require_cuda(chunk_max, chunk_sum, seq_lens)
    batch_size, num_query_heads, max_chunks = chunk_max.shape
    if out is None:
        out = torch.empty((batch_size, num_kv_heads, max_chunks), dtype=torch.float32, device=device)
    seq_lens = _prep_index(seq_lens).contiguous()
    _lib.call(
        "dsb_chunk_stats_to_head_scores",
        _lib.ptr(chunk_max.contiguous()),
        _lib.ptr(chunk_sum.contiguous()),
        _lib.ptr(seq_lens),
        batch_size,
        num_query_heads,
        num_kv_heads,
        chunk_size,
        max_chunks,
        _lib.ptr(out),
        _lib.ptr(lse_out),
        _lib.stream_ptr(device),
    )
    return out


def finalize_chunk_scores(
    parts: torch.Tensor,
    seq_lens: torch.Tensor,
    *,
    chunk_size: int,
    total_query_heads: int,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``[B, P, N]`` per-kv-head mass -> ``[B, N]`` head-mean normalised scores."""
    device = _lib.require_cuda(parts, seq_lens)
    if parts.ndim != 3 or parts.dtype != torch.float32 or parts.stride(2) != 1:
        raise ValueError("parts must be fp32 [batch, parts, chunks] with unit chunk stride")
    batch_size, num_parts, max_chunks = parts.shape
    if out is None:
        out = torch.empty((batch_size, max_chunks), dtype=torch.float32, device=device)
    seq_lens = _prep_index(seq_lens).contiguous()
    _lib.call(
        "dsb_finalize_chunk_scores",
        _lib.ptr(parts),
        parts.stride(0),
        parts.stride(1),
        num_parts,
        _lib.ptr(seq_lens),
        batch_size,
        total_query_heads,
        chunk_size,
        max_chunks,
        _lib.ptr(out),
        _lib.stream_ptr(device),
    )
    return out


def paged_chunk_attention_scores(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    softmax_lse: torch.Tensor | None,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    *,
    chunk_size: int,
    max_seq_len: int,
    scale: float,
) -> torch.Tensor:
    """Compute normalized logical-chunk attention scores from paged K.

    Drop-in for diffspec/kernels.py:95-150: returns ``[B, ceil(max_seq_len /
    chunk_size)]`` fp32, the mean over query heads of each chunk's attention
    mass divided by its valid token count (0 past ``seq_lens``).  Passing
    ``softmax_lse=None`` computes the log-sum-exp on the device.
    """
    head_scores = paged_chunk_head_scores(
        query, key_cache, softmax_lse, block_table, seq_lens,
        chunk_size=chunk_size, max_seq_len=max_seq_len, scale=scale,
    )
    return finalize_chunk_scores(
        head_scores, seq_lens, chunk_size=chunk_size, total_query_heads=query.shape[1]
    )


def gather_raw_kv_with_local_rope(
    raw_key_cache: torch.Tensor,
    raw_value_cache: torch.Tensor,
    block_table: torch.Tensor,
    selected_token_indices: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    *,
    rope_dim: int,
    is_neox_style: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gather raw paged KV and rotate K at compact local positions.

    Drop-in for diffspec/kernels.py:153-210.  ``selected_token_indices`` is
    ``[batch, working_tokens]`` with ``-1`` for padding (zero rows that still
    take a local position); returns ``(key, value)`` shaped
    ``[batch, tokens, heads, dim]``.  One fused kernel does the gather, the
    RoPE at local positions ``0..W-1`` and the write.
    """
    # diffspec/kernels.py:168-175
    if raw_key_cache.shape != raw_value_cache.shape or raw_key_cache.ndim != 4:
        raise ValueError("raw key/value caches must be matching 4-D tensors")
    if selected_token_indices.ndim != 2:
        raise ValueError("selected_token_indices must be two-dimensional")
    batch_size, working_tokens = selected_token_indices.shape
    num_blocks, block_size, num_kv_heads, head_dim = raw_key_cache.shape
    if block_table.shape[0] != batch_size:
        raise ValueError("block table batch size does not match token indices")
    if raw_key_cache.dtype != raw_value_cache.dtype:
        raise ValueError("raw key/value caches must share a dtype")
    if rope_dim < 0 or rope_dim > head_dim or rope_dim % 2:
        raise ValueError("rope_dim must be even and between zero and head_dim")
    if rope_dim and (
        cos_sin_cache.ndim != 2
        or cos_sin_cache.shape[0] < working_tokens
        or cos_sin_cache.shape[1] < rope_dim
        or cos_sin_cache.stride(1) != 1
    ):
        raise ValueError("cos/sin cache must contain all local positions and rotary dimensions")
    device = _lib.require_cuda(raw_key_cache, raw_value_cache, block_table, selected_token_indices)
    out_key = torch.empty(
        (batch_size, working_tokens, num_kv_heads, head_dim), dtype=raw_key_cache.dtype, device=device
    )
    out_value = torch.empty_like(out_key)
    if batch_size == 0 or working_tokens == 0:
        return out_key, out_value
    table = _prep_index(block_table)
    if table.stride(1) != 1:
        table = table.contiguous()
    sel = selected_token_indices.to(torch.int64).contiguous()
    cs = cos_sin_cache if rope_dim else raw_key_cache
    _lib.call(
        "dsb_gather_raw_kv_with_local_rope",
        _lib.ptr(raw_key_cache.contiguous()),
        _lib.ptr(raw_value_cache.contiguous()),
        num_blocks,
        block_size,
        num_kv_heads,
        head_dim,
        _lib.ptr(table),
        table.stride(0),
        table.shape[1],
        _lib.ptr(sel),
        batch_size,
        working_tokens,
        _lib.ptr(cs),
        _lib.dtype_code(cs.dtype),
        cs.stride(0) if rope_dim else 0,
        cs.shape[0] if rope_dim else 0,
        rope_dim,
        int(bool(is_neox_style)),
        _lib.dtype_code(raw_key_cache.dtype),
        _lib.ptr(out_key),
        _lib.ptr(out_value),
        _lib.ptr(_lib.error_flag(device)),
        _lib.stream_ptr(device),
    )
    return out_key, out_value


def kv_projection_write_raw(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    slots: torch.Tensor,
    positions: torch.Tensor,
    raw_key: torch.Tensor,
    raw_value: torch.Tensor,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Draft-layer K/V projection that also stores its rows in the raw cache.

    ``out = hidden @ weight.T`` (``hidden [T, hidden_size]``, ``weight
    [2 * Hk * D, hidden_size]``: K rows then V rows; fp32 accumulation, one
    rounding), returned as ``[T, 2 * Hk * D]``; row ``t``'s K and V halves
    are also written, pre-RoPE, to ``raw_key/raw_value [S, max_model_len, Hk,
    D]`` at ``[slots[t], positions[t]]`` (``slots[t] < 0``: padding).  This
    is the projection + ``_write_raw`` pair of diffspec/runtime.py:1602-1618
    in one launch.
    """
    if hidden.ndim != 2 or weight.ndim != 2 or weight.shape[1] != hidden.shape[1]:
        raise ValueError("hidden must be [T, hidden] and weight [2 * Hk * D, hidden]")
    if raw_key.ndim != 4 or raw_key.shape != raw_value.shape:
        raise ValueError("raw key/value must have matching 4-D shapes")
    num_slots, max_model_len, hk, d = raw_key.shape
    if weight.shape[0] != 2 * hk * d:
        raise ValueError("weight rows must be 2 * kv_heads * head_dim")
    if not (hidden.dtype == weight.dtype == raw_key.dtype == raw_value.dtype):
        raise ValueError("hidden, weight and raw caches must share a dtype")
    tokens = hidden.shape[0]
    if slots.shape[0] < tokens or positions.shape[0] < tokens:
        raise ValueError("slots/positions must cover every token")
    device = _lib.require_cuda(hidden, weight, slots, positions, raw_key, raw_value)
    if out is None:
        out = torch.empty((tokens, weight.shape[0]), dtype=hidden.dtype, device=device)
    elif out.shape != (tokens, weight.shape[0]) or out.dtype != hidden.dtype or not out.is_contiguous():
        raise ValueError("out must be contiguous [T, 2 * Hk * D] in the hidden dtype")
    hidden = hidden.contiguous()
    weight = weight.contiguous()
    slots = slots.to(torch.int32).contiguous()
    positions = positions.to(torch.int64).contiguous()
    if not (raw_key.is_contiguous() and raw_value.is_contiguous()):
        raise ValueError("raw caches must be contiguous")
    _lib.call(
        "dsb_kv_projection_write_raw",
        _lib.ptr(hidden), tokens, hidden.shape[1], _lib.ptr(weight), hk, d, _lib.ptr(slots),
        _lib.ptr(positions), _lib.ptr(raw_key), _lib.ptr(raw_value), num_slots, max_model_len,
        _lib.dtype_code(hidden.dtype), _lib.ptr(out), _lib.ptr(_lib.error_flag(device)),
        _lib.stream_ptr(device),
    )
    return out


def qkv_projection_write_raw(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    q_features: int,
    slots: torch.Tensor,
    positions: torch.Tensor,
    raw_key: torch.Tensor,
    raw_value: torch.Tensor,
    q_out: torch.Tensor | None = None,
    kv_out: torch.Tensor | None = None,
    prefetch_weight: bool = False,
    packed_weight: bool = False,
    prefetch_l2: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """The draft layer's query + K/V projection in one launch.

    ``weight [q_features + 2 * Hk * D, hidden_size]`` holds the query rows,
    then the K rows, then the V rows (a QKVParallelLinear weight).  Returns
    ``(q [T, q_features], kv [T, 2 * Hk * D])``; the K/V rows are also
    written, pre-RoPE, to the raw caches at ``[slots[t], positions[t]]`` as
    in :func:`kv_projection_write_raw`.  ``prefetch_weight`` lets the weight
    stream start before the previous kernel in the stream has finished (the
    weight must not be written by that kernel); ``prefetch_l2`` (with
    ``prefetch_weight``) also requests the next weight blocks of every CTA
    into L2 before that kernel has finished (faster alone; it puts more of
    the weight in L2);
    ``packed_weight``: ``weight`` is in the tile-packed layout of
    ``draft_layer.pack_linear_weight``.
    """
    if hidden.ndim != 2 or weight.ndim != 2 or weight.shape[1] != hidden.shape[1]:
        raise ValueError("hidden must be [T, hidden] and weight [q + 2 * Hk * D, hidden]")
    if raw_key.ndim != 4 or raw_key.shape != raw_value.shape:
        raise ValueError("raw key/value must have matching 4-D shapes")
    num_slots, max_model_len, hk, d = raw_key.shape
    if q_features < 0 or weight.shape[0] != q_features + 2 * hk * d:
        raise ValueError("weight rows must be q_features + 2 * kv_heads * head_dim")
    if not (hidden.dtype == weight.dtype == raw_key.dtype == raw_value.dtype):
        raise ValueError("hidden, weight and raw caches must share a dtype")
    tokens = hidden.shape[0]
    if slots.shape[0] < tokens or positions.shape[0] < tokens:
        raise ValueError("slots/positions must cover every token")
    device = _lib.require_cuda(hidden, weight, slots, positions, raw_key, raw_value, q_out, kv_out)
    for name, t, cols in (("q_out", q_out, q_features), ("kv_out", kv_out, 2 * hk * d)):
        if t is not None and (t.shape != (tokens, cols) or t.dtype != hidden.dtype
                              or not t.is_contiguous()):
            raise ValueError(f"{name} must be contiguous [T, {cols}] in the hidden dtype")
    if q_out is None:
        q_out = torch.empty((tokens, q_features), dtype=hidden.dtype, device=device)
    if kv_out is None:
        kv_out = torch.empty((tokens, 2 * hk * d), dtype=hidden.dtype, device=device)
    if not (hidden.is_contiguous() and weight.is_contiguous()):
        raise ValueError("hidden and weight must be contiguous")
    if slots.dtype != torch.int32 or positions.dtype != torch.int64:
        raise ValueError("slots must be int32 and positions int64")
    if not (raw_key.is_contiguous() and raw_value.is_contiguous()):
        raise ValueError("raw caches must be contiguous")
    _lib.call(
        "dsb_qkv_projection_write_raw",
        _lib.ptr(hidden), tokens, hidden.shape[1], _lib.ptr(weight), q_features, hk, d,
        _lib.ptr(slots), _lib.ptr(positions), _lib.ptr(raw_key), _lib.ptr(raw_value), num_slots,
        max_model_len, _lib.dtype_code(hidden.dtype), _lib.ptr(q_out), _lib.ptr(kv_out),
        (1 if prefetch_weight else 0) | (2 if packed_weight else 0) | (4 if prefetch_l2 else 0),
        _lib.ptr(_lib.error_flag(device)), _lib.stream_ptr(device),
    )
    return q_out, kv_out


def paged_decode_attention_lse(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    *,
    scale: float,
    max_seq_len: int,
    table_rows: torch.Tensor | None = None,
    tokens_per_split: int = 0,
    out: torch.Tensor | None = None,
    lse: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Target paged decode attention that also returns the softmax LSE.

    The B200 stand-in for the target's FIA call with ``softmax_lse_flag``
    (diffspec/ascend_patch.py:191-240) whose LSE ``capture_target_attention``
    stores (diffspec/runtime.py:841-894): ``query [rows, Hq, 128]`` against
    the paged ``key_cache`` / ``value_cache [blocks, block_size, Hk, 128]``,
    row ``r`` seeing the first ``seq_lens[r]`` tokens of block-table row
    ``table_rows[r]`` (default ``r``).  Returns ``(out [rows, Hq, 128],
    lse [rows, Hq] fp32)``, ``lse`` the natural log of the softmax
    denominator of ``scale * q . k`` — the ``softmax_lse`` that
    :func:`paged_chunk_attention_scores` takes.  ``tokens_per_split`` sets
    the split-KV length; 0 picks the library's default (1024 tokens when
    ``max_seq_len >= 16384``, else 512).
    """
    if query.ndim != 3 or key_cache.ndim != 4 or key_cache.shape != value_cache.shape:
        raise ValueError("query must be [rows, Hq, D] and the caches matching [blocks, bs, Hk, D]")
    rows, hq, d = query.shape
    num_blocks, block_size, hk, kd = key_cache.shape
    if d != kd or hq % hk:
        raise ValueError("head dims must match and Hq must be a multiple of Hk")
    if not (query.dtype == key_cache.dtype == value_cache.dtype):
        raise ValueError("query and caches must share a dtype")
    if block_table.ndim != 2 or seq_lens.numel() < rows:
        raise ValueError("block_table must be 2-D and seq_lens cover every row")
    if table_rows is not None and table_rows.numel() < rows:
        raise ValueError("table_rows must map every query row")
    if max_seq_len < 0:
        raise ValueError("max_seq_len must be >= 0")
    if tokens_per_split <= 0:  # the library's default split length (see the C ABI)
        tokens_per_split = 0
    device = _lib.require_cuda(query, key_cache, value_cache, block_table, seq_lens, table_rows)
    if out is None:
        out = torch.empty_like(query)
    if lse is None:
        lse = torch.empty((rows, hq), dtype=torch.float32, device=device)
    if out.shape != query.shape or out.dtype != query.dtype or not out.is_contiguous():
        raise ValueError("out must be contiguous and shaped like query")
    if lse.shape != (rows, hq) or lse.dtype != torch.float32 or not lse.is_contiguous():
        raise ValueError("lse must be contiguous fp32 [rows, Hq]")
    if rows == 0:
        return out, lse
    query = query.contiguous()
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("caches must be contiguous")
    table = _prep_index(block_table)
    if table.stride(1) != 1:
        table = table.contiguous()
    seq = _prep_index(seq_lens).contiguous()
    trows = None if table_rows is None else _prep_index(table_rows).contiguous()
    floats = _lib.load().dsb_paged_decode_scratch_floats(rows, hq, int(max_seq_len), tokens_per_split)
    scratch = torch.empty(max(floats, 1), dtype=torch.float32, device=device)
    _lib.call(
        "dsb_paged_decode_attention_lse",
        _lib.ptr(query), rows, hq, hk, d, _lib.ptr(key_cache), _lib.ptr(value_cache), num_blocks,
        block_size, _lib.ptr(table), table.stride(0), table.shape[0], table.shape[1],
        _lib.ptr(seq), _lib.ptr(trows), int(max_seq_len), float(scale),
        _lib.dtype_code(query.dtype), int(tokens_per_split), _lib.ptr(out), _lib.ptr(lse),
        _lib.ptr(scratch), scratch.numel(), _lib.ptr(_lib.error_flag(device)),
        _lib.stream_ptr(device),
    )
    return out, lse
