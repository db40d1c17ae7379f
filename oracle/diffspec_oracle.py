"""CPU oracle for the DiffSpec draft-context path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of the reference
vllm-ascend-hust-diffspec 0.3.0 for the hot path (retrieval scores, chunk
selection, compact history plans, gather + local RoPE rebuild, draft decode
attention, committed-query pick, raw-KV write).  Each function cites the
reference file:line it follows.  It is the checker for the CUDA library and
the timed CPU baseline of bench.py; the product path never imports it.

Parity status: pinned.  tests/golden/make_golden.py runs the reference itself
(its PyTorch CPU path and its Triton kernels under TRITON_INTERPRET=1) on
seeded inputs and stores the results in tests/golden/*.npz; the CPU test
suite checks this module against those fixtures and against the known-answer
vectors of the reference's own tests (tests/test_runtime.py).

Element types: arrays are float32/float64 numpy arrays holding values that
are exact in the storage dtype; ``round_to(x, dtype)`` rounds to bf16 / fp16
/ fp32 with round-to-nearest-even, the way a store to that dtype does.
"""

from __future__ import annotations

import math

import numpy as np

__all__ = [
    "round_to",
    "bf16_bits_to_f32",
    "f32_to_bf16_bits",
    "chunk_attention_scores",
    "paged_chunk_head_scores",
    "paged_chunk_attention_scores",
    "select_context_chunks",
    "history_budget",
    "history_indices",
    "history_plan",
    "decode_history_plan",
    "rebuild_compact_kv_from_plan",
    "gather_raw_kv_with_local_rope",
    "rope_rotate",
    "draft_decode_attention",
    "prepare_retrieval_rows",
    "write_raw",
    "request_rows",
    "capture_raw_kv",
    "selection_margin",
    "SlotTable",
]


# ----------------------------------------------------------------- dtypes
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest-even) and return the 16-bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round to the storage dtype ('bf16', 'f16', 'f32'), returned as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "f32":
        return x
    raise ValueError(dtype)


# ------------------------------------------------------- A2: dense scores
def chunk_attention_scores(query, keys, chunk_size, softmax_lse=None, scale=None, acc=np.float64):
    """diffspec/runtime.py:281-345.

    query [Hq, D], keys [T, Hk, D] -> [ceil(T / C)]: mean over query heads of
    each chunk's softmax mass divided by its token count (the last chunk by
    its partial count).  ``softmax_lse=None`` uses the logsumexp over all T
    tokens (:321-322).
    """
    query = np.asarray(query, dtype=acc)
    keys = np.asarray(keys, dtype=acc)
    hq, d = query.shape
    t, hk, _ = keys.shape
    if hq % hk:
        raise ValueError("query heads must be divisible by KV heads")
    if chunk_size <= 0:
        raise ValueError("chunk_size must be positive")
    if t == 0:
        return np.zeros(0, dtype=np.float64)
    g = hq // hk
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    # logits[h, t] = scale * q_h . k_{t, h // g}            (:313-319)
    logits = np.einsum("kgd,tkd->kgt", query.reshape(hk, g, d), keys).reshape(hq, t) * scale
    if softmax_lse is None:
        m = logits.max(axis=1, keepdims=True)
        lse = (m + np.log(np.exp(logits - m).sum(axis=1, keepdims=True)))[:, 0]
    else:
        lse = np.asarray(softmax_lse, dtype=acc).reshape(-1)
    mass = np.exp(logits - lse[:, None])                   # (:323)
    n = (t + chunk_size - 1) // chunk_size
    pad = n * chunk_size - t
    if pad:
        mass = np.pad(mass, ((0, 0), (0, pad)))
    chunk_mass = mass.reshape(hq, n, chunk_size).sum(axis=-1)  # (:330-333)
    counts = np.full(n, chunk_size, dtype=acc)
    counts[-1] = t - (n - 1) * chunk_size                       # (:334-344)
    return chunk_mass.mean(axis=0) / counts


# ------------------------------------------------------- A1: paged scores
def _gather_paged_keys(key_cache, block_table_row, length):
    bs = key_cache.shape[1]
    tok = np.arange(length)
    pages = np.asarray(block_table_row, dtype=np.int64)[tok // bs]
    return key_cache[pages, tok % bs]  # [L, Hk, D]


def paged_chunk_head_scores(query, key_cache, softmax_lse, block_table, seq_lens, chunk_size,
                            max_seq_len, scale, acc=np.float64):
    """Per-(row, kv head, chunk) unnormalised mass (diffspec/kernels.py:35-83).

    out[b, g, c] = sum_{h in group g} sum_{t in c, t < L_b} exp(scale q_h.k_t - lse_h).
    ``softmax_lse=None`` computes the per-head LSE over the row's L_b tokens.
    """
    query = np.asarray(query, dtype=acc)
    b_n, hq, d = query.shape
    hk = key_cache.shape[2]
    g = hq // hk
    n_max = (max_seq_len + chunk_size - 1) // chunk_size
    out = np.zeros((b_n, hk, n_max), dtype=acc)
    for b in range(b_n):
        length = int(seq_lens[b])
        if length <= 0:
            continue
        keys = np.asarray(_gather_paged_keys(key_cache, block_table[b], length), dtype=acc)
        logits = np.einsum("kgd,tkd->kgt", query[b].reshape(hk, g, d), keys) * scale
        if softmax_lse is None:
            m = logits.max(axis=2, keepdims=True)
            lse = m + np.log(np.exp(logits - m).sum(axis=2, keepdims=True))
        else:
            lse = np.asarray(softmax_lse, dtype=acc).reshape(b_n, hk, g)[b][:, :, None]
        mass = np.exp(logits - lse).sum(axis=1)  # [Hk, L]
        n = (length + chunk_size - 1) // chunk_size
        pad = n * chunk_size - length
        if pad:
            mass = np.pad(mass, ((0, 0), (0, pad)))
        out[b, :, :n] = mass.reshape(hk, n, chunk_size).sum(axis=-1)
    return out


def paged_chunk_attention_scores(query, key_cache, softmax_lse, block_table, seq_lens, chunk_size,
                                 max_seq_len, scale, acc=np.float64):
    """diffspec/kernels.py:95-150: [B, ceil(max_seq_len / C)] head-mean scores."""
    parts = paged_chunk_head_scores(query, key_cache, softmax_lse, block_table, seq_lens,
                                    chunk_size, max_seq_len, scale, acc)
    hq = np.asarray(query).shape[1]
    b_n, _, n_max = parts.shape
    out = np.zeros((b_n, n_max), dtype=acc)
    for b in range(b_n):
        length = int(seq_lens[b])
        for c in range(n_max):
            nv = max(0, min(chunk_size, length - c * chunk_size))
            if nv:
                out[b, c] = parts[b, :, c].sum() / nv / hq  # (:81-83, :150)
    return out


# ------------------------------------------------------- A4: selection
def _window_chunks(recent_window, chunk_size, token_budget):
    """Chunks of the rolling recent window; 1 (the reference) when it is None."""
    if recent_window is None:
        return 1
    if recent_window < chunk_size or recent_window % chunk_size or recent_window > token_budget:
        raise ValueError("recent_window must be a chunk-size multiple in [chunk_size, budget]")
    return recent_window // chunk_size


def select_context_chunks(chunk_scores, seq_len, chunk_size, token_budget, recent_window=None):
    """diffspec/runtime.py:348-414 with ties ranked by ascending chunk index.

    ``recent_window`` (tokens, a multiple of the chunk size; None = one chunk,
    the reference) is the window mode, which has no reference counterpart:
    with wc = recent_window / C the newest wc chunks are left out of the
    ranking (the rolling recent window of the plan holds them) and the top
    S - wc of chunks 0..n-1-wc are kept, plus the newest chunk, ascending.
    wc = 1 is exactly the reference's top S - 1 of chunks 0..n-2.
    Returns (chunk_indices, token_indices, chunk_scores) as numpy arrays.
    """
    chunk_scores = np.asarray(chunk_scores)
    if chunk_scores.ndim != 1:
        raise ValueError("chunk_scores must be one-dimensional")
    if seq_len < 0:
        raise ValueError("seq_len must be non-negative")
    if token_budget < chunk_size or token_budget % chunk_size != 0:
        raise ValueError("token_budget must be a positive chunk-size multiple")
    n = (seq_len + chunk_size - 1) // chunk_size
    if n != chunk_scores.size:
        raise ValueError("chunk score count does not match sequence length")
    if n == 0:
        e = np.zeros(0, dtype=np.int64)
        return e, e, chunk_scores
    max_chunks = token_budget // chunk_size
    wc = _window_chunks(recent_window, chunk_size, token_budget)
    if n <= max_chunks:
        chosen = np.arange(n, dtype=np.int64)
    else:
        # top (max_chunks - wc) of chunks 0..n-1-wc plus the newest (:371-390)
        cand = np.arange(n - wc)
        s = chunk_scores[: n - wc]
        order = np.lexsort((cand, -s.astype(np.float64)))  # score desc, index asc
        ranked = np.sort(cand[order[: max_chunks - wc]])
        chosen = np.concatenate([ranked, [n - 1]]).astype(np.int64)
    offsets = np.arange(chunk_size, dtype=np.int64)
    if seq_len % chunk_size:
        full = (chosen[:-1, None] * chunk_size + offsets[None, :]).reshape(-1)
        tail = np.arange((n - 1) * chunk_size, seq_len, dtype=np.int64)
        tokens = np.concatenate([full, tail])
    else:
        tokens = (chosen[:, None] * chunk_size + offsets[None, :]).reshape(-1)
    return chosen, tokens, chunk_scores[chosen]


def selection_margin(chunk_scores, seq_len, chunk_size, token_budget, recent_window=None):
    """Relative score gap at the top-k boundary (inf when nothing is ranked).

    Used to certify that a fp32 GPU score vector must select exactly what the
    fp64 oracle selects: the selection cannot change unless the rounding
    error exceeds this gap.  ``recent_window`` as in select_context_chunks.
    """
    s = np.asarray(chunk_scores, dtype=np.float64)
    n = (seq_len + chunk_size - 1) // chunk_size
    wc = _window_chunks(recent_window, chunk_size, token_budget)
    k = token_budget // chunk_size - wc
    if n <= token_budget // chunk_size or k <= 0:
        return math.inf
    cand = np.sort(s[: n - wc])[::-1]
    gap = cand[k - 1] - cand[k]
    return gap / max(abs(cand[k - 1]), 1e-30)


# ------------------------------------------------------- A5: history plans
def history_budget(token_budget, max_tree_depth, chunk_size):
    """diffspec/runtime.py:627-635."""
    return (token_budget - max_tree_depth - 1) // chunk_size * chunk_size


def history_indices(selected_tokens, history_end, chunk_size, hbudget, recent_window=None):
    """diffspec/runtime.py:1650-1681 (_history_indices).

    ``selected_tokens`` is None (no retrieval yet) or the selection's token ids.
    ``recent_window`` (window mode, no reference counterpart; None = one
    chunk, the reference) is the length of the rolling tail.
    """
    window = chunk_size if recent_window is None else recent_window
    if selected_tokens is not None:
        selected = np.asarray(selected_tokens, dtype=np.int64)
        tail_start = max(0, history_end - min(window, hbudget))
        prefix = selected[(selected >= 0) & (selected < tail_start)]
        if selected.size:
            newest_start = (selected[-1] // chunk_size) * chunk_size
            prefix = prefix[prefix < newest_start]
        tail = np.arange(tail_start, history_end, dtype=np.int64)
        prefix_budget = hbudget - tail.size
        # torch's selected_prefix[-prefix_budget:] keeps the whole tensor when
        # the budget exceeds its length
        prefix = prefix[max(0, len(prefix) - prefix_budget):] if prefix_budget else prefix[:0]
        return np.concatenate([prefix, tail])
    start = max(0, history_end - hbudget)
    return np.arange(start, history_end, dtype=np.int64)


def history_plan(slot, selected_chunks, history_end, chunk_size, hbudget, recent_window=None):
    """diffspec/runtime.py:1713-1735 (_history_plan_host) -> plan row (list).

    ``selected_chunks`` is None (no retrieval yet), [] (empty selection) or
    the ascending chunk ids of the slot's selection.  ``recent_window`` as in
    :func:`history_indices` (the rolling tail's length; None = one chunk).
    """
    window = chunk_size if recent_window is None else recent_window
    if selected_chunks is None:
        length = min(history_end, hbudget)
        return [slot, length, history_end - length, 0, 0]
    tail_length = min(history_end, window, hbudget)
    tail_start = history_end - tail_length
    chunks = [int(c) for c in selected_chunks]
    if not chunks:
        return [slot, tail_length, tail_start, 0, 0]
    prefix_end = min(tail_start, chunks[-1] * chunk_size)
    prefix_tokens = sum(max(0, min(chunk_size, prefix_end - c * chunk_size)) for c in chunks)
    prefix_length = min(prefix_tokens, hbudget - tail_length)
    return [slot, prefix_length + tail_length, tail_start, prefix_length,
            prefix_tokens - prefix_length, *chunks]


def decode_history_plan(plan, chunk_size):
    """Expand a plan row into absolute positions (tests/test_runtime.py:31-38)."""
    _, length, tail_start, prefix_length, prefix_drop, *chunks = [int(v) for v in plan]
    prefix = [chunks[(p + prefix_drop) // chunk_size] * chunk_size + (p + prefix_drop) % chunk_size
              for p in range(prefix_length)]
    return prefix + list(range(tail_start, tail_start + length - prefix_length))


# ------------------------------------------------------- RoPE
def rope_rotate(x, cos_sin_row, rotary_dim, is_neox_style):
    """Rotate [..., D] float32 at one position, fp32 math with products
    rounded before the add (compact_kv.py:57-108 evaluated without FMA).
    ``cos_sin_row`` holds [cos(0..half) | sin(0..half)]."""
    x = np.asarray(x, dtype=np.float32)
    out = x.copy()
    if rotary_dim == 0:
        return out
    half = rotary_dim // 2
    cos = np.asarray(cos_sin_row[:half], dtype=np.float32)
    sin = np.asarray(cos_sin_row[half:2 * half], dtype=np.float32)
    if is_neox_style:
        first = x[..., :half]
        second = x[..., half:rotary_dim]
        out[..., :half] = (first * cos) - (second * sin)
        out[..., half:rotary_dim] = (second * cos) + (first * sin)
    else:
        first = x[..., 0:rotary_dim:2]
        second = x[..., 1:rotary_dim:2]
        out[..., 0:rotary_dim:2] = (first * cos) - (second * sin)
        out[..., 1:rotary_dim:2] = (second * cos) + (first * sin)
    return out


# ------------------------------------------------------- A6: rebuild
def rebuild_compact_kv_from_plan(raw_key, raw_value, working_key, working_value, plan,
                                 cos_sin_cache, chunk_size, max_width, rotary_dim, is_neox_style,
                                 dtype="bf16"):
    """diffspec/compact_kv.py:8-133 (kernel) / :184-242 (API), in place.

    raw [S, L, H, D], working [S, H, W, D] (float32 arrays holding dtype
    values), plan [rows, 5 + W / C] int64.
    """
    for row in np.asarray(plan, dtype=np.int64):
        slot, hlen, tail_start, prefix_len, drop = (int(v) for v in row[:5])
        chunks = row[5:]
        for p in range(min(hlen, max_width)):
            if p < prefix_len:
                q = p + drop
                abs_pos = int(chunks[q // chunk_size]) * chunk_size + q % chunk_size
            else:
                abs_pos = tail_start + p - prefix_len
            k = raw_key[slot, abs_pos]  # [H, D]
            working_value[slot, :, p] = raw_value[slot, abs_pos]
            working_key[slot, :, p] = round_to(
                rope_rotate(k, cos_sin_cache[p], rotary_dim, is_neox_style), dtype)


# ------------------------------------------------------- A7: paged gather
def gather_raw_kv_with_local_rope(raw_key_cache, raw_value_cache, block_table,
                                  selected_token_indices, cos_sin_cache, rope_dim,
                                  is_neox_style=True, dtype="bf16"):
    """diffspec/kernels.py:153-210 -> (K, V) [B, W, H, D]; -1 ids give zero rows."""
    sel = np.asarray(selected_token_indices, dtype=np.int64)
    b_n, w = sel.shape
    _, bs, h, d = raw_key_cache.shape
    out_k = np.zeros((b_n, w, h, d), dtype=np.float32)
    out_v = np.zeros_like(out_k)
    for b in range(b_n):
        for p in range(w):
            idx = int(sel[b, p])
            if idx < 0:
                continue
            page = int(block_table[b][idx // bs])
            out_v[b, p] = raw_value_cache[page, idx % bs]
            out_k[b, p] = round_to(
                rope_rotate(raw_key_cache[page, idx % bs], cos_sin_cache[p], rope_dim,
                            is_neox_style), dtype)
    return out_k, out_v


# ------------------------------------------------------- A8: attention
def draft_decode_attention(query, key, value, working_key, working_value, slots, positions, scale,
                           out_rows=None, dtype="bf16"):
    """diffspec/runtime.py:2040-2077 (CPU loop), in place on the working caches.

    Writes key/value at each row's local position, then
    out[r, h] = softmax(scale * q[r, h] . K[slot, h // g, :pos+1]) . V[...]
    in fp64; rows >= len(slots) of the output are zero.
    """
    query = np.asarray(query, dtype=np.float64)
    n, hq, d = query.shape
    hk = working_key.shape[1]
    g = hq // hk
    out_rows = n if out_rows is None else out_rows
    out = np.zeros((out_rows, hq, d), dtype=np.float64)
    for r, (slot, pos) in enumerate(zip(slots, positions)):
        slot, pos = int(slot), int(pos)
        working_key[slot, :, pos] = key[r]
        working_value[slot, :, pos] = value[r]
        k = np.repeat(np.asarray(working_key[slot, :, : pos + 1], dtype=np.float64), g, axis=0)
        v = np.repeat(np.asarray(working_value[slot, :, : pos + 1], dtype=np.float64), g, axis=0)
        logits = np.einsum("hd,hsd->hs", query[r], k) * scale
        logits -= logits.max(axis=1, keepdims=True)
        p = np.exp(logits)
        p /= p.sum(axis=1, keepdims=True)
        out[r] = np.einsum("hs,hsd->hd", p, v)
    return round_to(out.astype(np.float32), dtype) if dtype else out


# ------------------------------------------------------- A3: committed-query pick
def prepare_retrieval_rows(query_ends, target_seq_lens, counts, active_slots):
    """diffspec/runtime.py:1223-1276 for linear proposals.

    Returns (query_index, retrieval_len, row_slot) per request; rows with no
    accepted token get retrieval_len 0 and row_slot -1 (skipped, :1254-1257).
    """
    q_index, r_len, r_slot = [], [], []
    start = 0
    for end, seq_len, count, slot in zip(query_ends, target_seq_lens, counts, active_slots):
        qlen = end - start
        count = int(count)
        if count > 0:
            off = min(max(count - 1, 0), qlen - 1)
            committed = min(max(count, 1), qlen)
            q_index.append(start + off)
            r_len.append(seq_len - qlen + committed)
            r_slot.append(slot)
        else:
            q_index.append(start)
            r_len.append(0)
            r_slot.append(-1)
        start = end
    return q_index, r_len, r_slot


# ------------------------------------------------------- (f) request slots
class SlotTable:
    """Canonical request slots (set_active_requests, diffspec/runtime.py:
    755-778): a request keeps its slot while it stays in the batch; the slots
    of requests that left are released first (their working length becomes
    0 and their selection is dropped); each request new to the table then
    takes the lowest free slot, in batch order; when none is left the call
    raises RuntimeError, after those releases and the assignments before it,
    leaving ``active`` as it was."""

    def __init__(self, num_slots: int):
        self.num_slots = num_slots
        self.slots: dict[str, int] = {}
        self.active: list[int] = []
        self.working_lens = [0] * num_slots
        self.selected: set[int] = set()

    def set_active_requests(self, request_ids) -> None:
        keep = set(request_ids)
        for rid in list(self.slots):
            if rid not in keep:
                slot = self.slots.pop(rid)
                self.selected.discard(slot)
                self.working_lens[slot] = 0
        used = set(self.slots.values())
        free = iter(sorted(set(range(self.num_slots)) - used))
        for rid in request_ids:
            if rid not in self.slots:
                nxt = next(free, None)
                if nxt is None:
                    raise RuntimeError("DiffSpec canonical request slots are exhausted")
                self.slots[rid] = nxt
        self.active = [self.slots[r] for r in request_ids]


# ------------------------------------------------------- A9: raw write
def write_raw(raw_key, raw_value, slots, positions, key, value):
    """diffspec/runtime.py:1602-1618: raw[slot_i, pos_i] = kv_i (in place)."""
    for i, (slot, pos) in enumerate(zip(slots, positions)):
        if int(slot) < 0:
            continue
        raw_key[int(slot), int(pos)] = key[i]
        raw_value[int(slot), int(pos)] = value[i]


def request_rows(query_ends, num_tokens):
    """Batch row of each token of a pass (diffspec/runtime.py:1580-1595)."""
    starts = [0, *[int(e) for e in query_ends]]
    rows, r = [], 0
    for t in range(num_tokens):
        while r + 1 < len(starts) - 1 and t >= starts[r + 1]:
            r += 1
        rows.append(r)
    return rows


def capture_raw_kv(raw_key, raw_value, slots, positions, key, value, history_lens, draft_step):
    """diffspec/runtime.py:1797-1877 inside a draft cycle (linear proposals):
    the first len(slots) rows are the requests (later rows are graph
    padding), written to the raw caches at their absolute positions; returns
    the step's local RoPE positions, history_len + draft_step for the
    requests (the root step at the history length, then one further per
    step, as the working lengths advance) and 0 for padding rows."""
    rows = len(slots)
    write_raw(raw_key, raw_value, slots, positions[:rows], key[:rows], value[:rows])
    local = np.zeros(len(positions), dtype=np.int64)
    local[:rows] = np.asarray(history_lens[:rows], dtype=np.int64) + draft_step
    return local


def kv_projection_write_raw(hidden, weight, slots, positions, raw_key, raw_value, dtype="bf16"):
    """The draft layer's K/V projection (vLLM linear: ``hidden @ weight.T``,
    weight rows K then V) followed by _write_raw (diffspec/runtime.py:1602-1618),
    in place on the raw caches.  Returns the projected rows rounded to `dtype`
    (fp32 products and sums, one rounding)."""
    kv = round_to(hidden.astype(np.float32) @ weight.astype(np.float32).T, dtype)
    hk, d = raw_key.shape[2], raw_key.shape[3]
    half = hk * d
    write_raw(raw_key, raw_value, slots, positions, kv[:, :half].reshape(-1, hk, d),
              kv[:, half:].reshape(-1, hk, d))
    return kv


# ------------------------------------------------------- target attention + LSE
def paged_decode_attention_lse(query, key_cache, value_cache, block_table, seq_lens, scale,
                               table_rows=None, dtype="bf16"):
    """The target verifier's attention with its softmax LSE (the FIA call with
    softmax_lse_flag, diffspec/ascend_patch.py:191-240, whose LSE
    capture_target_attention keeps, diffspec/runtime.py:841-894), in fp64:
    out [rows, Hq, D] rounded to `dtype`, lse [rows, Hq] (natural log of the
    softmax denominator of scale * q . k; -inf for an empty row)."""
    q = np.asarray(query, dtype=np.float64)
    rows, hq, d = q.shape
    _, bs, hk, _ = key_cache.shape
    group = hq // hk
    out = np.zeros((rows, hq, d), dtype=np.float32)
    lse = np.full((rows, hq), -np.inf, dtype=np.float32)
    for r in range(rows):
        length = int(seq_lens[r])
        if length <= 0:
            continue
        trow = r if table_rows is None else int(table_rows[r])
        toks = np.arange(length)
        blocks = np.asarray(block_table[trow], dtype=np.int64)[toks // bs]
        k = np.asarray(key_cache, dtype=np.float64)[blocks, toks % bs]   # [L, Hk, D]
        v = np.asarray(value_cache, dtype=np.float64)[blocks, toks % bs]
        for h in range(hq):
            s = (k[:, h // group] @ q[r, h]) * scale
            m = s.max()
            p = np.exp(s - m)
            out[r, h] = (p @ v[:, h // group]) / p.sum()
            lse[r, h] = m + np.log(p.sum())
    return round_to(out, dtype), lse


# ------------------------------------------------------- draft layer elementwise stages
# The draft model is vLLM's Eagle3 Llama layer (a dependency of the reference,
# vllm>=0.28.1rc1.dev319,<0.28.2 in pyproject.toml, not vendored); these
# restate its RMSNorm and SiLU-and-mul at the storage dtype with vLLM's
# rounding points, pinned by tests/golden/make_layer_golden.py against the
# vLLM installed in this image, and its RoPE at the working cache's local
# positions (diffspec/runtime.py:1767-1794) with rope_rotate above.
def linear(x, weight, residual=None, dtype="bf16"):
    """A draft-layer linear (vLLM linear layers: ``x @ weight.T``), fp32
    products and sums, plus ``residual`` before the one rounding when given."""
    y = np.asarray(x, dtype=np.float32) @ np.asarray(weight, dtype=np.float32).T
    if residual is not None:
        y = y + np.asarray(residual, dtype=np.float32)
    return round_to(y, dtype)


def rms_norm(x, weight, eps, dtype="bf16"):
    """vLLM rms_norm (vllm/ir/ops/layernorm.py in the vLLM of this image):
    round(round(x * 1/sqrt(mean(x^2) + eps)) * weight) per row, the
    normalised value rounded to the weight dtype before the weight product
    (fp64 sum of squares here, fp32 products)."""
    x = np.asarray(x, dtype=np.float32)
    ms = (x.astype(np.float64) ** 2).mean(-1, keepdims=True)
    inv = (1.0 / np.sqrt(ms + eps)).astype(np.float32)
    return round_to(round_to(x * inv, dtype) * np.asarray(weight, dtype=np.float32), dtype)


def silu_mul(gate_up, dtype="bf16"):
    """vLLM SiluAndMul of [rows, 2 * inter] rows holding gate then up:
    round(round(gate / (1 + e^-gate)) * up), silu rounded to the storage
    dtype before the product."""
    gu = np.asarray(gate_up, dtype=np.float64)
    inter = gu.shape[-1] // 2
    g, u = gu[..., :inter], gu[..., inter:]
    silu = round_to((g / (1.0 + np.exp(-g))).astype(np.float32), dtype)
    return round_to(silu * u.astype(np.float32), dtype)


def rope_qk(query, kv, positions, cos_sin, num_kv_heads, dtype="bf16"):
    """One draft step's RoPE: query [T, Hq * D] and the K half of kv [T, 2 * Hk
    * D] rotated (NeoX) at positions[t]; returns (query, key [T, Hk, D], value
    [T, Hk, D]) rounded to `dtype`."""
    t_n = query.shape[0]
    feats = kv.shape[1] // 2
    d = feats // num_kv_heads
    q = np.asarray(query, dtype=np.float32).reshape(t_n, -1, d).copy()
    k = np.asarray(kv[:, :feats], dtype=np.float32).reshape(t_n, num_kv_heads, d).copy()
    v = np.asarray(kv[:, feats:], dtype=np.float32).reshape(t_n, num_kv_heads, d).copy()
    for t in range(t_n):
        row = np.asarray(cos_sin[int(positions[t])], dtype=np.float32)
        q[t] = round_to(rope_rotate(q[t], row, d, True), dtype)
        k[t] = round_to(rope_rotate(k[t], row, d, True), dtype)
    return q.reshape(t_n, -1), k, v
