/*
 * diffspec_b200.h — C ABI of the B200 (sm_100a) DiffSpec draft-context path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, NULL = legacy default stream), enqueues its kernels on
 * that stream and returns without synchronising.  The return value is a
 * status code; on failure dsb_last_error() returns a message for the calling
 * thread.  Arguments are validated on the host before any launch; indices that
 * live in device memory (plans, block tables, slots, positions) are checked by
 * the kernels, which skip an out-of-range access and OR a bit into
 * *error_flag (when error_flag is non-NULL) instead of faulting.
 *
 * Layouts (row-major, contiguous unless a stride is given):
 *   query            [rows, num_query_heads, head_dim]
 *   paged key cache  [num_blocks, block_size, num_kv_heads, head_dim]
 *   raw draft KV     [num_slots, max_model_len, num_kv_heads, head_dim]
 *   working KV       [num_slots, num_kv_heads, working_budget, head_dim]
 *   plan row         [slot, history_len, tail_start, prefix_len, prefix_drop,
 *                     chunk_ids..., 0 padding]   (int64, width 5 + W / C)
 *
 * Reference interfaces replaced (paths inside vllm-ascend-hust-diffspec 0.3.0):
 *   see the comment above each function.
 */
#ifndef DIFFSPEC_B200_H_
#define DIFFSPEC_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define DSB_OK 0
#define DSB_ERR_INVALID 1     /* an argument failed validation               */
#define DSB_ERR_UNSUPPORTED 2 /* valid, but no kernel for this shape/dtype   */
#define DSB_ERR_CUDA 3        /* a CUDA launch or runtime call failed        */

/* element type codes */
#define DSB_BF16 0
#define DSB_F16 1
#define DSB_F32 2

/* bits OR-ed into *error_flag by kernels that met a bad device-side index */
#define DSB_FLAG_SLOT 1       /* slot outside [0, num_slots)                 */
#define DSB_FLAG_POSITION 2   /* token position outside its cache            */
#define DSB_FLAG_BLOCK 4      /* block-table entry outside [0, num_blocks)   */
#define DSB_FLAG_PLAN 8       /* malformed plan row                          */
#define DSB_FLAG_CAPACITY 16  /* selection larger than the per-slot capacity */
#define DSB_FLAG_TIMEOUT 32   /* a bounded wait for an asynchronous copy ran out */

const char *dsb_last_error(void);
int dsb_abi_version(void);

/* Per-(row, kv-head, chunk) retrieval mass with a caller-supplied softmax LSE:
 *   head_scores[b, g, c] = sum_{h in group g} sum_{t in chunk c, t < L_b}
 *                          exp(scale * q[b,h] . k[b,t,g] - lse[b,h])
 * head_scores is [batch, num_kv_heads, max_chunks] fp32; chunks at or past
 * L_b = seq_lens[b] are written as 0, so L_b = 0 marks a skipped row.
 * query_index (nullable) maps row b to the query/LSE row it reads; rows
 * mapped outside [0, query_rows) are flagged (DSB_FLAG_POSITION) and scored 0.
 * Replaces the device kernel of paged_chunk_attention_scores
 * (diffspec/kernels.py:11-92, launch at :131-149); the head mean of :150 is
 * dsb_finalize_chunk_scores. */
int dsb_paged_chunk_head_scores(
    const void *query, const float *softmax_lse, const int32_t *query_index,
    int32_t query_rows,
    const void *key_cache, const int32_t *block_table, int64_t block_table_stride,
    int64_t block_table_cols, const int32_t *seq_lens, int32_t batch,
    int32_t num_query_heads, int32_t num_kv_heads, int32_t head_dim,
    int32_t block_size, int64_t num_blocks, int32_t chunk_size, int32_t max_chunks,
    float scale, int32_t dtype, float *head_scores, int32_t *error_flag,
    void *stream);

/* Same pass without an LSE: per (row, query head, chunk) the maximum logit
 * in log2 units (log2(e) * scale * q.k) and the sum of exp(logit - max_logit)
 * ([batch, num_query_heads, max_chunks] fp32 each).  dsb_chunk_stats_to_head_scores turns them into head_scores with the
 * sequence-wide log-sum-exp, which is the softmax_lse=None branch of
 * chunk_attention_scores (diffspec/runtime.py:321-322). */
int dsb_paged_chunk_stats(
    const void *query, const int32_t *query_index, int32_t query_rows,
    const void *key_cache,
    const int32_t *block_table, int64_t block_table_stride, int64_t block_table_cols,
    const int32_t *seq_lens, int32_t batch, int32_t num_query_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int64_t num_blocks,
    int32_t chunk_size, int32_t max_chunks, float scale, int32_t dtype,
    float *chunk_max, float *chunk_sum, int32_t *error_flag, void *stream);

/* lse_out (nullable) receives the per-(row, query head) log-sum-exp. */
int dsb_chunk_stats_to_head_scores(
    const float *chunk_max, const float *chunk_sum, const int32_t *seq_lens,
    int32_t batch, int32_t num_query_heads, int32_t num_kv_heads,
    int32_t chunk_size, int32_t max_chunks, float *head_scores, float *lse_out,
    void *stream);

/* scores[b, c] = sum_p parts[b, p, c] / (n_valid(b, c) * total_query_heads),
 * n_valid = number of tokens of chunk c below seq_lens[b] (0 -> score 0).
 * This is the per-head normalisation and head mean of
 * diffspec/kernels.py:81-83,150 and diffspec/runtime.py:336-345, with the
 * per-kv-head parts summed in a fixed order. */
int dsb_finalize_chunk_scores(
    const float *parts, int64_t row_stride, int64_t part_stride, int32_t num_parts,
    const int32_t *seq_lens, int32_t batch, int32_t total_query_heads,
    int32_t chunk_size, int32_t max_chunks, float *scores, void *stream);

/* Device top-k chunk selection, one CTA per row (select_context_chunks,
 * diffspec/runtime.py:348-414, via set_chunk_scores :1554-1567).
 * Row scores are sum_p parts[row, p, c], divided by n_valid * normalize_heads
 * when normalize_heads > 0.  Part p = q * parts_per_group + i of a row lies at
 * parts + row * row_stride + q * group_stride + i * part_stride
 * (parts_per_group <= 0: one group, the [rows, parts, N] layout; world groups
 * of Hk / world parts: the [world, rows, Hk / world, N] result of an
 * all-gather of per-rank parts, read without a copy).  With n = ceil(L / C)
 * chunks, S = history_budget / C and WC = recent_window / C (recent_window 0
 * means C, the reference): n <= S keeps every chunk, otherwise the S - WC
 * highest-scoring chunks among 0..n-1-WC (ties go to the lower chunk index)
 * plus chunk n-1, in ascending order.  WC > 1 is the rolling-recent-window
 * mode, which has no reference counterpart: the newest WC chunks belong to
 * the plan's rolling tail and are not ranked.  recent_window must be a
 * chunk-size multiple in [C, history_budget].  Rows whose row_slots entry is
 * < 0 are left alone; the others overwrite sel_chunks[slot, :count] /
 * sel_count[slot].  The optional outputs mirror DiffSpecSelection (-1
 * padded). */
int dsb_select_context_chunks(
    const float *parts, int64_t row_stride, int64_t part_stride, int32_t num_parts,
    int32_t parts_per_group, int64_t group_stride, int32_t normalize_heads,
    const int32_t *seq_lens, const int32_t *row_slots, int32_t rows, int32_t max_chunks,
    int32_t chunk_size, int32_t history_budget, int32_t recent_window, int32_t *sel_chunks,
    int32_t sel_stride, int32_t *sel_count, int32_t num_slots, int64_t *out_chunk_indices,
    int64_t *out_token_indices, float *out_chunk_scores, int32_t *error_flag, void *stream);

/* Compact history plan rows (_history_plan_host, diffspec/runtime.py:1713-1735,
 * equal to _history_indices :1650-1681 once expanded).  history_end =
 * max(0, committed_lens[row] - 1); sel_count[slot] < 0 means "no retrieval
 * yet".  The rolling tail is the last min(recent_window, history_budget)
 * history tokens (recent_window 0 means chunk_size, the reference; a longer
 * window, a chunk-size multiple up to history_budget, is the window mode of
 * dsb_select_context_chunks).  plan is [rows, plan_width] int64 with
 * plan_width = 5 + W / C.  history_lens (nullable, [rows]) and working_lens
 * (nullable, [num_slots]) receive history_len. */
int dsb_build_history_plan(
    const int32_t *row_slots, const int32_t *committed_lens, int32_t rows,
    const int32_t *sel_chunks, int32_t sel_stride, const int32_t *sel_count,
    int32_t num_slots, int32_t chunk_size, int32_t history_budget, int32_t recent_window,
    int32_t plan_width, int64_t *plan, int32_t *history_lens, int32_t *working_lens,
    int32_t *error_flag, void *stream);

/* Fused gather + local-position RoPE + working-cache write
 * (rebuild_compact_kv_from_plan, diffspec/compact_kv.py:184-242, kernel
 * :8-133).  For p < history_len of each plan row the K row at its absolute
 * position is rotated at local position p (fp32 math, products rounded before
 * the sum) and stored; V and K dims >= rotary_dim are copied.  Positions at or
 * past history_len are untouched.  cos_sin_cache rows hold [cos | sin]. */
int dsb_rebuild_compact_kv_from_plan(
    const void *raw_key, const void *raw_value, void *working_key, void *working_value,
    const int64_t *plan, int32_t plan_rows, int32_t plan_width,
    const void *cos_sin_cache, int32_t cos_sin_dtype, int64_t cos_sin_stride,
    int64_t cos_sin_rows, int32_t num_slots, int64_t max_model_len,
    int32_t num_heads, int32_t head_dim, int32_t working_budget, int32_t chunk_size,
    int32_t max_width, int32_t rotary_dim, int32_t is_neox_style, int32_t dtype,
    int32_t *error_flag, void *stream);

/* History plan and working-cache rebuild in one launch
 * (_rebuild_working_cache_batched, diffspec/runtime.py:1737-1765, which runs
 * _history_plan_host :1713-1735 on the host, copies the plan to the device and
 * calls rebuild_compact_kv_from_plan).  Every row's plan is computed on the
 * device from its slot's selection state and committed length exactly as
 * dsb_build_history_plan does and drives the rebuild of the same launch, so
 * the working cache is bit-identical to dsb_build_history_plan followed by
 * dsb_rebuild_compact_kv_from_plan.  plan ([rows, plan_width], plan_width =
 * 5 + working_budget / chunk_size), history_lens ([rows]) and working_lens
 * ([num_slots]) receive the plan values when non-null; plan may be null only
 * when the fused kernel takes the shape (16-bit caches, head_dim 64/128/256),
 * otherwise it is the buffer of the two-launch path.  max_width =
 * history_budget; recent_window as in dsb_build_history_plan. */
int dsb_rebuild_working_cache(
    const void *raw_key, const void *raw_value, void *working_key, void *working_value,
    const int32_t *row_slots, const int32_t *committed_lens, int32_t rows,
    const int32_t *sel_chunks, int32_t sel_stride, const int32_t *sel_count,
    int32_t num_slots, int32_t chunk_size, int32_t history_budget, int32_t recent_window,
    int32_t plan_width, int64_t *plan, int32_t *history_lens, int32_t *working_lens,
    const void *cos_sin_cache, int32_t cos_sin_dtype, int64_t cos_sin_stride,
    int64_t cos_sin_rows, int64_t max_model_len, int32_t num_heads, int32_t head_dim,
    int32_t working_budget, int32_t rotary_dim, int32_t is_neox_style, int32_t dtype,
    int32_t *error_flag, void *stream);

/* Paged gather at selected token ids with RoPE at local positions 0..W-1
 * (gather_raw_kv_with_local_rope, diffspec/kernels.py:153-210).  Ids < 0 give
 * zero rows (which still take a local position).  Outputs are
 * [batch, working_tokens, num_heads, head_dim]. */
int dsb_gather_raw_kv_with_local_rope(
    const void *raw_key_cache, const void *raw_value_cache, int64_t num_blocks,
    int32_t block_size, int32_t num_heads, int32_t head_dim,
    const int32_t *block_table, int64_t block_table_stride, int64_t block_table_cols,
    const int64_t *selected_token_indices, int32_t batch, int32_t working_tokens,
    const void *cos_sin_cache, int32_t cos_sin_dtype, int64_t cos_sin_stride,
    int64_t cos_sin_rows, int32_t rotary_dim, int32_t is_neox_style, int32_t dtype,
    void *out_key, void *out_value, int32_t *error_flag, void *stream);

/* Draft decode attention over capacity-sized working caches
 * (_forward_linear_attention_npu, diffspec/runtime.py:2079-2134; CPU loop
 * :2040-2077).  With p_r = positions[r] + position_offset, row r writes
 * key[r]/value[r] into slot slots[r] at local position p_r and attends over
 * positions 0..p_r with a softmax of scale * q.k; rows r in [rows, out_rows)
 * get zero output.  position_offset lets the K draft steps of one cycle share
 * the plan's history_len vector (step j passes j).
 * Split-KV: each (row, kv head) is cut into num_splits pieces whose partial
 * softmax states go to `scratch` (dsb_draft_attention_scratch_floats floats);
 * the last piece to finish merges them.  `counters` holds rows * num_kv_heads
 * int32 that must be zero before the first call; every call leaves them
 * zero.  Calls sharing scratch/counters must not overlap on the GPU. */
int dsb_draft_decode_attention(
    const void *query, const void *key, const void *value, void *working_key,
    void *working_value, const int32_t *slots, const int32_t *positions,
    int32_t position_offset, int32_t rows, int32_t out_rows, int32_t num_slots, int32_t num_query_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t working_budget, float scale,
    int32_t dtype, void *output, float *scratch, int64_t scratch_floats,
    int32_t *counters, int32_t num_splits, int32_t *error_flag, void *stream);

/* dsb_draft_decode_attention for callers that cannot allocate device memory
 * (no counterpart in the reference).  A serving engine that reserves almost
 * all free memory for its KV cache up front, a step recorded during CUDA
 * stream capture, or a latency-bound caller that cannot absorb a possibly
 * device-synchronising cudaMalloc/cudaFree cannot provide the split scratch
 * and tickets that dsb_draft_decode_attention takes.  This variant uses the
 * library's own file-scope device arrays instead: 1048576 floats (4 MiB) of
 * split partials and 4096 tickets, held by every GPU that loads the library
 * until the process exits, and calls no allocating routine.  Calls needing
 * more scratch (rows * kv_heads * splits * padded heads * (2 + head_dim)
 * floats) or more than 4096 rows * kv_heads are rejected with
 * DSB_ERR_INVALID.  num_splits <= 0 picks the library default.  The first
 * call on a device looks the arrays' device addresses up (cudaGetSymbolAddress,
 * with that device current); make that first call before any stream capture.
 * Every call shares the arrays and clears the tickets it uses with a
 * memset on `stream`, so calls that overlap on the GPU (other streams,
 * concurrent graphs) race and must be serialised by the caller. */
int dsb_draft_decode_attention_static(
    const void *query, const void *key, const void *value, void *working_key,
    void *working_value, const int32_t *slots, const int32_t *positions,
    int32_t position_offset, int32_t rows, int32_t out_rows, int32_t num_slots,
    int32_t num_query_heads, int32_t num_kv_heads, int32_t head_dim,
    int32_t working_budget, float scale, int32_t dtype, void *output,
    int32_t num_splits, int32_t *error_flag, void *stream);

/* Split count the library would choose and the scratch size it then needs. */
int32_t dsb_draft_attention_default_splits(int32_t rows, int32_t num_kv_heads,
                                           int32_t working_budget, int32_t sm_count);
int64_t dsb_draft_attention_scratch_floats(int32_t rows, int32_t num_query_heads,
                                           int32_t num_kv_heads, int32_t head_dim,
                                           int32_t num_splits);

/* Draft-layer KV projection with the canonical raw-KV write in its epilogue:
 * the producer side of the draft-context path, replacing the projection ->
 * temporary -> _write_raw copy of diffspec/runtime.py:1602-1618 (fed by the
 * Eagle3 sink op, diffspec/vllm_patch.py:132-178).  out[t, f] =
 * sum_k hidden[t, k] * weight[f, k] (fp32 accumulation on the tensor cores,
 * rounded once to the cache dtype) for f < 2 * num_kv_heads * head_dim; the
 * first half of each output row is K, the second V.  The same values go to
 * raw_key / raw_value [num_slots, max_model_len, num_kv_heads, head_dim] at
 * [slots[t], positions[t]] (slots[t] < 0: padding, no cache row; bad slots or
 * positions set DSB_FLAG_SLOT / DSB_FLAG_POSITION).  hidden [tokens,
 * hidden_size] and weight [2 * num_kv_heads * head_dim, hidden_size] are
 * contiguous and 16-byte aligned; hidden_size is a multiple of 64 up to 65536
 * and num_kv_heads * head_dim a multiple of 128.  out (nullable) is
 * [tokens, 2 * num_kv_heads * head_dim]. */
int dsb_kv_projection_write_raw(
    const void *hidden, int32_t tokens, int32_t hidden_size, const void *weight,
    int32_t num_kv_heads, int32_t head_dim, const int32_t *slots, const int64_t *positions,
    void *raw_key, void *raw_value, int32_t num_slots, int64_t max_model_len, int32_t dtype,
    void *out, int32_t *error_flag, void *stream);

/* Target-model paged decode attention with the softmax LSE exported (the
 * FIA call with softmax_lse_flag of diffspec/ascend_patch.py:191-240 whose
 * LSE capture_target_attention keeps, diffspec/runtime.py:841-894).  For
 * query row r (block-table row table_rows[r], or r when table_rows is NULL;
 * the first seq_lens[r] tokens of that row visible) and query head h of kv
 * group h / (num_query_heads / num_kv_heads):
 *   out[r, h] = softmax(scale * q[r, h] . K^T) V      (rounded to dtype)
 *   lse[r, h] = log(sum_t exp(scale * q[r, h] . k_t))  (fp32, natural log;
 *               -inf and a zero output for an empty row)
 * query / out [query_rows, num_query_heads, 128]; caches [num_blocks,
 * block_size, num_kv_heads, 128]; block_table [block_table_rows,
 * block_table_cols] with row stride block_table_stride.  max_seq_len bounds
 * seq_lens and sets the split count (ceil(max_seq_len / tokens_per_split);
 * tokens_per_split <= 0 picks 1024 when max_seq_len >= 16384, else 512, in
 * this call and in dsb_paged_decode_scratch_floats alike); scratch holds
 * dsb_paged_decode_scratch_floats floats.  Bad table rows set DSB_FLAG_SLOT,
 * bad page entries DSB_FLAG_BLOCK (the token is skipped), a seq_lens entry
 * above the split count's reach (max_seq_len too small) DSB_FLAG_POSITION
 * (the row is cut there). */
int64_t dsb_paged_decode_scratch_floats(int32_t query_rows, int32_t num_query_heads,
                                        int32_t max_seq_len, int32_t tokens_per_split);
int dsb_paged_decode_attention_lse(
    const void *query, int32_t query_rows, int32_t num_query_heads, int32_t num_kv_heads,
    int32_t head_dim, const void *key_cache, const void *value_cache, int64_t num_blocks,
    int32_t block_size, const int32_t *block_table, int64_t block_table_stride,
    int64_t block_table_rows, int64_t block_table_cols, const int32_t *seq_lens,
    const int32_t *table_rows, int32_t max_seq_len, float scale, int32_t dtype,
    int32_t tokens_per_split, void *out, float *lse, float *scratch, int64_t scratch_floats,
    int32_t *error_flag, void *stream);

/* Epilogues and flags of the draft-layer linear entry points. */
#define DSB_LINEAR_PLAIN 0    /* out = x . W^T                                 */
#define DSB_LINEAR_RESIDUAL 1 /* out = x . W^T + residual (one rounding)       */
#define DSB_LINEAR_SWIGLU 2   /* out = silu(gate) * up of a gate/up-interleaved W */
#define DSB_LINEAR_PARTIAL_F32 3 /* out (float) = x . W^T unrounded: one rank's share
                                    of a row-split linear, for an fp32 all-reduce */
/* Request the weight before the previous kernel in the stream has finished
 * (programmatic dependent launch): the weight must not be written by that
 * kernel.  Activations, residuals and outputs are touched only after it. */
#define DSB_LINEAR_PREFETCH_WEIGHT 1
/* The weight is in the tile-packed layout of dsb_pack_linear_weight (every
 * 128-row x 64-column block the kernel streams is one contiguous 16 KB run,
 * already in its shared-memory image, staged by one bulk copy) instead of
 * row-major [rows, in_features]. */
#define DSB_LINEAR_PACKED_WEIGHT 2
/* With DSB_LINEAR_PREFETCH_WEIGHT: also request each CTA's next four weight
 * blocks past its ring into L2 before that wait, so HBM keeps streaming
 * while the previous kernel finishes.  Faster for a linear alone; it puts
 * more of the weight in L2, so leave it off where another kernel's working
 * set must stay in L2. */
#define DSB_LINEAR_PREFETCH_L2 4

/* Copy a row-major [rows, cols] weight (rows a multiple of 128, cols of 64;
 * BF16 or FP16, 16-byte aligned) into the tile-packed layout the linear
 * entry points read with DSB_LINEAR_PACKED_WEIGHT: block (m, kb) of 128 x 64
 * elements is stored contiguously at block index m * (cols / 64) + kb, row r
 * of it at 128 r bytes, its 16-byte piece p (elements 8 p .. 8 p + 7 of
 * weight[128 m + r][64 kb ..]) at piece position p ^ (r % 8) (the 128-byte
 * swizzle of the tensor cores' shared-memory operand layout).  A one-time,
 * load-time step (no counterpart
 * in the reference, whose projections are vLLM linear layers); out must not
 * alias weight.  The copy completes before the next kernel in the stream
 * starts, so a linear launch with DSB_LINEAR_PREFETCH_WEIGHT may follow it
 * directly. */
int dsb_pack_linear_weight(const void *weight, int64_t rows, int32_t cols, int32_t dtype,
                           void *out, void *stream);

/* The draft layer's query + K/V projection in one launch (vLLM
 * QKVParallelLinear of the Eagle3 layer, qkv input built at
 * diffspec/vllm_patch.py:189-225; K/V handed pre-RoPE to the canonical cache
 * by the sink op, vllm_patch.py:132-178 -> _write_raw, runtime.py:1602-1618).
 * weight is [q_features + 2 * num_kv_heads * head_dim, hidden_size]: query
 * rows, then K rows, then V rows.  q_out [tokens, q_features] receives the
 * query features; kv_out (nullable) [tokens, 2 * num_kv_heads * head_dim]
 * and the raw caches (as dsb_kv_projection_write_raw) the K/V features.
 * q_features is a multiple of 128 (0: K/V only). */
int dsb_qkv_projection_write_raw(
    const void *hidden, int32_t tokens, int32_t hidden_size, const void *weight,
    int32_t q_features, int32_t num_kv_heads, int32_t head_dim, const int32_t *slots,
    const int64_t *positions, void *raw_key, void *raw_value, int32_t num_slots,
    int64_t max_model_len, int32_t dtype, void *q_out, void *kv_out, int32_t flags,
    int32_t *error_flag, void *stream);

/* A linear layer of a draft decode step (the Eagle3 layer's o_proj,
 * gate_up_proj + SiluAndMul, down_proj): out[t, f] = sum_k x[t, k] *
 * weight[f, k] with fp32 accumulation, x [tokens, in_features] and weight
 * [weight_rows, in_features] contiguous and 16-byte aligned, in_features a
 * multiple of 64 (up to 65536), weight_rows a multiple of 128.
 * DSB_LINEAR_RESIDUAL adds residual[t, f] before the one rounding.
 * DSB_LINEAR_SWIGLU takes weight rows in 128-row tiles whose first 64 rows
 * are gate rows and last 64 the up rows of the same 64 output features
 * (tile i: gate rows 64 i .. 64 i + 63, then the matching up rows); the gate
 * and up values are rounded to the storage type and out[t, f] =
 * round(round(silu(gate)) * up) for f < weight_rows / 2 (vLLM SiluAndMul).  Row strides are in
 * elements. */
int dsb_draft_linear(const void *x, int32_t tokens, int32_t in_features, const void *weight,
                     int32_t weight_rows, int32_t epilogue, const void *residual,
                     int64_t residual_row_stride, void *out, int64_t out_row_stride,
                     int32_t dtype, int32_t flags, int32_t *error_flag, void *stream);

/* Elementwise stages of one draft decoder layer (the vLLM Eagle3 Llama layer
 * of the diffspec draft model, qkv input built at diffspec/vllm_patch.py:
 * 189-225; RoPE at the working cache's local positions, diffspec/runtime.py:
 * 1767-1794).  The reference runs each as eager tensor ops; these are one
 * launch apiece.
 *
 * dsb_rms_norm: out[r] = round(round(x[r] * rsqrt(mean(x[r]^2) + eps)) *
 * weight), fp32 math rounded where vLLM's rms_norm rounds, for rows r < rows
 * of cols elements (row strides in elements,
 * multiples of 8; cols a multiple of 8; 16-byte aligned; out must not
 * overlap x). */
int dsb_rms_norm(const void *x, int64_t x_row_stride, const void *weight, void *out,
                 int64_t out_row_stride, int32_t rows, int32_t cols, float eps, int32_t dtype,
                 void *stream);

/* dsb_add_rms_norm: the step after an all-reduced row-split linear.
 * x_out[r] = round(partial[r] + residual[r]) (fp32 partial, one rounding, as
 * the DSB_LINEAR_RESIDUAL epilogue of the whole linear rounds) and, when
 * weight is set, out[r] = rms_norm(x_out[r]) with dsb_rms_norm's arithmetic
 * bit for bit.  Row strides in elements (multiples of 8, >= cols), cols a
 * multiple of 8, 16-byte aligned rows; no counterpart in the reference
 * (vLLM's fused_add_rms_norm after a tensor-parallel all-reduce). */
int dsb_add_rms_norm(const float *partial, int64_t partial_row_stride, const void *residual,
                     int64_t residual_row_stride, const void *weight, void *x_out,
                     int64_t x_row_stride, void *out, int64_t out_row_stride, int32_t rows,
                     int32_t cols, float eps, int32_t dtype, void *stream);

/* dsb_rope_qk: NeoX rotation at positions[t] of a [cos | sin] table with
 * rotary_rows rows (products rounded before the add, as in the working-cache
 * rebuild) of one step's query heads, in place ([tokens, num_query_heads,
 * head_dim] with row stride query_row_stride), and of its key heads, read
 * from key (row stride key_row_stride, e.g. the packed rows of
 * dsb_kv_projection_write_raw) and written to key_out as contiguous [tokens,
 * num_kv_heads, head_dim] (key_out == key: in place, contiguous rows only).
 * With value non-NULL the value heads (row stride value_row_stride) are
 * copied unchanged to value_out in the same layout.  Token t is rotated at
 * positions[t] + position_offset (the K draft steps of one cycle share the
 * plan's history lengths, step j passing j, as in
 * dsb_draft_decode_attention); a position outside [0, rotary_rows) leaves
 * its rows unrotated and sets DSB_FLAG_POSITION.  Strides are in elements. */
int dsb_rope_qk(void *query, int64_t query_row_stride, int32_t num_query_heads,
                const void *key, int64_t key_row_stride, void *key_out,
                const void *value, int64_t value_row_stride, void *value_out,
                int32_t num_kv_heads, int32_t head_dim, const int32_t *positions,
                int32_t position_offset, int32_t tokens, const void *cos_sin, int64_t cos_sin_row_stride,
                int32_t rotary_rows, int32_t cos_sin_dtype, int32_t dtype,
                int32_t *error_flag, void *stream);

/* dsb_silu_mul: out[r, i] = round(round(silu(gate_up[r, i])) * gate_up[r,
 * intermediate + i]) for i < intermediate (fp32 math rounded where vLLM's
 * SiluAndMul rounds; the gate and up projections in one GEMM output).  intermediate and row strides are
 * multiples of 8 and rows 16-byte aligned. */
int dsb_silu_mul(const void *gate_up, int64_t gate_up_row_stride, void *out,
                 int64_t out_row_stride, int32_t rows, int32_t intermediate, int32_t dtype,
                 void *stream);

/* Committed-query pick of the retrieval hook
 * (_accept_target_queries, diffspec/runtime.py:1211-1276): for each of `rows`
 * real requests with query span [query_ends[r-1], query_ends[r]) and count
 * accepted tokens, query_index = start + clamp(count - 1, 0, len - 1) and
 * retrieval_len = target_seq_len - len + min(max(count, 1), len).  Rows with
 * count <= 0 get retrieval_len 0 and row_slots -1.  counts is int64 when
 * counts_are_int64, else int32.  status[0] (retrievals run) or status[1]
 * (skipped: nothing committed) is incremented when status is non-NULL. */
int dsb_prepare_retrieval_rows(
    const int32_t *query_ends, const int32_t *target_seq_lens, const void *counts,
    int32_t counts_are_int64, const int32_t *active_slots, int32_t rows,
    int32_t *query_index, int32_t *retrieval_lens, int32_t *row_slots,
    int32_t *status, void *stream);

/* Canonical pre-RoPE KV write (_write_raw, diffspec/runtime.py:1602-1618):
 * raw[slots[i], positions[i]] = kv[i] for i < tokens; slots[i] < 0 skips. */
int dsb_write_raw_kv(
    const void *key, const void *value, void *raw_key, void *raw_value,
    const int32_t *slots, const int64_t *positions, int32_t tokens,
    int32_t num_slots, int64_t max_model_len, int32_t num_heads, int32_t head_dim,
    int32_t dtype, int32_t *error_flag, void *stream);

/* The draft step's KV sink (capture_raw_kv, diffspec/runtime.py:1797-1877,
 * with _write_raw :1602-1618 and the position buffer of
 * graph_safe_rope_positions :1767-1794): rows i < tokens are the active
 * requests, whose key/value rows (row stride kv_row_stride elements, e.g.
 * the packed K/V of a projection) go to raw_key / raw_value at [slots[i],
 * positions[i]] (slots[i] < 0: no cache row) and whose local RoPE position
 * local_positions[i] = history_lens[i] + position_offset is returned
 * (DSB_FLAG_CAPACITY when it reaches working_budget), and working_lens
 * (nullable, [num_slots]) of its slot becomes that position + 1, the length
 * once the step's token is stored (as forward_attention leaves it,
 * runtime.py:2057-2058); rows tokens <= i < padded_tokens are graph padding:
 * no cache row, local position 0.  positions and local_positions are int64
 * when positions_are_int64, else int32; local_positions may be NULL (write
 * only). */
int dsb_capture_raw_kv(
    const void *key, const void *value, int64_t kv_row_stride, void *raw_key, void *raw_value,
    const int32_t *slots, const void *positions, int32_t positions_are_int64, int32_t tokens,
    int32_t padded_tokens, int32_t num_slots, int64_t max_model_len, int32_t num_heads,
    int32_t head_dim, int32_t dtype, const int32_t *history_lens, int32_t position_offset,
    int32_t working_budget, void *local_positions, int32_t *working_lens, int32_t *error_flag,
    void *stream);

/* Fused row-split linear + all-reduce over NVLink peer memory, for a
 * tensor-parallel draft layer (the all-reduce of vLLM's RowParallelLinear in
 * the Eagle3 layer the reference drafts through, diffspec/proposer.py:97-119).
 * Each rank owns one exchange buffer per all-reduce site, of
 * dsb_peer_buffer_bytes(world, tokens_max, features) bytes, created zeroed by
 * dsb_peer_buffer_create and mapped into the other ranks' processes with
 * dsb_ipc_handle / dsb_ipc_open (plain peer mappings; no multicast).
 * dsb_draft_linear_peer computes x . W^T like dsb_draft_linear and stores
 * each fp32 sum, tagged with the call's number in the same 8-byte store, into
 * this rank's slot of every rank's buffer (peer_bases[q] = rank q's buffer as
 * mapped in this process, a device array of world addresses; own_base = this
 * rank's buffer).  dsb_peer_add_rms_norm on each rank reads every rank's
 * partials from its own buffer as their tags show them arrived (a wait
 * bounded by time: DSB_FLAG_TIMEOUT, and the sums are then not meaningful),
 * sums them in rank order and finishes as dsb_add_rms_norm with that sum as
 * `partial`.  Every rank must issue the same sequence of
 * dsb_draft_linear_peer / dsb_peer_add_rms_norm calls on a site, alternating,
 * each on one stream; the call count lives in the buffer, so the sequence can
 * be captured and replayed as a CUDA graph.  world <= 8, features a multiple
 * of 8; weight_rows of the linear = features; tokens <= tokens_max. */
#define DSB_IPC_HANDLE_BYTES 64
int64_t dsb_peer_buffer_bytes(int32_t world, int32_t tokens_max, int32_t features);
int dsb_peer_buffer_create(int32_t world, int32_t tokens_max, int32_t features, void **base);
int dsb_peer_buffer_destroy(void *base);
int dsb_ipc_handle(void *base, void *handle);
int dsb_ipc_open(const void *handle, void **base);
int dsb_ipc_close(void *base);
int dsb_draft_linear_peer(const void *x, int32_t tokens, int32_t in_features, const void *weight,
                          int32_t weight_rows, const uint64_t *peer_bases, int32_t world,
                          int32_t rank, int32_t tokens_max, void *own_base, int32_t dtype,
                          int32_t flags, int32_t *error_flag, void *stream);
/* All-gather over the same buffers, created with tokens_max 1 and features =
 * count_max: dsb_peer_all_gather_send stores this rank's `count` floats,
 * tagged with the call's number, into its slot of every rank's buffer;
 * dsb_peer_all_gather_recv, after it on each rank, writes out[world][count]
 * (rank-major, what an NCCL all_gather_into_tensor gives) from its own buffer
 * once the tags show every rank's values arrived (bounded by time:
 * DSB_FLAG_TIMEOUT).  Replaces the NCCL all-gather of the per-kv-head chunk
 * mass of a head-sharded retrieval (the reference's all-reduce of scores,
 * diffspec/runtime.py:1292-1297).  count and count_max multiples of 8; the
 * send / receive pairs of a site alternate on every rank, as above. */
int dsb_peer_all_gather_send(const float *src, int64_t count, const uint64_t *peer_bases,
                             int32_t world, int32_t rank, int64_t count_max, void *own_base,
                             void *stream);
int dsb_peer_all_gather_recv(void *own_base, int32_t world, int64_t count, int64_t count_max,
                             float *out, int32_t *error_flag, void *stream);
int dsb_peer_add_rms_norm(void *own_base, int32_t world, int32_t tokens_max, const void *residual,
                          int64_t residual_row_stride, const void *weight, void *x_out,
                          int64_t x_row_stride, void *out, int64_t out_row_stride, int32_t rows,
                          int32_t cols, float eps, int32_t dtype, int32_t *error_flag,
                          void *stream);

/* Request slots on the device (set_active_requests, diffspec/runtime.py:
 * 755-778).  slot_keys[num_slots] is the slot table, kept on the device
 * between calls: the key of the request owning each slot, negative when the
 * slot is free (initialise it to -1).  request_keys[num_requests] are the
 * batch's requests in batch order, as non-negative keys that identify a
 * request for as long as it lives (the host interns its request ids).  One
 * launch (one CTA):
 *   1. releases every slot whose key is not in the batch: the key becomes -1,
 *      sel_count[slot] = -1 and working_lens[slot] = 0 (either may be NULL);
 *   2. gives every key new to the table the lowest free slot, in batch order
 *      of its first occurrence (a duplicated key shares its slot);
 *   3. writes active_slots[i], the slot of request i (-1 for a request left
 *      without one).
 * A key already in the table keeps its slot.  If more new keys arrive than
 * there are free slots, those that fit in batch order are assigned and
 * status[0] = how many were left without one (the reference raises at the
 * first, after the same releases and assignments); status[1] = free slots
 * after the call (status may be NULL).  A negative request key sets
 * DSB_FLAG_SLOT and gets slot -1.  num_slots and num_requests at most 4096. */
int dsb_assign_request_slots(int64_t *slot_keys, int32_t num_slots,
                             const int64_t *request_keys, int32_t num_requests,
                             int32_t *active_slots, int32_t *sel_count, int32_t *working_lens,
                             int32_t *status, int32_t *error_flag, void *stream);

/* slots[i] = active_slots[rows[i]] for i < n: the canonical slot of each
 * token of a pass from its batch row (the token -> slot map of
 * populate_prefill, diffspec/runtime.py:1336-1347).  A row outside
 * [0, num_active) gives slot -1 (no cache row) and sets DSB_FLAG_SLOT. */
int dsb_rows_to_slots(const int32_t *active_slots, int32_t num_active, const int32_t *rows,
                      int32_t n, int32_t *slots, int32_t *error_flag, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* DIFFSPEC_B200_H_ */
