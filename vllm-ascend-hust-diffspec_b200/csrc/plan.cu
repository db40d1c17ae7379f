// Small per-request kernels of the draft cycle: compact history plans (A5),
// the committed-query pick of the retrieval hook (A3) and the canonical raw-KV
// write with the draft step's local RoPE positions (A9).  All of them keep the reference's host Python loops on the
// device so a draft cycle needs no device-to-host copy.
#include "common.cuh"
#include "plan_row.cuh"

namespace dsb {
namespace {

// One warp per plan row (plan_row_warp).
__global__ void build_plan_kernel(const int32_t *__restrict__ row_slots,
                                  const int32_t *__restrict__ committed_lens, int rows,
                                  const int32_t *__restrict__ sel_chunks, int sel_stride,
                                  const int32_t *__restrict__ sel_count, int num_slots, int C,
                                  int HB, int window, int plan_width, int64_t *__restrict__ plan,
                                  int32_t *__restrict__ history_lens,
                                  int32_t *__restrict__ working_lens, int32_t *err) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  int64_t *out = plan + (int64_t)r * plan_width;
  const int slot = (row_slots != nullptr) ? row_slots[r] : r;
  if (slot < 0 || slot >= num_slots) {
    if (lane == 0) flag_error(err, DSB_FLAG_SLOT);
    for (int i = lane; i < plan_width; i += 32) out[i] = 0;
    if (lane == 0 && history_lens != nullptr) history_lens[r] = 0;
    return;
  }
  const int32_t *ch = sel_chunks + (int64_t)slot * sel_stride;
  const PlanRow pr = plan_row_warp(committed_lens[r], sel_count[slot], ch, sel_stride, C, HB,
                                   window, plan_width, lane, err);
  for (int i = lane; i < plan_width; i += 32) out[i] = plan_row_value(pr, slot, ch, i);
  if (lane == 0) {
    if (history_lens != nullptr) history_lens[r] = (int32_t)pr.hlen;
    if (working_lens != nullptr) working_lens[slot] = (int32_t)pr.hlen;
  }
}

// _accept_target_queries, diffspec/runtime.py:1211-1276 (linear proposals).
__global__ void prepare_rows_kernel(const int32_t *__restrict__ query_ends,
                                    const int32_t *__restrict__ target_seq_lens,
                                    const void *__restrict__ counts, int counts64,
                                    const int32_t *__restrict__ active_slots, int rows,
                                    int32_t *__restrict__ query_index,
                                    int32_t *__restrict__ retrieval_lens,
                                    int32_t *__restrict__ row_slots, int32_t *status) {
  pdl_begin();
  __shared__ int any;
  if (threadIdx.x == 0) any = 0;
  __syncthreads();
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const int start = (r == 0) ? 0 : query_ends[r - 1];
    const int qlen = query_ends[r] - start;
    const int64_t cnt = counts64 ? static_cast<const int64_t *>(counts)[r]
                                 : (int64_t) static_cast<const int32_t *>(counts)[r];
    if (cnt > 0 && qlen > 0) {
      const int off = (int)min(max(cnt - 1, (int64_t)0), (int64_t)(qlen - 1));
      const int committed = (int)min(max(cnt, (int64_t)1), (int64_t)qlen);
      query_index[r] = start + off;
      retrieval_lens[r] = target_seq_lens[r] - qlen + committed;
      row_slots[r] = active_slots[r];
      any = 1;
    } else {
      query_index[r] = max(start, 0);
      retrieval_lens[r] = 0;
      row_slots[r] = -1;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && status != nullptr) {
    if (any) status[0] += 1;
    else status[1] += 1;
  }
}

// One warp per token row: raw[slot, pos] = kv[i].
__global__ void write_raw_kernel(const uint4 *__restrict__ key, const uint4 *__restrict__ value,
                                 uint4 *__restrict__ raw_key, uint4 *__restrict__ raw_value,
                                 const int32_t *__restrict__ slots,
                                 const int64_t *__restrict__ positions, int tokens,
                                 int num_slots, int64_t max_model_len, int row_vecs,
                                 int32_t *err) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= tokens) return;
  const int slot = slots[i];
  if (slot < 0) return;
  const int64_t pos = positions[i];
  if (slot >= num_slots || pos < 0 || pos >= max_model_len) {
    if (lane == 0) flag_error(err, slot >= num_slots ? DSB_FLAG_SLOT : DSB_FLAG_POSITION);
    return;
  }
  const int64_t dst = ((int64_t)slot * max_model_len + pos) * row_vecs;
  const int64_t src = (int64_t)i * row_vecs;
  for (int v = lane; v < row_vecs; v += 32) {
    raw_key[dst + v] = key[src + v];
    raw_value[dst + v] = value[src + v];
  }
}

// The draft step's KV sink (capture_raw_kv, diffspec/runtime.py:1797-1877):
// one warp per token row.  Rows i < tokens are real requests: their K/V go to
// raw[slots[i], positions[i]], local_positions[i] = history_lens[i] +
// position_offset (the local RoPE position the step's keys take) and the
// slot's working length becomes local_positions[i] + 1; rows
// tokens <= i < padded_tokens are graph padding: no cache row, position 0.
template <typename P>
__global__ void capture_raw_kernel(const uint4 *__restrict__ key, const uint4 *__restrict__ value,
                                   int64_t kv_row_vecs, uint4 *__restrict__ raw_key,
                                   uint4 *__restrict__ raw_value,
                                   const int32_t *__restrict__ slots,
                                   const P *__restrict__ positions, int tokens, int padded,
                                   int num_slots, int64_t max_model_len, int row_vecs,
                                   const int32_t *__restrict__ history_lens, int offset,
                                   int working_budget, P *__restrict__ local_positions,
                                   int32_t *__restrict__ working_lens, int32_t *err) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= padded) return;
  if (i >= tokens) {
    if (lane == 0 && local_positions != nullptr) local_positions[i] = 0;
    return;
  }
  const int slot = slots[i];
  if (lane == 0 && local_positions != nullptr) {
    const int64_t lp = (int64_t)history_lens[i] + offset;
    if (lp < 0 || lp >= working_budget) flag_error(err, DSB_FLAG_CAPACITY);
    local_positions[i] = (P)lp;
    // the slot's working length once this step's token is stored
    if (working_lens != nullptr && slot >= 0 && slot < num_slots) working_lens[slot] = (int32_t)(lp + 1);
  }
  if (slot < 0) return;
  const int64_t pos = (int64_t)positions[i];
  if (slot >= num_slots || pos < 0 || pos >= max_model_len) {
    if (lane == 0) flag_error(err, slot >= num_slots ? DSB_FLAG_SLOT : DSB_FLAG_POSITION);
    return;
  }
  const int64_t dst = ((int64_t)slot * max_model_len + pos) * row_vecs;
  const int64_t src = (int64_t)i * kv_row_vecs;
  for (int v = lane; v < row_vecs; v += 32) {
    raw_key[dst + v] = key[src + v];
    raw_value[dst + v] = value[src + v];
  }
}

int elem_size(int dtype) { return dtype == DSB_F32 ? 4 : 2; }

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int dsb_build_history_plan(const int32_t *row_slots, const int32_t *committed_lens,
                                      int32_t rows, const int32_t *sel_chunks,
                                      int32_t sel_stride, const int32_t *sel_count,
                                      int32_t num_slots, int32_t chunk_size,
                                      int32_t history_budget, int32_t recent_window,
                                      int32_t plan_width, int64_t *plan, int32_t *history_lens,
                                      int32_t *working_lens, int32_t *error_flag,
                                      void *stream) {
  if (rows < 0) return fail(DSB_ERR_INVALID, "negative rows");
  if (rows == 0) return DSB_OK;
  if (!committed_lens || !sel_chunks || !sel_count || !plan)
    return fail(DSB_ERR_INVALID, "null pointer argument");
  if (chunk_size <= 0 || history_budget <= 0 || plan_width < 5 || sel_stride <= 0 ||
      num_slots <= 0)
    return fail(DSB_ERR_INVALID, "bad chunk size, budget, plan width or selection stride");
  if (recent_window == 0) recent_window = chunk_size;
  if (recent_window < chunk_size || recent_window % chunk_size || recent_window > history_budget)
    return fail(DSB_ERR_INVALID,
                "recent_window must be a chunk-size multiple in [chunk_size, history_budget]");
  launch_kernel(build_plan_kernel, dim3((rows + 3) / 4), dim3(128), 0, as_stream(stream),
      row_slots, committed_lens, rows, sel_chunks, sel_stride, sel_count, num_slots,
      chunk_size, history_budget, recent_window, plan_width, plan, history_lens, working_lens,
      error_flag);
  return check_launch("build_plan_kernel");
}

extern "C" int dsb_prepare_retrieval_rows(const int32_t *query_ends,
                                          const int32_t *target_seq_lens, const void *counts,
                                          int32_t counts_are_int64,
                                          const int32_t *active_slots, int32_t rows,
                                          int32_t *query_index, int32_t *retrieval_lens,
                                          int32_t *row_slots, int32_t *status, void *stream) {
  if (rows < 0) return fail(DSB_ERR_INVALID, "negative rows");
  if (rows == 0) return DSB_OK;
  if (!query_ends || !target_seq_lens || !counts || !active_slots || !query_index ||
      !retrieval_lens || !row_slots)
    return fail(DSB_ERR_INVALID, "null pointer argument");
  launch_kernel(prepare_rows_kernel, dim3(1), dim3(256), 0, as_stream(stream),
      query_ends, target_seq_lens, counts, counts_are_int64, active_slots, rows, query_index,
      retrieval_lens, row_slots, status);
  return check_launch("prepare_rows_kernel");
}

extern "C" int dsb_write_raw_kv(const void *key, const void *value, void *raw_key,
                                void *raw_value, const int32_t *slots,
                                const int64_t *positions, int32_t tokens, int32_t num_slots,
                                int64_t max_model_len, int32_t num_heads, int32_t head_dim,
                                int32_t dtype, int32_t *error_flag, void *stream) {
  if (tokens < 0) return fail(DSB_ERR_INVALID, "negative token count");
  if (tokens == 0) return DSB_OK;
  if (!key || !value || !raw_key || !raw_value || !slots || !positions)
    return fail(DSB_ERR_INVALID, "null pointer argument");
  if (dtype != DSB_BF16 && dtype != DSB_F16 && dtype != DSB_F32)
    return fail(DSB_ERR_INVALID, "unknown dtype");
  const int64_t row_bytes = (int64_t)num_heads * head_dim * elem_size(dtype);
  if (num_heads <= 0 || head_dim <= 0 || row_bytes % 16)
    return fail(DSB_ERR_UNSUPPORTED, "KV row must be a multiple of 16 bytes");
  const int warps = 8;
  launch_kernel(write_raw_kernel, dim3((tokens + warps - 1) / warps), dim3(warps * 32), 0, as_stream(stream),
      static_cast<const uint4 *>(key), static_cast<const uint4 *>(value),
      static_cast<uint4 *>(raw_key), static_cast<uint4 *>(raw_value), slots, positions, tokens,
      num_slots, max_model_len, (int)(row_bytes / 16), error_flag);
  return check_launch("write_raw_kernel");
}

extern "C" int dsb_capture_raw_kv(const void *key, const void *value, int64_t kv_row_stride,
                                  void *raw_key, void *raw_value, const int32_t *slots,
                                  const void *positions, int32_t positions_are_int64,
                                  int32_t tokens, int32_t padded_tokens, int32_t num_slots,
                                  int64_t max_model_len, int32_t num_heads, int32_t head_dim,
                                  int32_t dtype, const int32_t *history_lens,
                                  int32_t position_offset, int32_t working_budget,
                                  void *local_positions, int32_t *working_lens,
                                  int32_t *error_flag, void *stream) {
  if (tokens < 0 || padded_tokens < tokens)
    return fail(DSB_ERR_INVALID, "token counts must satisfy 0 <= tokens <= padded_tokens");
  if (padded_tokens == 0) return DSB_OK;
  if (tokens > 0 && (!key || !value || !raw_key || !raw_value || !slots || !positions))
    return fail(DSB_ERR_INVALID, "null pointer argument");
  if (local_positions != nullptr && tokens > 0 && !history_lens)
    return fail(DSB_ERR_INVALID, "local positions need the rows' history lengths");
  if (dtype != DSB_BF16 && dtype != DSB_F16 && dtype != DSB_F32)
    return fail(DSB_ERR_INVALID, "unknown dtype");
  const int64_t row_elems = (int64_t)num_heads * head_dim;
  const int64_t row_bytes = row_elems * elem_size(dtype);
  if (num_heads <= 0 || head_dim <= 0 || row_bytes % 16)
    return fail(DSB_ERR_UNSUPPORTED, "KV row must be a multiple of 16 bytes");
  if (kv_row_stride < row_elems || (kv_row_stride * elem_size(dtype)) % 16)
    return fail(DSB_ERR_INVALID, "key/value row stride must cover a row and keep 16-byte rows");
  if (max_model_len <= 0 || num_slots <= 0 || working_budget <= 0)
    return fail(DSB_ERR_INVALID, "cache geometry must be positive");
  const int warps = 8;
  const dim3 grid((padded_tokens + warps - 1) / warps), block(warps * 32);
  const int64_t kv_vecs = kv_row_stride * elem_size(dtype) / 16;
  if (positions_are_int64)
    launch_kernel(capture_raw_kernel<int64_t>, grid, block, 0, as_stream(stream),
        static_cast<const uint4 *>(key), static_cast<const uint4 *>(value), kv_vecs,
        static_cast<uint4 *>(raw_key), static_cast<uint4 *>(raw_value), slots,
        static_cast<const int64_t *>(positions), tokens, padded_tokens, num_slots, max_model_len,
        (int)(row_bytes / 16), history_lens, position_offset, working_budget,
        static_cast<int64_t *>(local_positions), working_lens, error_flag);
  else
    launch_kernel(capture_raw_kernel<int32_t>, grid, block, 0, as_stream(stream),
        static_cast<const uint4 *>(key), static_cast<const uint4 *>(value), kv_vecs,
        static_cast<uint4 *>(raw_key), static_cast<uint4 *>(raw_value), slots,
        static_cast<const int32_t *>(positions), tokens, padded_tokens, num_slots, max_model_len,
        (int)(row_bytes / 16), history_lens, position_offset, working_budget,
        static_cast<int32_t *>(local_positions), working_lens, error_flag);
  return check_launch("capture_raw_kernel");
}
