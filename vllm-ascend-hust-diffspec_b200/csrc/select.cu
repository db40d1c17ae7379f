// Device chunk selection (DiffSpec row A4): exact top-k by radix select.
//
// Reference: select_context_chunks, diffspec/runtime.py:348-414, applied per
// request by set_chunk_scores :1554-1567 and the loop at :1298-1308.  A
// rolling recent window of WC chunks (window mode, no reference counterpart;
// WC = 1 is the reference) leaves the newest WC chunks out of the ranking.  The
// reference runs torch.topk + sort per request on the host's behalf; here one
// CTA per row finds the (S-1)-th largest score with a 4-pass 8-bit radix
// select on order-preserving 32-bit keys, then emits the winners in ascending
// chunk order with two block scans.  Equal scores at the threshold are taken
// from the lowest chunk index upwards, so the result is a pure function of the
// score vector (torch.topk leaves that order unspecified).
#include <cmath>

#include "common.cuh"

namespace dsb {
namespace {

constexpr int kThreads = 512;
constexpr int kWarpsSel = kThreads / 32;

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// Where the score parts of a row lie: part p = q * per_group + i sits at
// row + q * group_stride + i * part_stride (one group: the [rows, parts, N]
// layout; world groups: the [world, rows, parts / world, N] layout of an
// all-gather of per-rank parts).
struct PartsLayout {
  int64_t part_stride, group_stride;
  int num_parts, per_group;
};

__device__ __forceinline__ float chunk_score(const float *__restrict__ row, const PartsLayout &pl,
                                             int normalize_heads, int L, int C, int c) {
  float s = 0.f;
  for (int p = 0; p < pl.num_parts; ++p) {
    const int q = p / pl.per_group, i = p - q * pl.per_group;
    s += row[(int64_t)q * pl.group_stride + (int64_t)i * pl.part_stride + c];
  }
  if (normalize_heads > 0) {
    const int nv = max(0, min(C, L - c * C));
    s = (nv > 0) ? s / (float)nv / (float)normalize_heads : 0.f;
  }
  return s;
}

// Exclusive block scan of one int per thread; returns the block total.
__device__ __forceinline__ int block_exclusive_scan(int v, int *warp_tot, int &excl) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = (lane < kWarpsSel) ? warp_tot[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    if (lane < kWarpsSel) warp_tot[lane] = wi - w;  // exclusive warp offsets
    if (lane == kWarpsSel - 1) warp_tot[kWarpsSel] = wi;
  }
  __syncthreads();
  excl = warp_tot[warp] + incl - v;
  const int total = warp_tot[kWarpsSel];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kThreads)
select_chunks_kernel(const float *__restrict__ parts, int64_t row_stride, const PartsLayout pl,
                     int normalize_heads, const int32_t *__restrict__ seq_lens,
                     const int32_t *__restrict__ row_slots, int max_chunks, int C, int S, int WC,
                     int32_t *__restrict__ sel_chunks, int sel_stride,
                     int32_t *__restrict__ sel_count, int num_slots,
                     int64_t *__restrict__ out_ci, int64_t *__restrict__ out_ti,
                     float *__restrict__ out_cs, int32_t *err) {
  pdl_begin();
  extern __shared__ uint32_t keys[];  // [max_chunks] order keys, then [S] chosen ids
  int32_t *chosen = reinterpret_cast<int32_t *>(keys + max_chunks);
  __shared__ int hist[256];
  __shared__ int warp_tot[kWarpsSel + 1];
  __shared__ int sh_digit, sh_greater;

  const int row = blockIdx.x;
  const int slot = (row_slots != nullptr) ? row_slots[row] : row;
  if (slot < 0) return;  // row not committed: selection left unchanged
  const int L = max(0, seq_lens[row]);
  int n = (L + C - 1) / C;
  if (n > max_chunks) {
    if (threadIdx.x == 0) flag_error(err, DSB_FLAG_CAPACITY);
    n = max_chunks;
  }
  const float *srow = parts + (int64_t)row * row_stride;
  int count;
  if (n <= S) {
    for (int i = threadIdx.x; i < n; i += kThreads) chosen[i] = i;
    count = n;
  } else {
    // Rank chunks 0..n-1-WC (the newest WC chunks are the rolling window's;
    // WC = 1 is the reference) for S - WC places; chunk n-1 is always kept.
    const int m = n - WC;
    const int k = S - WC;
    for (int i = threadIdx.x; i < m; i += kThreads)
      keys[i] = order_key(chunk_score(srow, pl, normalize_heads, L, C, i));
    __syncthreads();
    uint32_t prefix = 0, pmask = 0;
    int k_rem = k;
    if (k > 0) {
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < m; i += kThreads) {
          const uint32_t u = keys[i];
          if ((u & pmask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
          const int lane = threadIdx.x;
          int loc[8], lsum = 0;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            loc[j] = hist[lane * 8 + j];
            lsum += loc[j];
          }
          int incl = lsum;  // sum over lanes >= lane
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_down_sync(0xffffffffu, incl, o);
            if (lane + o < 32) incl += v;
          }
          int cum = incl - lsum;  // keys in higher bins
#pragma unroll
          for (int j = 7; j >= 0; --j) {
            if (cum < k_rem && cum + loc[j] >= k_rem) {
              sh_digit = lane * 8 + j;
              sh_greater = cum;
            }
            cum += loc[j];
          }
        }
        __syncthreads();
        prefix |= (uint32_t)sh_digit << shift;
        pmask |= 255u << shift;
        k_rem -= sh_greater;
        __syncthreads();
      }
    }
    const uint32_t thr = prefix;
    const int need_eq = k_rem;  // keys equal to thr that are taken, lowest index first
    const int per = (m + kThreads - 1) / kThreads;
    const int i0 = min(m, (int)threadIdx.x * per), i1 = min(m, i0 + per);
    int n_eq = 0;
    if (k > 0)
      for (int i = i0; i < i1; ++i) n_eq += (keys[i] == thr);
    int eq_base;
    block_exclusive_scan(n_eq, warp_tot, eq_base);
    int n_sel = 0;
    if (k > 0) {
      int r = eq_base;
      for (int i = i0; i < i1; ++i) {
        const uint32_t u = keys[i];
        if (u > thr) ++n_sel;
        else if (u == thr) n_sel += (r++ < need_eq);
      }
    }
    int pos;
    block_exclusive_scan(n_sel, warp_tot, pos);
    if (k > 0) {
      int r = eq_base;
      for (int i = i0; i < i1; ++i) {
        const uint32_t u = keys[i];
        bool take = false;
        if (u > thr) take = true;
        else if (u == thr) take = (r++ < need_eq);
        if (take) chosen[pos++] = i;
      }
    }
    if (threadIdx.x == 0) chosen[k] = n - 1;
    count = k + 1;
  }
  __syncthreads();

  if (sel_count != nullptr && sel_chunks != nullptr) {
    if (slot >= num_slots || count > sel_stride) {
      if (threadIdx.x == 0) flag_error(err, slot >= num_slots ? DSB_FLAG_SLOT : DSB_FLAG_CAPACITY);
    } else {
      for (int i = threadIdx.x; i < count; i += kThreads)
        sel_chunks[(int64_t)slot * sel_stride + i] = chosen[i];
      if (threadIdx.x == 0) sel_count[slot] = count;
    }
  }
  if (out_ci != nullptr)
    for (int i = threadIdx.x; i < S; i += kThreads)
      out_ci[(int64_t)row * S + i] = (i < count) ? chosen[i] : -1;
  if (out_cs != nullptr)
    for (int i = threadIdx.x; i < S; i += kThreads)
      out_cs[(int64_t)row * S + i] =
          (i < count) ? chunk_score(srow, pl, normalize_heads, L, C, chosen[i]) : 0.f;
  if (out_ti != nullptr) {
    for (int j = threadIdx.x; j < S * C; j += kThreads) {
      const int i = j / C, o = j % C;
      int64_t v = -1;
      if (i < count - 1) v = (int64_t)chosen[i] * C + o;
      else if (i == count - 1) {
        const int64_t tok = (int64_t)(n - 1) * C + o;
        v = (tok < L) ? tok : -1;
      }
      out_ti[(int64_t)row * S * C + j] = v;
    }
  }
  (void)key_value;
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int dsb_select_context_chunks(
    const float *parts, int64_t row_stride, int64_t part_stride, int32_t num_parts,
    int32_t parts_per_group, int64_t group_stride, int32_t normalize_heads,
    const int32_t *seq_lens, const int32_t *row_slots, int32_t rows, int32_t max_chunks,
    int32_t chunk_size, int32_t history_budget, int32_t recent_window, int32_t *sel_chunks,
    int32_t sel_stride, int32_t *sel_count, int32_t num_slots, int64_t *out_chunk_indices,
    int64_t *out_token_indices, float *out_chunk_scores, int32_t *error_flag, void *stream) {
  if (rows < 0 || max_chunks < 0 || num_parts < 0) return fail(DSB_ERR_INVALID, "negative sizes");
  if (rows == 0) return DSB_OK;
  if (!seq_lens || (max_chunks > 0 && !parts)) return fail(DSB_ERR_INVALID, "null pointer argument");
  if (chunk_size <= 0 || history_budget < chunk_size || history_budget % chunk_size)
    return fail(DSB_ERR_INVALID, "token_budget must be a positive chunk-size multiple");
  if (parts_per_group <= 0) parts_per_group = num_parts > 0 ? num_parts : 1;
  if (num_parts % parts_per_group)
    return fail(DSB_ERR_INVALID, "num_parts must be a multiple of parts_per_group");
  if (recent_window == 0) recent_window = chunk_size;
  if (recent_window < chunk_size || recent_window % chunk_size || recent_window > history_budget)
    return fail(DSB_ERR_INVALID,
                "recent_window must be a chunk-size multiple in [chunk_size, token_budget]");
  const int S = history_budget / chunk_size;
  if ((sel_chunks != nullptr) != (sel_count != nullptr))
    return fail(DSB_ERR_INVALID, "sel_chunks and sel_count go together");
  if (sel_chunks != nullptr && (sel_stride < S || num_slots <= 0))
    return fail(DSB_ERR_INVALID, "selection state narrower than token_budget / chunk_size");
  const size_t smem = sizeof(uint32_t) * ((size_t)max_chunks + (size_t)S);
  if (smem > 220 * 1024) return fail(DSB_ERR_UNSUPPORTED, "too many chunks for one CTA");
  if (int st_ = ensure_smem((const void *)select_chunks_kernel, smem); st_ != DSB_OK) return st_;
  const PartsLayout pl{part_stride, group_stride, num_parts, parts_per_group};
  launch_kernel(select_chunks_kernel, dim3(rows), dim3(kThreads), smem, as_stream(stream),
      parts, row_stride, pl, normalize_heads, seq_lens, row_slots, max_chunks, chunk_size, S,
      recent_window / chunk_size, sel_chunks, sel_stride, sel_count, num_slots,
      out_chunk_indices, out_token_indices, out_chunk_scores, error_flag);
  return check_launch("select_chunks_kernel");
}
