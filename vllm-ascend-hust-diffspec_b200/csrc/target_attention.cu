// Target-model paged decode attention that also exports the softmax LSE.
//
// Reference: the target verifier's attention runs as FIA with
// softmax_lse_flag forced on (diffspec/ascend_patch.py:191-240) so that
// capture_target_attention (diffspec/runtime.py:841-894) can keep the LSE
// for the chunk-retrieval scores (kernels.py:11-150 divides by exp(lse)).
// On B200 the LSE falls out of a flash-decode epilogue: this kernel computes
//   out[r, h]  = sum_t softmax_t(scale * q[r, h] . k_t) v_t
//   lse[r, h]  = log sum_t exp(scale * q[r, h] . k_t)          (natural log)
// over the first seq_lens[r] tokens of the row's paged K/V, so retrieval
// can score chunks with it instead of running its own LSE pass.
//
// B200 design: decode attention is bound by the K/V stream (2 * D * 2 bytes
// per token and kv head).  Split-KV: CTA (split, kv head, row) streams
// tokens_per_split tokens of one kv head for all G = Hq / Hk query heads of
// the group (the K/V rows are read once per group, not once per query
// head); a warp takes every fourth token, lane l holding elements
// 4l..4l+3 of the K and V rows (256-byte coalesced rows), two tokens in
// flight per warp; online softmax in base 2 per query head.  The warps'
// states merge in shared memory and each CTA writes one (max, sum, acc[D])
// partial per query head; a second launch merges the splits in order
// (deterministic) and writes out and lse.  No waits on other CTAs.
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace dsb {
namespace {

constexpr int kTaD = 128;       // head_dim handled
constexpr int kTaWarps = 4;
constexpr float kTaLog2e = 1.4426950408889634f;
constexpr float kTaLn2 = 0.6931471805599453f;

struct TaArgs {
  const void *q, *k, *v;
  const int32_t *bt, *seq, *trows;
  int64_t bt_stride, bt_cols, bt_rows, nblocks;
  int bs, hq, hk, rows, splits, tps;
  float scale_log2;
  float *part;  // [rows, hq, splits, D + 2]: acc[D], max, sum
  void *out;
  float *lse;
  int32_t *err;
};

template <typename T>
__device__ __forceinline__ void load4(const T *p, float (&f)[4]) {
  const uint2 w = *reinterpret_cast<const uint2 *>(p);
  const float2 a = unpack2<T>(w.x), b = unpack2<T>(w.y);
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

template <typename T, int G>
__global__ void __launch_bounds__(kTaWarps * 32) paged_decode_split_kernel(const TaArgs a) {
  __shared__ float s_m[kTaWarps][G], s_l[kTaWarps][G];
  __shared__ float s_acc[kTaWarps][G][kTaD];
  pdl_begin();
  const int split = blockIdx.x, h = blockIdx.y, r = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int L = a.seq[r];
  const int trow = a.trows != nullptr ? a.trows[r] : r;
  if (trow < 0 || trow >= a.bt_rows) {
    if (threadIdx.x == 0 && split == 0 && h == 0) flag_error(a.err, DSB_FLAG_SLOT);
    L = 0;
  }
  const int64_t cap = a.bt_cols * a.bs;  // tokens the table row can address
  if ((int64_t)L > cap) L = (int)cap;
  if (L < 0) L = 0;
  const int s0 = split * a.tps, s1 = min(L, s0 + a.tps);

  float q[G][4], m[G], l[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    load4(static_cast<const T *>(a.q) + ((int64_t)r * a.hq + h * G + g) * kTaD + 4 * lane, q[g]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      q[g][j] *= a.scale_log2;
      acc[g][j] = 0.f;
    }
    m[g] = -INFINITY;
    l[g] = 0.f;
  }
  const T *kc = static_cast<const T *>(a.k), *vc = static_cast<const T *>(a.v);
  const int32_t *row_bt = a.bt + (int64_t)trow * a.bt_stride;

  // One token: its K/V row offset, or -1 when the page entry is bad.
  auto row_of = [&](int t) -> int64_t {
    const int blk = row_bt[t / a.bs];
    if (blk < 0 || blk >= a.nblocks) return -1;
    return (((int64_t)blk * a.bs + t % a.bs) * a.hk + h) * kTaD + 4 * lane;
  };
  auto consume = [&](const float (&kf)[4], const float (&vf)[4]) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s = q[g][0] * kf[0];
      s = fmaf(q[g][1], kf[1], s);
      s = fmaf(q[g][2], kf[2], s);
      s = fmaf(q[g][3], kf[3], s);
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float mn = fmaxf(m[g], s);
      const float c = exp2f(m[g] - mn), p = exp2f(s - mn);
      l[g] = fmaf(l[g], c, p);
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[g][j] = fmaf(acc[g][j], c, p * vf[j]);
      m[g] = mn;
    }
  };

  bool bad = false;
  int t = s0 + warp;
  for (; t + kTaWarps < s1; t += 2 * kTaWarps) {  // two tokens in flight
    const int64_t o0 = row_of(t), o1 = row_of(t + kTaWarps);
    float k0[4] = {0.f, 0.f, 0.f, 0.f}, v0[4] = {0.f, 0.f, 0.f, 0.f};
    float k1[4] = {0.f, 0.f, 0.f, 0.f}, v1[4] = {0.f, 0.f, 0.f, 0.f};
    if (o0 >= 0) {
      load4(kc + o0, k0);
      load4(vc + o0, v0);
    }
    if (o1 >= 0) {
      load4(kc + o1, k1);
      load4(vc + o1, v1);
    }
    if (o0 >= 0) consume(k0, v0); else bad = true;
    if (o1 >= 0) consume(k1, v1); else bad = true;
  }
  if (t < s1) {
    const int64_t o0 = row_of(t);
    if (o0 >= 0) {
      float k0[4], v0[4];
      load4(kc + o0, k0);
      load4(vc + o0, v0);
      consume(k0, v0);
    } else {
      bad = true;
    }
  }
  if (bad && lane == 0) flag_error(a.err, DSB_FLAG_BLOCK);

  // Merge the four warps' states, then write this split's partial.
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) s_acc[warp][g][4 * lane + j] = acc[g][j];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * kTaD; i += kTaWarps * 32) {
    const int g = i / kTaD, d = i % kTaD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTaWarps; ++w) M = fmaxf(M, s_m[w][g]);
    float sum = 0.f, ac = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kTaWarps; ++w) {
        const float f = exp2f(s_m[w][g] - M);
        sum = fmaf(s_l[w][g], f, sum);
        ac = fmaf(s_acc[w][g][d], f, ac);
      }
    }
    float *p = a.part + (((int64_t)r * a.hq + h * G + g) * a.splits + split) * (kTaD + 2);
    p[d] = ac;
    if (d == 0) {
      p[kTaD] = M;
      p[kTaD + 1] = sum;
    }
  }
}

// One CTA per (row, query head), thread = output element: merge the splits
// in order.
template <typename T>
__global__ void __launch_bounds__(kTaD) paged_decode_merge_kernel(const TaArgs a) {
  pdl_begin();
  const int64_t rh = blockIdx.x;  // r * hq + head
  const int d = threadIdx.x;
  const float *p = a.part + rh * a.splits * (kTaD + 2);
  float M = -INFINITY;
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, p[s * (kTaD + 2) + kTaD]);
  float sum = 0.f, ac = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < a.splits; ++s) {
      const float *q = p + s * (kTaD + 2);
      const float f = exp2f(q[kTaD] - M);
      sum = fmaf(q[kTaD + 1], f, sum);
      ac = fmaf(q[d], f, ac);
    }
  }
  const float y = sum > 0.f ? ac / sum : 0.f;
  static_cast<T *>(a.out)[rh * kTaD + d] = Elem<T>::from_f(y);
  if (d == 0) a.lse[rh] = sum > 0.f ? (M + log2f(sum)) * kTaLn2 : -INFINITY;
}

template <typename T, int G> void launch_group(const TaArgs &a, cudaStream_t st) {
  launch_kernel(paged_decode_split_kernel<T, G>, dim3(a.splits, a.hk, a.rows),
                dim3(kTaWarps * 32), 0, st, a);
}

template <typename T> int launch_typed(const TaArgs &a, int group, cudaStream_t st) {
  switch (group) {
    case 1: launch_group<T, 1>(a, st); break;
    case 2: launch_group<T, 2>(a, st); break;
    case 4: launch_group<T, 4>(a, st); break;
    case 8: launch_group<T, 8>(a, st); break;
    case 16: launch_group<T, 16>(a, st); break;
    default: return fail(DSB_ERR_UNSUPPORTED, "query heads per kv head must be 1, 2, 4, 8 or 16");
  }
  if (int e = check_launch("paged_decode_split_kernel")) return e;
  launch_kernel(paged_decode_merge_kernel<T>, dim3((unsigned)(a.rows * a.hq)), dim3(kTaD), 0, st,
                a);
  return check_launch("paged_decode_merge_kernel");
}

int splits_for(int32_t max_seq_len, int32_t tokens_per_split) {
  return std::max(1, (max_seq_len + tokens_per_split - 1) / tokens_per_split);
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int64_t dsb_paged_decode_scratch_floats(int32_t query_rows, int32_t num_query_heads,
                                                    int32_t max_seq_len, int32_t tokens_per_split) {
  if (query_rows <= 0 || num_query_heads <= 0 || max_seq_len < 0 || tokens_per_split <= 0) return 0;
  return (int64_t)query_rows * num_query_heads * splits_for(max_seq_len, tokens_per_split) *
         (kTaD + 2);
}

extern "C" int dsb_paged_decode_attention_lse(
    const void *query, int32_t query_rows, int32_t num_query_heads, int32_t num_kv_heads,
    int32_t head_dim, const void *key_cache, const void *value_cache, int64_t num_blocks,
    int32_t block_size, const int32_t *block_table, int64_t block_table_stride,
    int64_t block_table_rows, int64_t block_table_cols, const int32_t *seq_lens,
    const int32_t *table_rows, int32_t max_seq_len, float scale, int32_t dtype,
    int32_t tokens_per_split, void *out, float *lse, float *scratch, int64_t scratch_floats,
    int32_t *error_flag, void *stream) {
  if (query_rows < 0) return fail(DSB_ERR_INVALID, "negative query_rows");
  if (query_rows == 0) return DSB_OK;
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_INVALID, "query and caches must be BF16 or FP16");
  if (num_query_heads <= 0 || num_kv_heads <= 0 || num_query_heads % num_kv_heads)
    return fail(DSB_ERR_INVALID, "query heads must be a positive multiple of kv heads");
  if (head_dim != kTaD) return fail(DSB_ERR_UNSUPPORTED, "head_dim must be 128");
  if (num_blocks <= 0 || block_size <= 0 || block_table_rows <= 0 || block_table_cols <= 0 ||
      block_table_stride < block_table_cols || max_seq_len < 0)
    return fail(DSB_ERR_INVALID, "bad cache or block-table geometry");
  if (tokens_per_split <= 0) tokens_per_split = 512;
  if (!(scale > 0.f)) return fail(DSB_ERR_INVALID, "scale must be positive");
  if (!query || !key_cache || !value_cache || !block_table || !seq_lens || !out || !lse || !scratch)
    return fail(DSB_ERR_INVALID, "null pointer argument");
  const int splits = splits_for(max_seq_len, tokens_per_split);
  if (splits > 65535 || num_kv_heads > 65535 || query_rows > 65535)
    return fail(DSB_ERR_UNSUPPORTED, "grid too large");
  if (scratch_floats < dsb_paged_decode_scratch_floats(query_rows, num_query_heads, max_seq_len,
                                                       tokens_per_split))
    return fail(DSB_ERR_INVALID, "scratch smaller than dsb_paged_decode_scratch_floats");
  if (reinterpret_cast<uintptr_t>(query) % 8 || reinterpret_cast<uintptr_t>(key_cache) % 8 ||
      reinterpret_cast<uintptr_t>(value_cache) % 8)
    return fail(DSB_ERR_UNSUPPORTED, "query and caches must be 8-byte aligned");
  TaArgs a{};
  a.q = query;
  a.k = key_cache;
  a.v = value_cache;
  a.bt = block_table;
  a.seq = seq_lens;
  a.trows = table_rows;
  a.bt_stride = block_table_stride;
  a.bt_cols = block_table_cols;
  a.bt_rows = block_table_rows;
  a.nblocks = num_blocks;
  a.bs = block_size;
  a.hq = num_query_heads;
  a.hk = num_kv_heads;
  a.rows = query_rows;
  a.splits = splits;
  a.tps = tokens_per_split;
  a.scale_log2 = scale * kTaLog2e;
  a.part = scratch;
  a.out = out;
  a.lse = lse;
  a.err = error_flag;
  const int group = num_query_heads / num_kv_heads;
  cudaStream_t st = as_stream(stream);
  return dtype == DSB_BF16 ? launch_typed<__nv_bfloat16>(a, group, st)
                           : launch_typed<__half>(a, group, st);
}
