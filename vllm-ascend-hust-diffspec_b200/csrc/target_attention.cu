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
// head); each warp takes every fourth 16-token tile and runs it through the
// tensor cores (S = Q K^T and O += P V with mma.sync, base-2 online softmax
// on the accumulators, P split into hi + lo 16-bit terms).  The warps'
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

__device__ __forceinline__ uint32_t ta_word(const uint4 &v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

constexpr int kTaTile = 16;                // tokens per warp tile
constexpr int kTaVStride = kTaD * 2 + 16;  // bytes per staged V row (padded: ldmatrix without conflicts)
constexpr int kTaVBytes = kTaTile * kTaVStride;

template <int G> struct TaSmem {
  static constexpr int kMerge = kTaWarps * G * kTaD * 4 + kTaWarps * 16 * 2 * 4;
  static constexpr int kStage = kTaWarps * kTaVBytes;
  static constexpr int kBytes = kMerge > kStage ? kMerge : kStage;
};

// Split-KV partial of one (split, kv head, row) on the tensor cores
// (mma.sync m16n8k16, fp32 accumulate).  Per 16-token tile a warp computes
//   S[16 heads x 16 tokens] = Q . K^T   (A = the group's query heads, rows
//                                         >= G zero; B = the K rows, loaded
//                                         straight into fragments with the
//                                         head dim permuted the same way in
//                                         A and B)
// then the base-2 online softmax on S's accumulators, and
//   O[16 heads x 128] += P . V          (A = P from S's accumulators, split
//                                         into hi + lo 16-bit terms; B = V
//                                         rows staged in padded shared memory
//                                         and read with ldmatrix.trans).
template <typename T, int G>
__global__ void __launch_bounds__(kTaWarps * 32) paged_decode_split_kernel(const TaArgs a) {
  static_assert(G <= 16, "at most 16 query heads per kv head");
  // V staging during the loop, the warps' states for the merge after it
  __shared__ __align__(16) uint8_t s_raw[TaSmem<G>::kBytes];
  pdl_begin();
  const int split = blockIdx.x, h = blockIdx.y, r = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  int L = a.seq[r];
  const int trow = a.trows != nullptr ? a.trows[r] : r;
  if (trow < 0 || trow >= a.bt_rows) {
    if (threadIdx.x == 0 && split == 0 && h == 0) flag_error(a.err, DSB_FLAG_SLOT);
    L = 0;
  }
  const int64_t cap = a.bt_cols * a.bs;  // tokens the table row can address
  if ((int64_t)L > cap) {  // seq_lens[r] beyond its block-table row
    if (threadIdx.x == 0 && split == 0 && h == 0) flag_error(a.err, DSB_FLAG_POSITION);
    L = (int)cap;
  }
  if (L < 0) L = 0;
  if ((int64_t)L > (int64_t)a.splits * a.tps) {  // seq_lens[r] above max_seq_len
    if (threadIdx.x == 0 && split == 0 && h == 0) flag_error(a.err, DSB_FLAG_POSITION);
    L = a.splits * a.tps;
  }
  const int s0 = split * a.tps, s1 = min(L, s0 + a.tps);

  // Q A-fragments: rows g and g + 8 are query heads h * G + g (+ 8) when < G.
  uint4 qlo[4], qhi[4];
  {
    const T *qb = static_cast<const T *>(a.q) + ((int64_t)r * a.hq + h * G) * kTaD;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      qlo[j] = g < G ? *reinterpret_cast<const uint4 *>(qb + g * kTaD + 8 * (4 * j + t))
                     : make_uint4(0, 0, 0, 0);
      qhi[j] = g + 8 < G ? *reinterpret_cast<const uint4 *>(qb + (g + 8) * kTaD + 8 * (4 * j + t))
                         : make_uint4(0, 0, 0, 0);
    }
  }
  float o[16][4];
#pragma unroll
  for (int dn = 0; dn < 16; ++dn)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[dn][j] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;  // rows g, g + 8

  const T *kc = static_cast<const T *>(a.k), *vc = static_cast<const T *>(a.v);
  const int32_t *row_bt = a.bt + (int64_t)trow * a.bt_stride;
  uint8_t *vs = s_raw + warp * kTaVBytes;
  bool bad = false;
  // element offset of token `tok`'s row for this kv head, or -1
  auto row_of = [&](int tok) -> int64_t {
    const int blk = row_bt[tok / a.bs];
    if (blk < 0 || blk >= a.nblocks) return -1;
    return (((int64_t)blk * a.bs + tok % a.bs) * a.hk + h) * kTaD;
  };

  for (int T0 = s0 + warp * kTaTile; T0 < s1; T0 += kTaWarps * kTaTile) {
    // ---- loads: K rows of tokens T0 + g and T0 + 8 + g; V chunks to stage
    uint4 k0[4], k1[4], vv[8];
    {
      const int ta = T0 + g, tb = T0 + 8 + g;
      const int64_t oa = ta < s1 ? row_of(ta) : -2, ob = tb < s1 ? row_of(tb) : -2;
      bad |= (oa == -1) || (ob == -1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        k0[j] = oa >= 0 ? *reinterpret_cast<const uint4 *>(kc + oa + 8 * (4 * j + t))
                        : make_uint4(0, 0, 0, 0);
        k1[j] = ob >= 0 ? *reinterpret_cast<const uint4 *>(kc + ob + 8 * (4 * j + t))
                        : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {  // chunk c = lane + 32 i: row c / 16, 16-byte column c % 16
        const int c = lane + 32 * i, row = c >> 4, col = c & 15;
        const int tok = T0 + row;
        const int64_t ov = tok < s1 ? row_of(tok) : -2;
        vv[i] = ov >= 0 ? *reinterpret_cast<const uint4 *>(vc + ov + 8 * col) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = lane + 32 * i;
      *reinterpret_cast<uint4 *>(vs + (c >> 4) * kTaVStride + (c & 15) * 16) = vv[i];
    }

    // ---- S = Q K^T: two n-tiles of 8 tokens, 8 k-steps of 16 head-dim values
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float ce[4] = {0.f, 0.f, 0.f, 0.f}, co[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const int w0 = 2 * s, w1 = 2 * s + 1;
        const uint32_t af[4] = {ta_word(qlo[w0 / 4], w0 % 4), ta_word(qhi[w0 / 4], w0 % 4),
                                ta_word(qlo[w1 / 4], w1 % 4), ta_word(qhi[w1 / 4], w1 % 4)};
        const uint4 *kk = nt == 0 ? k0 : k1;
        const uint32_t bf[2] = {ta_word(kk[w0 / 4], w0 % 4), ta_word(kk[w1 / 4], w1 % 4)};
        Mma<T>::run((s & 1) ? co : ce, af, bf);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tok = T0 + 8 * nt + 2 * t + (j & 1);
        sc[nt][j] = tok < s1 ? (ce[j] + co[j]) * a.scale_log2 : -INFINITY;
      }
    }
    // ---- online softmax (rows g: j = 0, 1; rows g + 8: j = 2, 3)
    float mx_lo = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
    float mx_hi = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
    }
    // finite: token T0 is visible to every row of the tile
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    const float c_lo = exp2f(m_lo - mn_lo), c_hi = exp2f(m_hi - mn_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float p[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      p[nt][0] = exp2f(sc[nt][0] - mn_lo);
      p[nt][1] = exp2f(sc[nt][1] - mn_lo);
      p[nt][2] = exp2f(sc[nt][2] - mn_hi);
      p[nt][3] = exp2f(sc[nt][3] - mn_hi);
    }
    l_lo = l_lo * c_lo + (p[0][0] + p[0][1] + p[1][0] + p[1][1]);  // this lane's share
    l_hi = l_hi * c_hi + (p[0][2] + p[0][3] + p[1][2] + p[1][3]);
#pragma unroll
    for (int dn = 0; dn < 16; ++dn) {
      o[dn][0] *= c_lo;
      o[dn][1] *= c_lo;
      o[dn][2] *= c_hi;
      o[dn][3] *= c_hi;
    }
    uint32_t ph[4], pl[4];
    pack2_split<T>(p[0][0], p[0][1], ph[0], pl[0]);
    pack2_split<T>(p[0][2], p[0][3], ph[1], pl[1]);
    pack2_split<T>(p[1][0], p[1][1], ph[2], pl[2]);
    pack2_split<T>(p[1][2], p[1][3], ph[3], pl[3]);
    __syncwarp();
    // ---- O += P V over 16 n-tiles of 8 head-dim values
#pragma unroll
    for (int dn = 0; dn < 16; ++dn) {
      uint32_t bv[2];
      ldsm_x2_trans(bv, vs + (lane & 15) * kTaVStride + dn * 16);
      Mma<T>::run(o[dn], ph, bv);
      Mma<T>::run(o[dn], pl, bv);
    }
    __syncwarp();  // the next tile overwrites the staged V
  }
  if (bad) flag_error(a.err, DSB_FLAG_BLOCK);

  // Warp state -> shared memory (rows < G), then merge the four warps.
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
  }
  __syncthreads();  // V staging no longer needed
  float *s_acc = reinterpret_cast<float *>(s_raw);  // [warps][G][D]
  float *s_ml = s_acc + kTaWarps * G * kTaD;        // [warps][16][2]: max, sum
#pragma unroll
  for (int dn = 0; dn < 16; ++dn)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int row = g + ((j & 2) ? 8 : 0), d = 8 * dn + 2 * t + (j & 1);
      if (row < G) s_acc[(warp * G + row) * kTaD + d] = o[dn][j];
    }
  if (t == 0) {
    s_ml[(warp * 16 + g) * 2] = m_lo;
    s_ml[(warp * 16 + g) * 2 + 1] = l_lo;
    s_ml[(warp * 16 + g + 8) * 2] = m_hi;
    s_ml[(warp * 16 + g + 8) * 2 + 1] = l_hi;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * kTaD; i += kTaWarps * 32) {
    const int hh = i / kTaD, d = i % kTaD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTaWarps; ++w) M = fmaxf(M, s_ml[(w * 16 + hh) * 2]);
    float sum = 0.f, ac = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kTaWarps; ++w) {
        const float f = exp2f(s_ml[(w * 16 + hh) * 2] - M);
        sum = fmaf(s_ml[(w * 16 + hh) * 2 + 1], f, sum);
        ac = fmaf(s_acc[(w * G + hh) * kTaD + d], f, ac);
      }
    }
    float *pp = a.part + (((int64_t)r * a.hq + h * G + hh) * a.splits + split) * (kTaD + 2);
    pp[d] = ac;
    if (d == 0) {
      pp[kTaD] = M;
      pp[kTaD + 1] = sum;
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

int64_t splits_for(int32_t max_seq_len, int32_t tokens_per_split) {
  return std::max<int64_t>(1, ((int64_t)max_seq_len + tokens_per_split - 1) / tokens_per_split);
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int64_t dsb_paged_decode_scratch_floats(int32_t query_rows, int32_t num_query_heads,
                                                    int32_t max_seq_len, int32_t tokens_per_split) {
  if (query_rows <= 0 || num_query_heads <= 0 || max_seq_len < 0) return 0;
  if (tokens_per_split <= 0) tokens_per_split = 512;  // the launch's default
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
  const int64_t splits = splits_for(max_seq_len, tokens_per_split);
  if (splits > 65535 || num_kv_heads > 65535 || query_rows > 65535)
    return fail(DSB_ERR_UNSUPPORTED, "grid too large");
  if (scratch_floats < dsb_paged_decode_scratch_floats(query_rows, num_query_heads, max_seq_len,
                                                       tokens_per_split))
    return fail(DSB_ERR_INVALID, "scratch smaller than dsb_paged_decode_scratch_floats");
  if (reinterpret_cast<uintptr_t>(query) % 16 || reinterpret_cast<uintptr_t>(key_cache) % 16 ||
      reinterpret_cast<uintptr_t>(value_cache) % 16)
    return fail(DSB_ERR_UNSUPPORTED, "query and caches must be 16-byte aligned");
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
  a.splits = (int)splits;
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
