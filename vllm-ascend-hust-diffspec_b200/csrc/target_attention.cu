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
  int page_tiles;  // 1: page size and split length multiples of 16 (a tile lies in one page)
  float scale_log2;
  float *part;  // [rows, hq, splits, D + 2]: acc[D], max, sum
  void *out;
  float *lse;
  int32_t *err;
};

constexpr int kTaTile = 16;                    // tokens per warp tile
constexpr int kTaStages = 3;                   // tiles in a warp's ring (2 in flight while one computes)
constexpr int kTaRowBytes = kTaD * 2 + 16;     // staged K/V row, padded: ldmatrix without conflicts
constexpr int kTaStageBytes = 2 * kTaTile * kTaRowBytes;           // K tile + V tile
constexpr int kTaRingBytes = kTaWarps * kTaStages * kTaStageBytes;  // 104,448 B: 2 CTAs per SM

template <int G> struct TaSmem {
  static constexpr int kMerge = kTaWarps * G * kTaD * 4 + kTaWarps * 16 * 2 * 4;
  static constexpr int kBytes = kMerge > kTaRingBytes ? kMerge : kTaRingBytes;
};

// 16 bytes of a staged row: a cp.async (L2 only) from `src`, or zeros stored
// directly when the row has no source.  A zero store never meets a copy in
// flight to the same bytes: a stage is refilled only after the wait on its
// previous fill.
__device__ __forceinline__ void ta_cp16_or_zero(uint32_t dst, const void *src, bool valid) {
  if (valid)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
  else
    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0u) : "memory");
}

__device__ __forceinline__ void ta_ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ta_ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Split-KV partial of one (split, kv head, row) on the tensor cores
// (mma.sync m16n8k16, fp32 accumulate).  The split's 16-token tiles go
// round-robin to the four warps; each warp streams its tiles through a
// private 3-stage cp.async ring (K and V rows of a tile staged in padded
// shared memory, two tiles in flight while the third is computed) and per
// tile computes
//   S[16 heads x 16 tokens] = Q . K^T   (A = the group's query heads from
//                                         registers, rows >= G zero; B = the
//                                         K rows by ldmatrix)
// then the base-2 online softmax on S's accumulators, and
//   O[16 heads x 128] += P . V          (A = P from S's accumulators, split
//                                         into hi + lo 16-bit terms; B = the
//                                         V rows by ldmatrix.trans).
// Rows past the split (or past seq_lens) are zero-filled and masked; a page
// entry outside the cache is flagged and its tokens read as zeros.
template <typename T, int G>
__global__ void __launch_bounds__(kTaWarps * 32, 2) paged_decode_split_kernel(const TaArgs a) {
  static_assert(G <= 16, "at most 16 query heads per kv head");
  extern __shared__ __align__(128) uint8_t s_raw[];  // rings, then the warps' states
  pdl_begin();
  // kv head fastest: the Hk CTAs of one (split, row) read the quarters of
  // the same token rows, and run side by side (DRAM row locality)
  const int h = blockIdx.x, split = blockIdx.y, r = blockIdx.z;
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

  // Q A-fragments of the 8 k-steps: rows g and g + 8 are query heads
  // h * G + g (+ 8) when < G; columns 16 s + 2 t (+ 8).
  uint32_t qa[8][4];
  {
    const T *qb = static_cast<const T *>(a.q) + ((int64_t)r * a.hq + h * G) * kTaD;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int c = 16 * s + 2 * t;
      qa[s][0] = g < G ? *reinterpret_cast<const uint32_t *>(qb + g * kTaD + c) : 0u;
      qa[s][1] = g + 8 < G ? *reinterpret_cast<const uint32_t *>(qb + (g + 8) * kTaD + c) : 0u;
      qa[s][2] = g < G ? *reinterpret_cast<const uint32_t *>(qb + g * kTaD + c + 8) : 0u;
      qa[s][3] = g + 8 < G ? *reinterpret_cast<const uint32_t *>(qb + (g + 8) * kTaD + c + 8) : 0u;
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
  const uint32_t ring = smem_u32(s_raw) + warp * kTaStages * kTaStageBytes;
  const int64_t tok_stride = (int64_t)a.hk * kTaD;  // elements between consecutive tokens of a page
  bool bad = false;

  // Stage tile k of this split: instruction i moves K and V rows 2 i and
  // 2 i + 1 (lanes 0-15 and 16-31, 16 bytes each).  When every tile lies in
  // one page (page size and split length multiples of 16), one table entry
  // serves the tile; otherwise each row looks up its own.
  auto issue = [&](int k, int stage) {
    const int T0 = s0 + kTaTile * k;
    const uint32_t kd = ring + stage * kTaStageBytes, vd = kd + kTaTile * kTaRowBytes;
    const int col = lane & 15;
    int64_t tile_base = -1;
    if (a.page_tiles) {
      const int blk = row_bt[T0 / a.bs];
      if (blk >= 0 && blk < a.nblocks)
        tile_base = (((int64_t)blk * a.bs + T0 % a.bs) * a.hk + h) * kTaD;
      else
        bad = true;
    }
#pragma unroll
    for (int i = 0; i < kTaTile / 2; ++i) {
      const int row = 2 * i + (lane >> 4), tok = T0 + row;
      int64_t off = -1;
      if (tok < s1) {
        if (a.page_tiles) {
          if (tile_base >= 0) off = tile_base + row * tok_stride;
        } else {
          const int blk = row_bt[tok / a.bs];
          if (blk >= 0 && blk < a.nblocks)
            off = (((int64_t)blk * a.bs + tok % a.bs) * a.hk + h) * kTaD;
          else
            bad = true;
        }
      }
      const int64_t src = off >= 0 ? off + 8 * col : 0;
      ta_cp16_or_zero(kd + row * kTaRowBytes + col * 16, kc + src, off >= 0);
      ta_cp16_or_zero(vd + row * kTaRowBytes + col * 16, vc + src, off >= 0);
    }
  };

  const int ntiles = s1 > s0 ? (s1 - s0 + kTaTile - 1) / kTaTile : 0;
  const int mine = ntiles > warp ? (ntiles - warp + kTaWarps - 1) / kTaWarps : 0;
#pragma unroll
  for (int i = 0; i < kTaStages - 1; ++i) {
    if (i < mine) issue(warp + kTaWarps * i, i);
    cp_async_commit();
  }
  for (int i = 0; i < mine; ++i) {
    {
      const int nxt = i + kTaStages - 1;  // into the stage computed last iteration
      if (nxt < mine) issue(warp + kTaWarps * nxt, nxt % kTaStages);
      cp_async_commit();
    }
    cp_async_wait<kTaStages - 1>();
    __syncwarp();
    const int T0 = s0 + kTaTile * (warp + kTaWarps * i);
    const uint32_t kb = ring + (i % kTaStages) * kTaStageBytes, vb = kb + kTaTile * kTaRowBytes;

    // ---- S = Q K^T: 8 k-steps, both 8-token n-tiles from one ldmatrix.x4
    float ce[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    float co[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const uint32_t k_lane = kb + (((lane >> 4) & 1) * 8 + (lane & 7)) * kTaRowBytes +
                            ((lane >> 3) & 1) * 16;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      uint32_t kf[4];
      ta_ldsm_x4(kf, k_lane + s * 32);
      const uint32_t b0[2] = {kf[0], kf[1]}, b1[2] = {kf[2], kf[3]};
      Mma<T>::run((s & 1) ? co[0] : ce[0], qa[s], b0);
      Mma<T>::run((s & 1) ? co[1] : ce[1], qa[s], b1);
    }
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tok = T0 + 8 * nt + 2 * t + (j & 1);
        sc[nt][j] = tok < s1 ? (ce[nt][j] + co[nt][j]) * a.scale_log2 : -INFINITY;
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
    // ---- O += P V: two 8-dim n-tiles per ldmatrix.x4.trans
    const uint32_t v_lane = vb + (lane & 15) * kTaRowBytes + (lane >> 4) * 16;
#pragma unroll
    for (int dn = 0; dn < 16; dn += 2) {
      uint32_t vf[4];
      ta_ldsm_x4_trans(vf, v_lane + dn * 16);
      const uint32_t b0[2] = {vf[0], vf[1]}, b1[2] = {vf[2], vf[3]};
      Mma<T>::run(o[dn], ph, b0);
      Mma<T>::run(o[dn], pl, b0);
      Mma<T>::run(o[dn + 1], ph, b1);
      Mma<T>::run(o[dn + 1], pl, b1);
    }
    __syncwarp();  // the stage is refilled next iteration
  }
  cp_async_wait<0>();
  if (bad) flag_error(a.err, DSB_FLAG_BLOCK);

  // Warp state -> shared memory (rows < G), then merge the four warps.
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
  }
  __syncthreads();  // every warp is done with its ring
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

template <typename T, int G> int launch_group(const TaArgs &a, cudaStream_t st) {
  auto kern = paged_decode_split_kernel<T, G>;
  constexpr size_t smem = TaSmem<G>::kBytes;
  if (int e = ensure_smem((const void *)kern, smem); e != DSB_OK) return e;
  launch_kernel(kern, dim3(a.hk, a.splits, a.rows), dim3(kTaWarps * 32), smem, st, a);
  return DSB_OK;
}

template <typename T> int launch_typed(const TaArgs &a, int group, cudaStream_t st) {
  int e = DSB_OK;
  switch (group) {
    case 1: e = launch_group<T, 1>(a, st); break;
    case 2: e = launch_group<T, 2>(a, st); break;
    case 4: e = launch_group<T, 4>(a, st); break;
    case 8: e = launch_group<T, 8>(a, st); break;
    case 16: e = launch_group<T, 16>(a, st); break;
    default: return fail(DSB_ERR_UNSUPPORTED, "query heads per kv head must be 1, 2, 4, 8 or 16");
  }
  if (e != DSB_OK) return e;
  if (int e2 = check_launch("paged_decode_split_kernel")) return e2;
  launch_kernel(paged_decode_merge_kernel<T>, dim3((unsigned)(a.rows * a.hq)), dim3(kTaD), 0, st,
                a);
  return check_launch("paged_decode_merge_kernel");
}

// The split length when the caller passes <= 0: 1024 tokens for long
// contexts (max_seq_len >= 16384: fewer CTA ramp-ups and a smaller merge;
// 266 us against 313 us at 16 rows x 40960 tokens), 512 otherwise (more
// splits to fill the GPU when the rows are short).
int32_t default_tokens_per_split(int32_t max_seq_len) {
  return max_seq_len >= 16384 ? 1024 : 512;
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
  if (tokens_per_split <= 0) tokens_per_split = default_tokens_per_split(max_seq_len);
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
  if (tokens_per_split <= 0) tokens_per_split = default_tokens_per_split(max_seq_len);
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
  a.page_tiles = (block_size % kTaTile == 0 && tokens_per_split % kTaTile == 0) ? 1 : 0;
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
