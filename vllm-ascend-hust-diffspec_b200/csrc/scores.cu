// Chunk-score retrieval over a paged K history (DiffSpec row A1/A2).
//
// Reference: diffspec/kernels.py:11-150 (Triton, one program per
// (request, chunk, query head), K re-read once per query head) and the dense
// CPU form diffspec/runtime.py:281-345.
//
// B200 design: one warp streams a contiguous run of chunks of ONE kv head and
// scores all query heads of its GQA group at once with mma.sync m16n8k16 in
// "swap-AB" form: S^T[16 tokens x 8 heads] = K[16 x D] * Q^T[D x 8].  Each K
// row is therefore read from HBM exactly once, straight into the A fragment
// registers with 16-byte loads (no shared-memory staging, no bank conflicts):
// lane (g, t) = (lane / 4, lane % 4) owns tokens g and g + 8 of the tile and
// the head-dim slab {8 * (4j + t) .. +8 : j < D/32}.  The contraction order
// over head_dim is permuted consistently for Q and K, which leaves the dot
// product unchanged; the k-steps alternate between two accumulators to halve
// the dependent mma chain.  Each 16-token tile's sum over tokens and query
// heads is reduced by a fixed shuffle tree and a chunk adds its tiles in tile
// order, so the per-(row, kv head, chunk) mass is deterministic and
// independent of how kv heads are sharded across GPUs.
//
// Measured alternatives, not kept: a per-warp cp.async ring in shared memory
// (3 tiles per warp, twice the bytes in flight, block table staged in shared
// memory) gave the same bits and ran 1 us slower (121.4 vs 120.3 us), and a
// persistent TMA-fed variant (a producer
// warp bulk-copying 16 KB pages into a 3 x 64 KB shared-memory ring, eight
// consumer warps scoring from it) ran at 148 us against this kernel's 133 us
// on the config-2 retrieval (671 MB): with ~128 KB in flight per SM the bulk
// copies saw 2-4 us of latency under full load, while 16 register-fed warps
// per SM keep more, smaller requests in flight.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>

#include "common.cuh"

namespace dsb {
namespace {

constexpr int kWarps = 8;
constexpr int kMaxChunksPerCta = 16;  // chunks of one row per CTA: 2 .. 16, chosen per launch

template <int D> struct KTile {
  uint4 lo[D / 32];  // token g of the 16-token tile
  uint4 hi[D / 32];  // token g + 8
};

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// Locate key row `tok` of kv head `kvh` in the paged cache; nullptr if the
// token is masked or its block-table entry is out of range.
template <typename T>
__device__ __forceinline__ const T *paged_row(const T *key_cache, const int32_t *bt_row,
                                              int64_t bt_cols, int block_size,
                                              int64_t num_blocks, int Hk, int D, int kvh,
                                              int tok, int32_t *err) {
  const int lb = tok / block_size;
  if (lb >= bt_cols) {
    flag_error(err, DSB_FLAG_BLOCK);
    return nullptr;
  }
  const int64_t pb = bt_row[lb];
  if (pb < 0 || pb >= num_blocks) {
    flag_error(err, DSB_FLAG_BLOCK);
    return nullptr;
  }
  const int64_t row = pb * block_size + (tok - lb * block_size);
  return key_cache + (row * Hk + kvh) * D;
}

template <typename T, int D>
__device__ __forceinline__ void load_token(uint4 (&dst)[D / 32], const T *row, int t) {
  if (row != nullptr) {
#pragma unroll
    for (int j = 0; j < D / 32; ++j) dst[j] = ldg_stream(row + 8 * (4 * j + t), l2_evict_first());
  } else {
#pragma unroll
    for (int j = 0; j < D / 32; ++j) dst[j] = make_uint4(0, 0, 0, 0);
  }
}

// (M, S) <- (M, S) merged with (m, s): running max and sum of exp2 in base 2.
__device__ __forceinline__ void merge_ms(float &M, float &S, float m, float s) {
  const float mn = fmaxf(M, m);
  S = (mn == -INFINITY) ? 0.f : S * exp2f(M - mn) + s * exp2f(m - mn);
  M = mn;
}

// One 16-token tile of one kv head.  lo / hi: this lane's head-dim words of
// tokens g and g + 8 (A fragments in the permuted order); va / vb: whether
// those tokens count.  !STATS: `mass` = the tile's sum over valid tokens and
// heads of exp2(s * scale_log2 - lse2), reduced over the warp by a fixed xor
// tree (every lane holds it).  STATS: per (n-tile, head 2t + j) the tile's
// (max, sum) merged over its 16 tokens (every lane of a column holds it).
// Both kernels below score tiles with this one function and combine tiles in
// tile order, so a chunk's value does not depend on which warp scored it.
template <typename T, int D, int NT, bool STATS>
__device__ __forceinline__ void eval_tile(const uint4 (&lo)[D / 32], const uint4 (&hi)[D / 32],
                                          bool va, bool vb, const uint32_t (&qf)[NT][D / 16][2],
                                          const float (&lse2)[NT][2], int group, float scale_log2,
                                          int t, float &mass, float (&tm)[NT][2],
                                          float (&ts)[NT][2]) {
  constexpr int KS = D / 16;
  float acc = 0.f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      tm[nt][j] = -INFINITY;
      ts[nt][j] = 0.f;
    }
    // two accumulators (even / odd k-steps) halve the dependent mma chain
    float ce[4] = {0.f, 0.f, 0.f, 0.f}, co[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const uint32_t a[4] = {word_of(lo[(2 * s) / 4], (2 * s) % 4),
                             word_of(hi[(2 * s) / 4], (2 * s) % 4),
                             word_of(lo[(2 * s + 1) / 4], (2 * s + 1) % 4),
                             word_of(hi[(2 * s + 1) / 4], (2 * s + 1) % 4)};
      Mma<T>::run((s & 1) ? co : ce, a, qf[nt][s]);
    }
    const float cf[4] = {ce[0] + co[0], ce[1] + co[1], ce[2] + co[2], ce[3] + co[3]};
    // cf: (token g, head 2t), (g, 2t+1), (g+8, 2t), (g+8, 2t+1)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int hj = j & 1;
      const bool tv = (j < 2) ? va : vb;
      const bool hv = nt * 8 + 2 * t + hj < group;
      if (!STATS) {
        if (tv && hv) acc += exp2f(fmaf(cf[j], scale_log2, -lse2[nt][hj]));
      } else if (tv && hv) {
        const float x = cf[j] * scale_log2;
        const float mn = fmaxf(tm[nt][hj], x);
        ts[nt][hj] = ts[nt][hj] * exp2f(tm[nt][hj] - mn) + exp2f(x - mn);
        tm[nt][hj] = mn;
      }
    }
  }
  if (!STATS) {
    mass = warp_sum(acc);
  } else {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {  // merge over the 8 token groups
          const float mo = __shfl_xor_sync(0xffffffffu, tm[nt][j], o);
          const float so = __shfl_xor_sync(0xffffffffu, ts[nt][j], o);
          merge_ms(tm[nt][j], ts[nt][j], mo, so);
        }
  }
}

// Q^T B fragments for one kv head (lane (g, t) holds query head g of each
// n-tile, head-dim words in the permuted order of the K A-fragments) and the
// heads' LSE in base 2.
template <typename T, int D, int NT, bool STATS>
__device__ __forceinline__ void load_query(const T *query, const float *lse, int qrow, int Hq,
                                           int group, int kvh, int g, int t,
                                           uint32_t (&qf)[NT][D / 16][2], float (&lse2)[NT][2]) {
  constexpr int KS = D / 16;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int h = nt * 8 + g;
    uint4 qv[D / 32];
    if (h < group) {
      const T *qp = query + ((int64_t)qrow * Hq + kvh * group + h) * D;
#pragma unroll
      for (int j = 0; j < D / 32; ++j) qv[j] = *reinterpret_cast<const uint4 *>(qp + 8 * (4 * j + t));
    } else {
#pragma unroll
      for (int j = 0; j < D / 32; ++j) qv[j] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      qf[nt][s][0] = word_of(qv[(2 * s) / 4], (2 * s) % 4);
      qf[nt][s][1] = word_of(qv[(2 * s + 1) / 4], (2 * s + 1) % 4);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int hh = nt * 8 + 2 * t + j;
      lse2[nt][j] = (!STATS && hh < group) ? lse[(int64_t)qrow * Hq + kvh * group + hh] * kLog2e : 0.f;
    }
  }
}

template <typename T, int D, int NT, bool STATS>
__global__ void __launch_bounds__(kWarps * 32)
chunk_scores_mma_kernel(const T *__restrict__ query, const float *__restrict__ lse,
                        const int32_t *__restrict__ query_index, int query_rows,
                        const T *__restrict__ key_cache, const int32_t *__restrict__ block_table,
                        int64_t bt_stride, int64_t bt_cols, const int32_t *__restrict__ seq_lens,
                        int Hq, int Hk, int block_size, int64_t num_blocks, int chunk,
                        int max_chunks, int cpc, float scale_log2, float *__restrict__ out,
                        float *__restrict__ out_sum, int32_t *err) {
  pdl_begin();
  constexpr int KS = D / 16;  // mma k-steps over head_dim
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int group = Hq / Hk;
  const int qrow = (query_index != nullptr) ? query_index[b] : b;
  const bool qrow_ok = qrow >= 0 && qrow < query_rows;
  if (!qrow_ok && threadIdx.x == 0 && blockIdx.x == 0 && seq_lens[b] > 0)
    flag_error(err, DSB_FLAG_POSITION);
  const int L = qrow_ok ? seq_lens[b] : 0;
  const int c_begin = blockIdx.x * cpc;
  const int n_ch = min(cpc, max_chunks - c_begin);
  if (n_ch <= 0) return;
  const int total = Hk * n_ch;  // items, kv-head major
  const int per_warp = (total + kWarps - 1) / kWarps;
  const int i_begin = warp * per_warp;
  const int i_end = min(total, i_begin + per_warp);
  const int tiles_per_chunk = chunk / 16;
  const int32_t *bt_row = block_table + (int64_t)b * bt_stride;

  uint32_t qf[NT][KS][2];
  float lse2[NT][2];
  int loaded_kvh = -1;

  for (int item = i_begin; item < i_end; ++item) {
    const int kvh = item / n_ch;
    const int c = c_begin + item % n_ch;
    const int tok0 = c * chunk;
    if (tok0 >= L) {  // chunk past the (retrieval) length: zero mass
      if (lane == 0 && !STATS) out[((int64_t)b * Hk + kvh) * max_chunks + c] = 0.f;
      if (STATS && g == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int h = nt * 8 + 2 * t + j;
            if (h < group) {
              const int64_t o = ((int64_t)b * Hq + kvh * group + h) * max_chunks + c;
              out[o] = -INFINITY;
              out_sum[o] = 0.f;
            }
          }
      }
      continue;
    }
    if (kvh != loaded_kvh) {
      load_query<T, D, NT, STATS>(query, lse, qrow, Hq, group, kvh, g, t, qf, lse2);
      loaded_kvh = kvh;
    }

    // Tiles are scored one by one and combined in tile order.
    float mass = 0.f;
    float M[NT][2], S[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        M[nt][j] = -INFINITY;
        S[nt][j] = 0.f;
      }

    // Register double buffer over the chunk's 16-token tiles.
    KTile<D> buf[2];
    auto issue = [&](KTile<D> &dst, int mt) {
      const int ta = tok0 + mt * 16 + g, tb = ta + 8;
      const T *ra = (ta < L) ? paged_row(key_cache, bt_row, bt_cols, block_size, num_blocks,
                                         Hk, D, kvh, ta, err)
                             : nullptr;
      const T *rb = (tb < L) ? paged_row(key_cache, bt_row, bt_cols, block_size, num_blocks,
                                         Hk, D, kvh, tb, err)
                             : nullptr;
      load_token<T, D>(dst.lo, ra, t);
      load_token<T, D>(dst.hi, rb, t);
    };
    auto consume = [&](const KTile<D> &src, int mt) {
      const bool va = tok0 + mt * 16 + g < L;
      const bool vb = tok0 + mt * 16 + g + 8 < L;
      float tmass, tm[NT][2], ts[NT][2];
      eval_tile<T, D, NT, STATS>(src.lo, src.hi, va, vb, qf, lse2, group, scale_log2, t, tmass,
                                 tm, ts);
      if (!STATS) {
        mass += tmass;
      } else {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) merge_ms(M[nt][j], S[nt][j], tm[nt][j], ts[nt][j]);
      }
    };

    issue(buf[0], 0);
    for (int mt = 0; mt < tiles_per_chunk; mt += 2) {
      if (mt + 1 < tiles_per_chunk) issue(buf[1], mt + 1);
      consume(buf[0], mt);
      if (mt + 1 >= tiles_per_chunk) break;
      if (mt + 2 < tiles_per_chunk) issue(buf[0], mt + 2);
      consume(buf[1], mt + 1);
    }

    if (!STATS) {
      if (lane == 0) out[((int64_t)b * Hk + kvh) * max_chunks + c] = mass;
    } else {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int h = nt * 8 + 2 * t + j;
          if (g == 0 && h < group) {
            const int64_t o = ((int64_t)b * Hq + kvh * group + h) * max_chunks + c;
            out[o] = M[nt][j];
            out_sum[o] = S[nt][j];
          }
        }
    }
  }
}

// Fallback for shapes the tensor-core kernel does not cover (head_dim not in
// {64, 128, 256}, chunk % 16 != 0, groups above 16, fp32 caches): one warp per
// (row, kv head, chunk), one lane per token, fp32 FMA.
template <typename T, bool STATS>
__global__ void __launch_bounds__(128)
chunk_scores_generic_kernel(const T *__restrict__ query, const float *__restrict__ lse,
                            const int32_t *__restrict__ query_index, int query_rows,
                            const T *__restrict__ key_cache,
                            const int32_t *__restrict__ block_table, int64_t bt_stride,
                            int64_t bt_cols, const int32_t *__restrict__ seq_lens, int Hq,
                            int Hk, int D, int block_size, int64_t num_blocks, int chunk,
                            int max_chunks, float scale_log2, float *__restrict__ out,
                            float *__restrict__ out_sum, int32_t *err) {
  pdl_begin();
  extern __shared__ float qs_all[];
  const int b = blockIdx.y, c = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int group = Hq / Hk;
  float *qs = qs_all + warp * group * D;
  const int qrow = (query_index != nullptr) ? query_index[b] : b;
  const bool qrow_ok = qrow >= 0 && qrow < query_rows;
  if (!qrow_ok && threadIdx.x == 0 && c == 0 && seq_lens[b] > 0) flag_error(err, DSB_FLAG_POSITION);
  const int L = qrow_ok ? seq_lens[b] : 0;
  const int32_t *bt_row = block_table + (int64_t)b * bt_stride;
  const int tok0 = c * chunk;
  for (int kvh = warp; kvh < Hk; kvh += 4) {
    if (tok0 >= L) {
      if (!STATS) {
        if (lane == 0) out[((int64_t)b * Hk + kvh) * max_chunks + c] = 0.f;
      } else {
        for (int h = lane; h < group; h += 32) {
          const int64_t o = ((int64_t)b * Hq + kvh * group + h) * max_chunks + c;
          out[o] = -INFINITY;
          out_sum[o] = 0.f;
        }
      }
      continue;
    }
    __syncwarp();
    for (int i = lane; i < group * D; i += 32)
      qs[i] = Elem<T>::to_f(query[((int64_t)qrow * Hq + kvh * group) * D + i]);
    __syncwarp();
    const int n_tok = min(chunk, L - tok0);
    float acc = 0.f;
    for (int h = 0; h < group; ++h) {
      const float l2 = STATS ? 0.f : lse[(int64_t)qrow * Hq + kvh * group + h] * kLog2e;
      float mm = -INFINITY, ss = 0.f;
      for (int i = lane; i < n_tok; i += 32) {
        const T *row = paged_row(key_cache, bt_row, bt_cols, block_size, num_blocks, Hk, D,
                                 kvh, tok0 + i, err);
        if (row == nullptr) continue;
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot = fmaf(qs[h * D + d], Elem<T>::to_f(row[d]), dot);
        if (!STATS) {
          acc += exp2f(fmaf(dot, scale_log2, -l2));
        } else {
          const float x = dot * scale_log2;
          const float mn = fmaxf(mm, x);
          ss = ss * exp2f(mm - mn) + exp2f(x - mn);
          mm = mn;
        }
      }
      if (STATS) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float mo = __shfl_xor_sync(0xffffffffu, mm, o);
          const float so = __shfl_xor_sync(0xffffffffu, ss, o);
          const float mn = fmaxf(mm, mo);
          ss = (mn == -INFINITY) ? 0.f : ss * exp2f(mm - mn) + so * exp2f(mo - mn);
          mm = mn;
        }
        if (lane == 0) {
          const int64_t o = ((int64_t)b * Hq + kvh * group + h) * max_chunks + c;
          out[o] = mm;
          out_sum[o] = ss;
        }
      }
    }
    if (!STATS) {
      acc = warp_sum(acc);
      if (lane == 0) out[((int64_t)b * Hk + kvh) * max_chunks + c] = acc;
    }
  }
}

// LSE over all chunks of each (row, query head), then per-kv-head mass.
__global__ void __launch_bounds__(256)
stats_to_head_scores_kernel(const float *__restrict__ cmax, const float *__restrict__ csum,
                            const int32_t *__restrict__ seq_lens, int Hq, int Hk, int chunk,
                            int max_chunks, float *__restrict__ head_scores,
                            float *__restrict__ lse_out) {
  pdl_begin();
  extern __shared__ float lse2[];
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int L = seq_lens[b];
  const int n_valid = (L + chunk - 1) / chunk;
  const int group = Hq / Hk;
  for (int h = warp; h < Hq; h += nwarps) {
    const float *mrow = cmax + ((int64_t)b * Hq + h) * max_chunks;
    const float *srow = csum + ((int64_t)b * Hq + h) * max_chunks;
    float mm = -INFINITY;
    for (int c = lane; c < n_valid; c += 32) mm = fmaxf(mm, mrow[c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
    float ss = 0.f;
    if (mm != -INFINITY)
      for (int c = lane; c < n_valid; c += 32) ss += srow[c] * exp2f(mrow[c] - mm);
    ss = warp_sum(ss);
    const float l2 = (mm == -INFINITY) ? -INFINITY : mm + log2f(ss);
    if (lane == 0) {
      lse2[h] = l2;
      if (lse_out != nullptr) lse_out[(int64_t)b * Hq + h] = l2 / kLog2e;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < Hk * max_chunks; i += blockDim.x) {
    const int kvh = i / max_chunks, c = i % max_chunks;
    float acc = 0.f;
    if (c < n_valid) {
      for (int j = 0; j < group; ++j) {
        const int h = kvh * group + j;
        const int64_t o = ((int64_t)b * Hq + h) * max_chunks + c;
        if (lse2[h] != -INFINITY && csum[o] > 0.f) acc += csum[o] * exp2f(cmax[o] - lse2[h]);
      }
    }
    head_scores[((int64_t)b * Hk + kvh) * max_chunks + c] = acc;
  }
}

__global__ void __launch_bounds__(256)
finalize_scores_kernel(const float *__restrict__ parts, int64_t row_stride,
                       int64_t part_stride, int num_parts,
                       const int32_t *__restrict__ seq_lens, int total_heads, int chunk,
                       int max_chunks, float *__restrict__ scores) {
  pdl_begin();
  const int b = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= max_chunks) return;
  const int L = seq_lens[b];
  const int nv = max(0, min(chunk, L - c * chunk));
  float s = 0.f;
  if (nv > 0) {
    const float *p = parts + (int64_t)b * row_stride + c;
    for (int q = 0; q < num_parts; ++q) s += p[(int64_t)q * part_stride];
    s = s / (float)nv / (float)total_heads;
  }
  scores[(int64_t)b * max_chunks + c] = s;
}

struct ScoreArgs {
  const void *query;
  const float *lse;
  const int32_t *qidx;
  int qrows;
  const void *kc;
  const int32_t *bt;
  int64_t bt_stride, bt_cols;
  const int32_t *seq;
  int B, Hq, Hk, D, bs;
  int64_t nblocks;
  int C, max_chunks;
  float scale;
  int dtype;
  float *out, *out_sum;
  int32_t *err;
  cudaStream_t st;
};

int validate(const ScoreArgs &a, bool stats) {
  if (a.B < 0 || a.max_chunks < 0) return fail(DSB_ERR_INVALID, "negative batch or chunk count");
  if (a.B == 0 || a.max_chunks == 0) return DSB_OK;
  if (!a.query || !a.kc || !a.bt || !a.seq || !a.out || (stats && !a.out_sum) ||
      (!stats && !a.lse))
    return fail(DSB_ERR_INVALID, "null pointer argument");
  if (a.qidx == nullptr) {
    if (a.qrows < a.B) return fail(DSB_ERR_INVALID, "query_rows is smaller than the batch");
  } else if (a.qrows <= 0) {
    return fail(DSB_ERR_INVALID, "query_rows must be positive");
  }
  if (a.Hq <= 0 || a.Hk <= 0 || a.Hq % a.Hk)
    return fail(DSB_ERR_INVALID, "query heads must be divisible by KV heads");
  if (a.D <= 0 || a.bs <= 0 || a.C <= 0 || a.nblocks <= 0 || a.bt_cols <= 0)
    return fail(DSB_ERR_INVALID, "head_dim, block_size, chunk_size, blocks must be positive");
  if (a.dtype != DSB_BF16 && a.dtype != DSB_F16 && a.dtype != DSB_F32)
    return fail(DSB_ERR_INVALID, "unknown dtype");
  return DSB_OK;
}

// Chunks per CTA: the per-launch time is about (waves of CTAs) x (items of
// the busiest warp), so the count minimising that product (the largest such
// count, for fewer CTAs) is taken; the tail wave and uneven warps cost as
// much as they weigh.
int pick_chunks_per_cta(int64_t max_chunks, int64_t rows, int hk, int64_t resident) {
  int best = 2;
  int64_t best_cost = INT64_MAX;
  for (int cpc = 2; cpc <= kMaxChunksPerCta; ++cpc) {
    const int64_t ctas = (max_chunks + cpc - 1) / cpc * rows;
    const int64_t waves = (ctas + resident - 1) / resident;
    const int64_t per_warp = ((int64_t)hk * cpc + kWarps - 1) / kWarps;
    const int64_t cost = waves * per_warp;
    if (cost <= best_cost) {
      best_cost = cost;
      best = cpc;
    }
  }
  return best;
}

template <typename T, int D, int NT, bool STATS>
int launch_mma(const ScoreArgs &a) {
  auto kern = chunk_scores_mma_kernel<T, D, NT, STATS>;
  const int cpc = pick_chunks_per_cta(a.max_chunks, a.B, a.Hk,
                                      resident_ctas((const void *)kern, kWarps * 32, 0));
  const dim3 grid((unsigned)((a.max_chunks + cpc - 1) / cpc), a.B);
  launch_kernel(kern, grid, dim3(kWarps * 32), 0, a.st,
      static_cast<const T *>(a.query), a.lse, a.qidx, a.qrows, static_cast<const T *>(a.kc), a.bt,
      a.bt_stride, a.bt_cols, a.seq, a.Hq, a.Hk, a.bs, a.nblocks, a.C, a.max_chunks, cpc,
      a.scale * kLog2e, a.out, a.out_sum, a.err);
  return check_launch("chunk_scores_mma_kernel");
}

template <typename T, bool STATS>
int dispatch_typed(const ScoreArgs &a) {
  const int group = a.Hq / a.Hk;
  const bool mma_ok = (a.C % 16 == 0) && group <= 16 &&
                      (a.D == 64 || a.D == 128 || a.D == 256) && !std::is_same<T, float>::value;
  if constexpr (!std::is_same<T, float>::value) {
    if (mma_ok) {
      const int nt = group <= 8 ? 1 : 2;
#define DSB_SC(DD, NN)                                                     \
  if (a.D == DD && nt == NN) return launch_mma<T, DD, NN, STATS>(a);
      DSB_SC(64, 1) DSB_SC(64, 2) DSB_SC(128, 1) DSB_SC(128, 2) DSB_SC(256, 1) DSB_SC(256, 2)
#undef DSB_SC
    }
  }
  const size_t smem = sizeof(float) * 4 * (size_t)group * a.D;
  if (smem > 200 * 1024) return fail(DSB_ERR_UNSUPPORTED, "group * head_dim too large");
  auto kern = chunk_scores_generic_kernel<T, STATS>;
  if (int st_ = ensure_smem((const void *)kern, smem); st_ != DSB_OK) return st_;
  dim3 grid(a.max_chunks, a.B);
  launch_kernel(kern, dim3(grid), dim3(128), smem, a.st, static_cast<const T *>(a.query), a.lse,
                a.qidx, a.qrows, static_cast<const T *>(a.kc), a.bt, a.bt_stride, a.bt_cols, a.seq,
                a.Hq, a.Hk, a.D, a.bs, a.nblocks, a.C, a.max_chunks, a.scale * kLog2e, a.out,
                a.out_sum, a.err);
  return check_launch("chunk_scores_generic_kernel");
}

template <bool STATS>
int run_scores(const ScoreArgs &a) {
  int v = validate(a, STATS);
  if (v != DSB_OK || a.B == 0 || a.max_chunks == 0) return v;
  if (a.max_chunks > 65535 * 2 || a.B > 65535)
    return fail(DSB_ERR_UNSUPPORTED, "grid too large");
  switch (a.dtype) {
    case DSB_BF16: return dispatch_typed<__nv_bfloat16, STATS>(a);
    case DSB_F16: return dispatch_typed<__half, STATS>(a);
    default: return dispatch_typed<float, STATS>(a);
  }
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int dsb_paged_chunk_head_scores(
    const void *query, const float *softmax_lse, const int32_t *query_index, int32_t query_rows,
    const void *key_cache, const int32_t *block_table, int64_t block_table_stride,
    int64_t block_table_cols, const int32_t *seq_lens, int32_t batch,
    int32_t num_query_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int64_t num_blocks, int32_t chunk_size, int32_t max_chunks, float scale, int32_t dtype,
    float *head_scores, int32_t *error_flag, void *stream) {
  ScoreArgs a{query, softmax_lse, query_index, query_rows, key_cache, block_table, block_table_stride,
              block_table_cols, seq_lens, batch, num_query_heads, num_kv_heads, head_dim,
              block_size, num_blocks, chunk_size, max_chunks, scale, dtype, head_scores,
              nullptr, error_flag, as_stream(stream)};
  return run_scores<false>(a);
}

extern "C" int dsb_paged_chunk_stats(
    const void *query, const int32_t *query_index, int32_t query_rows, const void *key_cache,
    const int32_t *block_table, int64_t block_table_stride, int64_t block_table_cols,
    const int32_t *seq_lens, int32_t batch, int32_t num_query_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t block_size, int64_t num_blocks, int32_t chunk_size,
    int32_t max_chunks, float scale, int32_t dtype, float *chunk_max, float *chunk_sum,
    int32_t *error_flag, void *stream) {
  ScoreArgs a{query, nullptr, query_index, query_rows, key_cache, block_table, block_table_stride,
              block_table_cols, seq_lens, batch, num_query_heads, num_kv_heads, head_dim,
              block_size, num_blocks, chunk_size, max_chunks, scale, dtype, chunk_max,
              chunk_sum, error_flag, as_stream(stream)};
  return run_scores<true>(a);
}

extern "C" int dsb_chunk_stats_to_head_scores(const float *chunk_max, const float *chunk_sum,
                                              const int32_t *seq_lens, int32_t batch,
                                              int32_t num_query_heads, int32_t num_kv_heads,
                                              int32_t chunk_size, int32_t max_chunks,
                                              float *head_scores, float *lse_out,
                                              void *stream) {
  if (batch < 0 || max_chunks < 0) return fail(DSB_ERR_INVALID, "negative sizes");
  if (batch == 0 || max_chunks == 0) return DSB_OK;
  if (!chunk_max || !chunk_sum || !seq_lens || !head_scores)
    return fail(DSB_ERR_INVALID, "null pointer argument");
  if (num_query_heads <= 0 || num_kv_heads <= 0 || num_query_heads % num_kv_heads ||
      chunk_size <= 0)
    return fail(DSB_ERR_INVALID, "bad head counts or chunk size");
  const size_t smem = sizeof(float) * num_query_heads;
  launch_kernel(stats_to_head_scores_kernel, dim3(batch), dim3(256), smem, as_stream(stream),
      chunk_max, chunk_sum, seq_lens, num_query_heads, num_kv_heads, chunk_size, max_chunks,
      head_scores, lse_out);
  return check_launch("stats_to_head_scores_kernel");
}

extern "C" int dsb_finalize_chunk_scores(const float *parts, int64_t row_stride,
                                         int64_t part_stride, int32_t num_parts,
                                         const int32_t *seq_lens, int32_t batch,
                                         int32_t total_query_heads, int32_t chunk_size,
                                         int32_t max_chunks, float *scores, void *stream) {
  if (batch < 0 || max_chunks < 0 || num_parts < 0) return fail(DSB_ERR_INVALID, "negative sizes");
  if (batch == 0 || max_chunks == 0) return DSB_OK;
  if (!parts || !seq_lens || !scores) return fail(DSB_ERR_INVALID, "null pointer argument");
  if (total_query_heads <= 0 || chunk_size <= 0)
    return fail(DSB_ERR_INVALID, "bad head count or chunk size");
  dim3 grid((max_chunks + 255) / 256, batch);
  launch_kernel(finalize_scores_kernel, dim3(grid), dim3(256), 0, as_stream(stream),
      parts, row_stride, part_stride, num_parts, seq_lens, total_query_heads, chunk_size,
      max_chunks, scores);
  return check_launch("finalize_scores_kernel");
}
