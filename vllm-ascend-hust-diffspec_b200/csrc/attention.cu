// GQA draft decode attention over capacity-sized working caches (row A8).
//
// Reference: _forward_linear_attention_npu, diffspec/runtime.py:2079-2134
// (index_copy of the new K/V, an index_select copy of the whole working cache
// when slots are reordered, then the closed FIA op with per-request valid
// lengths) and its CPU loop :2040-2077.
//
// B200 design (split-KV flash decode, one CTA per (split, kv head, row)):
//  * slots are read through the slot vector, so reordered batches copy nothing;
//  * the new token's K/V is read from the step's inputs and stored into the
//    cache by the CTA whose split owns that position (nobody reads it back);
//  * both products run on tensor cores with mma.sync m16n8k16 in swap-AB form,
//    so the 8 query heads of a GQA group fill the N=8 side exactly:
//      S^T[16 tok x 8 heads] = K[16 x D] Q^T[D x 8]          (A = K from HBM)
//      O^T[D x 8 heads]     += V^T[D x 16 tok] P^T[16 x 8]    (A = V from HBM)
//    K and V go from HBM straight into A-fragment registers with 16-byte
//    loads: lane (g, t) loads K tokens g, g+8 at head-dim slab t, and V tokens
//    2t, 2t+1, 2t+8, 2t+9 at head-dim runs {8 * (8j + g) .. +8 : j < D/64}
//    (each load instruction covers contiguous 128-byte runs); the V pairs are
//    formed with one byte-permute per register.  P goes C-layout ->
//    B-layout through a 256-byte per-warp shared tile and ldmatrix.trans.
//  * the online softmax runs in base 2 in fp32; splits publish (m, l, O)
//    partials and the last split of each (row, kv head) to finish merges them
//    (an atomic ticket, no spin wait).
#include <cmath>
#include <map>
#include <mutex>
#include <string>

#include "common.cuh"

namespace dsb {
namespace {

constexpr int kAttnWarps = 4;

struct AttnArgs {
  const void *query, *key, *value;
  void *wk, *wv;
  const int32_t *slots, *positions;
  int position_offset;
  int rows, out_rows, num_slots, Hq, Hk, W;
  float scale_log2;
  void *out;
  float *scratch;
  int32_t *counters;
  int num_splits, split_tokens;
  int32_t *err;
};

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

template <typename T, int D>
__device__ __forceinline__ void zero_heads(T *out, int row, int Hq, int h0, int n) {
  uint4 *o = reinterpret_cast<uint4 *>(out + ((int64_t)row * Hq + h0) * D);
  for (int i = threadIdx.x; i < n * D * (int)sizeof(T) / 16; i += blockDim.x)
    o[i] = make_uint4(0, 0, 0, 0);
}

template <typename T, int D, int NT>
__global__ void __launch_bounds__(kAttnWarps * 32)
draft_attention_kernel(const AttnArgs a) {
  constexpr int KS = D / 16;   // k-steps of Q.K over head_dim
  constexpr int NM = D / 16;   // M-tiles of O^T over head_dim
  constexpr int GP = NT * 8;   // padded heads per group
  constexpr int VPL = D / 64;  // 16-byte V vectors per token per lane
  extern __shared__ float smem[];
  float *s_o = smem;                                    // [warps][GP][D]
  float *s_m = s_o + kAttnWarps * GP * D;               // [warps][GP]
  float *s_l = s_m + kAttnWarps * GP;                   // [warps][GP]
  T *s_p = reinterpret_cast<T *>(s_l + kAttnWarps * GP);  // [warps][16][GP]
  __shared__ int s_last;

  const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int group = a.Hq / a.Hk;
  T *out = static_cast<T *>(a.out);
  if (row >= a.rows) {
    if (split == 0) zero_heads<T, D>(out, row, a.Hq, kvh * group, group);
    return;
  }
  const int slot = a.slots[row];
  const int pos = a.positions[row] + a.position_offset;
  if (slot < 0 || slot >= a.num_slots || pos < 0 || pos >= a.W) {
    if (split == 0) {
      if (threadIdx.x == 0)
        flag_error(a.err, (slot < 0 || slot >= a.num_slots) ? DSB_FLAG_SLOT : DSB_FLAG_POSITION);
      zero_heads<T, D>(out, row, a.Hq, kvh * group, group);
    }
    return;
  }
  const int len = pos + 1;
  const int active = (len + a.split_tokens - 1) / a.split_tokens;
  if (split >= active) return;
  const int ts = split * a.split_tokens;
  const int te = min(len, ts + a.split_tokens);

  const T *wk = static_cast<const T *>(a.wk) + ((int64_t)slot * a.Hk + kvh) * a.W * D;
  const T *wv = static_cast<const T *>(a.wv) + ((int64_t)slot * a.Hk + kvh) * a.W * D;
  const T *nk = static_cast<const T *>(a.key) + ((int64_t)row * a.Hk + kvh) * D;
  const T *nv = static_cast<const T *>(a.value) + ((int64_t)row * a.Hk + kvh) * D;

  if (pos >= ts && pos < te) {  // store this step's K/V at its local position
    constexpr int VE = 16 / sizeof(T);
    for (int i = threadIdx.x; i < D / VE; i += blockDim.x) {
      reinterpret_cast<uint4 *>(static_cast<T *>(a.wk) +
                                (((int64_t)slot * a.Hk + kvh) * a.W + pos) * D)[i] =
          reinterpret_cast<const uint4 *>(nk)[i];
      reinterpret_cast<uint4 *>(static_cast<T *>(a.wv) +
                                (((int64_t)slot * a.Hk + kvh) * a.W + pos) * D)[i] =
          reinterpret_cast<const uint4 *>(nv)[i];
    }
  }

  // Q^T B-fragments: lane (g, t) holds head nt*8+g, slab t of head_dim.
  uint32_t qf[NT][KS][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int h = nt * 8 + g;
    uint4 qv[D / 32];
    if (h < group) {
      const T *qp = static_cast<const T *>(a.query) + ((int64_t)row * a.Hq + kvh * group + h) * D;
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
  }

  float o[NT][NM][4];
  float m_run[NT][2], l_run[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int i = 0; i < NM; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) o[nt][i][c] = 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      m_run[nt][j] = -INFINITY;
      l_run[nt][j] = 0.f;
    }
  }
  T *pw = s_p + warp * 16 * GP;

  for (int base = ts + warp * 16; base < te; base += kAttnWarps * 16) {
    // ---- loads (masked tokens read nothing and contribute zeros)
    uint4 ka[D / 32], kb[D / 32], vv[4][VPL];
    {
      const int ta = base + g, tb = base + g + 8;
      const T *ra = (ta == pos) ? nk : wk + (int64_t)ta * D;
      const T *rb = (tb == pos) ? nk : wk + (int64_t)tb * D;
#pragma unroll
      for (int j = 0; j < D / 32; ++j) {
        ka[j] = (ta < te) ? ldg_stream(ra + 8 * (4 * j + t)) : make_uint4(0, 0, 0, 0);
        kb[j] = (tb < te) ? ldg_stream(rb + 8 * (4 * j + t)) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int tv = base + 2 * t + (q & 1) + (q >> 1) * 8;
        const T *rv = (tv == pos) ? nv : wv + (int64_t)tv * D;
#pragma unroll
        for (int j = 0; j < VPL; ++j)
          vv[q][j] = (tv < te) ? ldg_stream(rv + 8 * (8 * j + g)) : make_uint4(0, 0, 0, 0);
      }
    }
    const bool va = base + g < te, vb = base + g + 8 < te;

    // ---- S^T = K Q^T, online softmax, P -> shared
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const uint32_t af[4] = {word_of(ka[(2 * s) / 4], (2 * s) % 4),
                                word_of(kb[(2 * s) / 4], (2 * s) % 4),
                                word_of(ka[(2 * s + 1) / 4], (2 * s + 1) % 4),
                                word_of(kb[(2 * s + 1) / 4], (2 * s + 1) % 4)};
        Mma<T>::run(c, af, qf[nt][s]);
      }
      float x[4];
      x[0] = va ? c[0] * a.scale_log2 : -INFINITY;
      x[1] = va ? c[1] * a.scale_log2 : -INFINITY;
      x[2] = vb ? c[2] * a.scale_log2 : -INFINITY;
      x[3] = vb ? c[3] * a.scale_log2 : -INFINITY;
      float p[4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float mx = fmaxf(x[j], x[j + 2]);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float mn = fmaxf(m_run[nt][j], mx);
        float alpha;
        if (mn == -INFINITY) {
          alpha = 1.f;
          p[j] = 0.f;
          p[j + 2] = 0.f;
        } else {
          alpha = exp2f(m_run[nt][j] - mn);
          p[j] = exp2f(x[j] - mn);
          p[j + 2] = exp2f(x[j + 2] - mn);
        }
        m_run[nt][j] = mn;
        l_run[nt][j] = l_run[nt][j] * alpha + p[j] + p[j + 2];
#pragma unroll
        for (int i = 0; i < NM; ++i) {
          o[nt][i][j] *= alpha;
          o[nt][i][j + 2] *= alpha;
        }
      }
      uint32_t *prow = reinterpret_cast<uint32_t *>(pw);
      prow[(g * GP + nt * 8 + 2 * t) / 2] = pack2<T>(p[0], p[1]);
      prow[((g + 8) * GP + nt * 8 + 2 * t) / 2] = pack2<T>(p[2], p[3]);
    }
    __syncwarp();
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) ldsm_x2_trans(pb[nt], pw + (lane & 15) * GP + nt * 8);
    __syncwarp();

    // ---- O^T += V^T P^T
#pragma unroll
    for (int i = 0; i < NM; ++i) {
      const int e_lo = i, e_hi = NM + i;  // element index inside the lane's D/8 run
      const uint32_t sel_lo = (e_lo & 1) ? 0x7632u : 0x5410u;
      const uint32_t sel_hi = (e_hi & 1) ? 0x7632u : 0x5410u;
      const int wl = e_lo / 2, wh = e_hi / 2;  // 32-bit word inside the run
      const uint32_t af[4] = {
          __byte_perm(word_of(vv[0][wl / 4], wl % 4), word_of(vv[1][wl / 4], wl % 4), sel_lo),
          __byte_perm(word_of(vv[0][wh / 4], wh % 4), word_of(vv[1][wh / 4], wh % 4), sel_hi),
          __byte_perm(word_of(vv[2][wl / 4], wl % 4), word_of(vv[3][wl / 4], wl % 4), sel_lo),
          __byte_perm(word_of(vv[2][wh / 4], wh % 4), word_of(vv[3][wh / 4], wh % 4), sel_hi)};
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) Mma<T>::run(o[nt][i], af, pb[nt]);
    }
  }

  // ---- merge the warps of this CTA
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float l = l_run[nt][j];
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (g == 0) {
        s_m[warp * GP + nt * 8 + 2 * t + j] = m_run[nt][j];
        s_l[warp * GP + nt * 8 + 2 * t + j] = l;
      }
    }
#pragma unroll
    for (int i = 0; i < NM; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int h = nt * 8 + 2 * t + (c & 1);
        const int e = (c < 2) ? i : NM + i;  // element of the lane's V run list
        const int d = 64 * (e / 8) + 8 * g + e % 8;
        s_o[(warp * GP + h) * D + d] = o[nt][i][c];
      }
  }
  __syncthreads();

  const int n_out = group * D;
  T *orow = out + ((int64_t)row * a.Hq + kvh * group) * D;
  if (active == 1) {
    for (int idx = threadIdx.x; idx < n_out; idx += blockDim.x) {
      const int h = idx / D, d = idx % D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w * GP + h]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = (s_m[w * GP + h] == -INFINITY) ? 0.f : exp2f(s_m[w * GP + h] - M);
        L += s_l[w * GP + h] * f;
        O += s_o[(w * GP + h) * D + d] * f;
      }
      orow[idx] = Elem<T>::from_f(O / L);
    }
    return;
  }

  // ---- publish this split's partial state
  const int64_t part_floats = (int64_t)GP * (2 + D);
  float *part_base = a.scratch + ((int64_t)row * a.Hk + kvh) * a.num_splits * part_floats;
  float *part = part_base + (int64_t)split * part_floats;
  for (int idx = threadIdx.x; idx < GP * (D + 1); idx += blockDim.x) {
    if (idx < GP) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w * GP + idx]);
      float L = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w)
        L += (s_m[w * GP + idx] == -INFINITY) ? 0.f : s_l[w * GP + idx] * exp2f(s_m[w * GP + idx] - M);
      part[idx] = M;
      part[GP + idx] = L;
    } else {
      const int k = idx - GP, h = k / D, d = k % D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w * GP + h]);
      float O = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w)
        O += (s_m[w * GP + h] == -INFINITY) ? 0.f
                                            : s_o[(w * GP + h) * D + d] * exp2f(s_m[w * GP + h] - M);
      part[2 * GP + k] = O;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&a.counters[row * a.Hk + kvh], 1);
    s_last = (prev == active - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Merge: stage every split's (m, l) in shared memory (one independent load
  // per thread), fold them into per-split weights exp2(m_s - M) / L, then
  // each output float4 sums `active` independent float4 loads.
  float *w_s = s_o;  // [active][GP]; the CTA's own O staging is no longer needed
  float *l_s = s_o + (size_t)active * GP;
  for (int i = threadIdx.x; i < active * GP; i += blockDim.x) {
    const float *ps = part_base + (int64_t)(i / GP) * part_floats;
    w_s[i] = __ldcg(ps + i % GP);
    l_s[i] = __ldcg(ps + GP + i % GP);
  }
  __syncthreads();
  for (int h = threadIdx.x; h < GP; h += blockDim.x) {
    float M = -INFINITY;
    for (int s2 = 0; s2 < active; ++s2) M = fmaxf(M, w_s[s2 * GP + h]);
    float L = 0.f;
    for (int s2 = 0; s2 < active; ++s2) {
      const float ms = w_s[s2 * GP + h];
      const float f = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
      w_s[s2 * GP + h] = f;
      L += l_s[s2 * GP + h] * f;
    }
    const float inv = 1.f / L;
    for (int s2 = 0; s2 < active; ++s2) w_s[s2 * GP + h] *= inv;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < n_out / 4; idx += blockDim.x) {
    const int h = (4 * idx) / D, d = (4 * idx) % D;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int s2 = 0; s2 < active; ++s2) {
      const float4 o = __ldcg(reinterpret_cast<const float4 *>(
          part_base + (int64_t)s2 * part_floats + 2 * GP + h * D + d));
      const float f = w_s[s2 * GP + h];
      acc.x += o.x * f;
      acc.y += o.y * f;
      acc.z += o.z * f;
      acc.w += o.w * f;
    }
    orow[4 * idx] = Elem<T>::from_f(acc.x);
    orow[4 * idx + 1] = Elem<T>::from_f(acc.y);
    orow[4 * idx + 2] = Elem<T>::from_f(acc.z);
    orow[4 * idx + 3] = Elem<T>::from_f(acc.w);
  }
  if (threadIdx.x == 0) a.counters[row * a.Hk + kvh] = 0;
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int32_t dsb_draft_attention_default_splits(int32_t rows, int32_t num_kv_heads,
                                                      int32_t working_budget, int32_t sm_count) {
  if (rows <= 0 || num_kv_heads <= 0 || working_budget <= 0) return 1;
  if (sm_count <= 0) sm_count = 148;
  const int64_t pairs = (int64_t)rows * num_kv_heads;
  int64_t splits = (4LL * sm_count + pairs - 1) / pairs;
  int64_t max_splits = (working_budget + 31) / 32;
  if (max_splits > 64) max_splits = 64;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  return (int32_t)splits;
}

extern "C" int64_t dsb_draft_attention_scratch_floats(int32_t rows, int32_t num_query_heads,
                                                     int32_t num_kv_heads, int32_t head_dim,
                                                     int32_t num_splits) {
  if (rows <= 0 || num_kv_heads <= 0 || num_query_heads <= 0 || num_splits <= 0) return 0;
  const int group = num_query_heads / num_kv_heads;
  const int gp = group <= 8 ? 8 : 16;
  return (int64_t)rows * num_kv_heads * num_splits * gp * (2 + head_dim);
}

extern "C" int dsb_draft_decode_attention(
    const void *query, const void *key, const void *value, void *working_key,
    void *working_value, const int32_t *slots, const int32_t *positions,
    int32_t position_offset, int32_t rows, int32_t out_rows, int32_t num_slots, int32_t num_query_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t working_budget, float scale, int32_t dtype, void *output,
    float *scratch, int64_t scratch_floats, int32_t *counters, int32_t num_splits,
    int32_t *error_flag, void *stream) {
  if (rows < 0 || out_rows < rows) return fail(DSB_ERR_INVALID, "out_rows must be >= rows >= 0");
  if (out_rows == 0) return DSB_OK;
  if (num_query_heads <= 0 || num_kv_heads <= 0 || num_query_heads % num_kv_heads)
    return fail(DSB_ERR_INVALID, "query heads must be divisible by KV heads");
  if (num_slots <= 0 || working_budget <= 0) return fail(DSB_ERR_INVALID, "empty working cache");
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_UNSUPPORTED, "draft attention runs on BF16 or FP16 caches");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(DSB_ERR_UNSUPPORTED, "draft attention supports head_dim 64, 128 or 256");
  const int group = num_query_heads / num_kv_heads;
  if (group > 16) return fail(DSB_ERR_UNSUPPORTED, "draft attention supports GQA groups up to 16");
  if (!query || !key || !value || !working_key || !working_value || !slots || !positions ||
      !output || (rows > 0 && !counters))
    return fail(DSB_ERR_INVALID, "null pointer argument");
  if (num_splits <= 0) return fail(DSB_ERR_INVALID, "num_splits must be positive");
  if (out_rows > 65535 || num_kv_heads > 65535) return fail(DSB_ERR_UNSUPPORTED, "grid too large");
  int split_tokens = (working_budget + num_splits - 1) / num_splits;
  split_tokens = (split_tokens + 31) / 32 * 32;
  // the last split stages (m, l) of every split in the CTA's shared memory,
  // which holds 2 * head_dim floats per padded head
  const int max_splits = 2 * head_dim;
  if ((working_budget + split_tokens - 1) / split_tokens > max_splits)
    split_tokens = ((working_budget + max_splits - 1) / max_splits + 31) / 32 * 32;
  const int splits = (working_budget + split_tokens - 1) / split_tokens;
  if (splits > 1 && rows > 0) {
    const int64_t need = dsb_draft_attention_scratch_floats(rows, num_query_heads, num_kv_heads,
                                                            head_dim, splits);
    if (!scratch || scratch_floats < need)
      return fail(DSB_ERR_INVALID, "attention scratch is smaller than dsb_draft_attention_scratch_floats");
  }
  AttnArgs a{query, key, value, working_key, working_value, slots, positions, position_offset,
             rows, out_rows,
             num_slots, num_query_heads, num_kv_heads, working_budget, scale * kLog2e, output,
             scratch, counters, splits, split_tokens, error_flag};
  cudaStream_t st = as_stream(stream);
  const int nt = group <= 8 ? 1 : 2;
#define DSB_AT(TT, DD, NN)                                                              \
  if (head_dim == DD && nt == NN) {                                                     \
    constexpr int GP = NN * 8;                                                          \
    const size_t smem = sizeof(float) * (kAttnWarps * GP * DD + 2 * kAttnWarps * GP) +  \
                        sizeof(TT) * kAttnWarps * 16 * GP;                              \
    auto kern = draft_attention_kernel<TT, DD, NN>;                                     \
    if (int st_ = ensure_smem((const void *)kern, smem); st_ != DSB_OK) return st_;    \
    kern<<<dim3(splits, num_kv_heads, out_rows), kAttnWarps * 32, smem, st>>>(a);      \
    return check_launch("draft_attention_kernel");                                      \
  }
  if (dtype == DSB_BF16) {
    DSB_AT(__nv_bfloat16, 64, 1) DSB_AT(__nv_bfloat16, 64, 2)
    DSB_AT(__nv_bfloat16, 128, 1) DSB_AT(__nv_bfloat16, 128, 2)
    DSB_AT(__nv_bfloat16, 256, 1) DSB_AT(__nv_bfloat16, 256, 2)
  } else {
    DSB_AT(__half, 64, 1) DSB_AT(__half, 64, 2)
    DSB_AT(__half, 128, 1) DSB_AT(__half, 128, 2)
    DSB_AT(__half, 256, 1) DSB_AT(__half, 256, 2)
  }
#undef DSB_AT
  return fail(DSB_ERR_UNSUPPORTED, "no draft attention kernel for this shape");
}

// ---------------------------------------------------------------------------
// Draft attention without any allocation by the caller or the library.
//
// Some callers cannot call cudaMalloc when they run the draft step: a serving
// engine that reserves nearly all free device memory for its KV cache at start
// and then forbids ad-hoc allocations, a host that records the step into a
// CUDA graph (allocation is not allowed during stream capture), or a caller
// whose latency budget cannot absorb cudaMalloc/cudaFree, which may
// synchronise the device.  For them the split-KV partials and merge tickets
// live in the fixed arrays below, which every GPU that loads this library
// holds until the process exits (4 MiB + 16 KiB per device).
//
// In host code the array names are host-side stand-ins, not device
// addresses; their device addresses are looked up with cudaGetSymbolAddress
// once per device, with that device current, on the first call made on it.
namespace dsb {
namespace {

constexpr int64_t kStaticScratchFloats = 1 << 20;  // 4 MiB of split partials
constexpr int kStaticTickets = 4096;                 // rows * kv_heads limit

static __device__ __align__(256) float g_static_scratch[kStaticScratchFloats];
static __device__ __align__(256) int32_t g_static_tickets[kStaticTickets];

struct StaticScratch {
  float *scratch = nullptr;
  int32_t *tickets = nullptr;
};

int static_scratch_for_current_device(StaticScratch &out) {
  static std::mutex mu;
  static std::map<int, StaticScratch> per_device;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(DSB_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  auto it = per_device.find(dev);
  if (it != per_device.end()) {
    out = it->second;
    return DSB_OK;
  }
  StaticScratch s;
  e = cudaGetSymbolAddress(reinterpret_cast<void **>(&s.scratch), g_static_scratch);
  if (e != cudaSuccess)
    return fail(DSB_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
  e = cudaGetSymbolAddress(reinterpret_cast<void **>(&s.tickets), g_static_tickets);
  if (e != cudaSuccess)
    return fail(DSB_ERR_CUDA, std::string("cudaGetSymbolAddress(tickets): ") + cudaGetErrorString(e));
  per_device[dev] = s;
  out = s;
  return DSB_OK;
}

}  // namespace
}  // namespace dsb

extern "C" int dsb_draft_decode_attention_static(
    const void *query, const void *key, const void *value, void *working_key,
    void *working_value, const int32_t *slots, const int32_t *positions,
    int32_t position_offset, int32_t rows, int32_t out_rows, int32_t num_slots,
    int32_t num_query_heads, int32_t num_kv_heads, int32_t head_dim, int32_t working_budget,
    float scale, int32_t dtype, void *output, int32_t num_splits, int32_t *error_flag,
    void *stream) {
  if (rows < 0 || out_rows < rows) return fail(DSB_ERR_INVALID, "out_rows must be >= rows >= 0");
  if (out_rows == 0) return DSB_OK;
  if (num_query_heads <= 0 || num_kv_heads <= 0 || num_query_heads % num_kv_heads)
    return fail(DSB_ERR_INVALID, "query heads must be divisible by KV heads");
  if (num_slots <= 0 || working_budget <= 0) return fail(DSB_ERR_INVALID, "empty working cache");
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_UNSUPPORTED, "draft attention runs on BF16 or FP16 caches");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(DSB_ERR_UNSUPPORTED, "draft attention supports head_dim 64, 128 or 256");
  const int group = num_query_heads / num_kv_heads;
  if (group > 16) return fail(DSB_ERR_UNSUPPORTED, "draft attention supports GQA groups up to 16");
  if (!query || !key || !value || !working_key || !working_value || !slots || !positions || !output)
    return fail(DSB_ERR_INVALID, "null pointer argument");
  if (out_rows > 65535 || num_kv_heads > 65535) return fail(DSB_ERR_UNSUPPORTED, "grid too large");
  if ((int64_t)rows * num_kv_heads > kStaticTickets)
    return fail(DSB_ERR_INVALID, "rows * num_kv_heads exceeds the static ticket array (4096)");
  if (num_splits <= 0)
    num_splits = dsb_draft_attention_default_splits(rows, num_kv_heads, working_budget, sm_count());
  int split_tokens = (working_budget + num_splits - 1) / num_splits;
  split_tokens = (split_tokens + 31) / 32 * 32;
  const int max_splits = 2 * head_dim;
  if ((working_budget + split_tokens - 1) / split_tokens > max_splits)
    split_tokens = ((working_budget + max_splits - 1) / max_splits + 31) / 32 * 32;
  const int splits = (working_budget + split_tokens - 1) / split_tokens;
  const int64_t need =
      dsb_draft_attention_scratch_floats(rows, num_query_heads, num_kv_heads, head_dim, splits);
  if (splits > 1 && need > kStaticScratchFloats)
    return fail(DSB_ERR_INVALID,
                "split partials need " + std::to_string(need) +
                    " floats, more than the static scratch (1048576 floats = 4 MiB); "
                    "pass fewer splits or use dsb_draft_decode_attention");
  StaticScratch st_mem;
  if (int st = static_scratch_for_current_device(st_mem); st != DSB_OK) return st;
  cudaStream_t st = as_stream(stream);
  // The arrays are shared by every call: tickets must start at zero, so
  // clear the ones this call uses (a plain memset, no allocation).
  if (rows > 0) {
    cudaError_t e = cudaMemsetAsync(st_mem.tickets, 0, sizeof(int32_t) * rows * num_kv_heads, st);
    if (e != cudaSuccess) return fail(DSB_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  }
  AttnArgs a{query, key, value, working_key, working_value, slots, positions, position_offset,
             rows, out_rows, num_slots, num_query_heads, num_kv_heads, working_budget,
             scale * kLog2e, output, st_mem.scratch, st_mem.tickets, splits, split_tokens,
             error_flag};
  const int nt = group <= 8 ? 1 : 2;
#define DSB_ATS(TT, DD, NN)                                                            \
  if (head_dim == DD && nt == NN) {                                                    \
    constexpr int GP = NN * 8;                                                         \
    const size_t smem = sizeof(float) * (kAttnWarps * GP * DD + 2 * kAttnWarps * GP) + \
                        sizeof(TT) * kAttnWarps * 16 * GP;                             \
    auto kern = draft_attention_kernel<TT, DD, NN>;                                    \
    if (int st_ = ensure_smem((const void *)kern, smem); st_ != DSB_OK) return st_;   \
    kern<<<dim3(splits, num_kv_heads, out_rows), kAttnWarps * 32, smem, st>>>(a);     \
    return check_launch("draft_attention_kernel (static scratch)");                    \
  }
  if (dtype == DSB_BF16) {
    DSB_ATS(__nv_bfloat16, 64, 1) DSB_ATS(__nv_bfloat16, 64, 2)
    DSB_ATS(__nv_bfloat16, 128, 1) DSB_ATS(__nv_bfloat16, 128, 2)
    DSB_ATS(__nv_bfloat16, 256, 1) DSB_ATS(__nv_bfloat16, 256, 2)
  } else {
    DSB_ATS(__half, 64, 1) DSB_ATS(__half, 64, 2)
    DSB_ATS(__half, 128, 1) DSB_ATS(__half, 128, 2)
    DSB_ATS(__half, 256, 1) DSB_ATS(__half, 256, 2)
  }
#undef DSB_ATS
  return fail(DSB_ERR_UNSUPPORTED, "no draft attention kernel for this shape");
}
