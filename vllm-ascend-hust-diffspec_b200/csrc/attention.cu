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
#include <climits>
#include <cmath>
#include <cstdlib>
#include <type_traits>
#include <map>
#include <mutex>
#include <string>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tma_umma.cuh"

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

template <int D> struct AttnStages { static constexpr int value = D >= 256 ? 2 : 3; };

// 16-byte cp.async global -> shared; when !valid nothing is read and the
// destination is zero-filled.
__device__ __forceinline__ void cp_async16_zfill(void *smem_dst, const void *gmem_src, bool valid) {
  if (valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
  } else {
    *reinterpret_cast<uint4 *>(smem_dst) = make_uint4(0, 0, 0, 0);
  }
}

template <typename T, int D, int NT>
constexpr size_t attn_smem_bytes() {
  return sizeof(uint4) * kAttnWarps * AttnStages<D>::value * (D / 8) * 32 +
         sizeof(float) * 2 * kAttnWarps * NT * 8 + sizeof(T) * kAttnWarps * 2 * 16 * NT * 8;
}

template <typename T, int D>
__device__ __forceinline__ void zero_heads(T *out, int row, int Hq, int h0, int n) {
  uint4 *o = reinterpret_cast<uint4 *>(out + ((int64_t)row * Hq + h0) * D);
  for (int i = threadIdx.x; i < n * D * (int)sizeof(T) / 16; i += blockDim.x)
    o[i] = make_uint4(0, 0, 0, 0);
}

// Four outputs as one 8-byte store (16-bit element types).
template <typename T>
__device__ __forceinline__ void store4(T *p, const float4 &v) {
  *reinterpret_cast<uint2 *>(p) = make_uint2(pack2<T>(v.x, v.y), pack2<T>(v.z, v.w));
}

// The elected last CTA of a (row, kv head) merges the `active` published
// partials [GP m | GP l | GP x D o]: stage every split's (m, l) in shared
// memory (one independent load per thread), fold them into per-split weights
// exp2(m_s - M) / L, then each output float4 sums `active` independent
// float4 loads.  s_buf holds 2 * active * GP floats.
template <typename T, int D, int GP>
__device__ __forceinline__ void merge_published(const float *part_base, int64_t part_floats,
                                                int active, T *orow, int n_out, float *s_buf) {
  // Merge: stage every split's (m, l) in shared memory (one independent load
  // per thread), fold them into per-split weights exp2(m_s - M) / L, then
  // each output float4 sums `active` independent float4 loads.
  float *w_s = s_buf;  // [active][GP]
  float *l_s = s_buf + (size_t)active * GP;
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
    store4<T>(orow + 4 * idx, acc);
  }
}

// Combine the CTA's warps (staged in s_o/s_m/s_l) and either store the
// normalised output (single split) or publish a partial; the last split of a
// (row, kv head) to finish merges all partials.
template <typename T, int D, int GP, int WARPS>
__device__ __forceinline__ void merge_and_store(const AttnArgs &a, float *s_o, const float *s_m,
                                                const float *s_l, T *out, int row, int kvh,
                                                int split, int active, int group, int *s_last) {
  const int n_out = group * D;
  T *orow = out + ((int64_t)row * a.Hq + kvh * group) * D;
  if (active == 1) {
    for (int idx = threadIdx.x; idx < n_out; idx += blockDim.x) {
      const int h = idx / D, d = idx % D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_m[w * GP + h]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
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
      for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_m[w * GP + idx]);
      float L = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w)
        L += (s_m[w * GP + idx] == -INFINITY) ? 0.f : s_l[w * GP + idx] * exp2f(s_m[w * GP + idx] - M);
      part[idx] = M;
      part[GP + idx] = L;
    } else {
      const int k = idx - GP, h = k / D, d = k % D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_m[w * GP + h]);
      float O = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w)
        O += (s_m[w * GP + h] == -INFINITY) ? 0.f
                                            : s_o[(w * GP + h) * D + d] * exp2f(s_m[w * GP + h] - M);
      part[2 * GP + k] = O;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&a.counters[row * a.Hk + kvh], 1);
    (*s_last) = (prev == active - 1);
  }
  __syncthreads();
  if (!(*s_last)) return;
  __threadfence();
  merge_published<T, D, GP>(part_base, part_floats, active, orow, n_out, s_o);
  if (threadIdx.x == 0) a.counters[row * a.Hk + kvh] = 0;
}

template <typename T, int D, int NT>
__global__ void __launch_bounds__(kAttnWarps * 32)
draft_attention_kernel(const AttnArgs a) {
  pdl_begin();
  constexpr int KS = D / 16;   // k-steps of Q.K over head_dim
  constexpr int NM = D / 16;   // M-tiles of O^T over head_dim
  constexpr int GP = NT * 8;   // padded heads per group
  constexpr int VPL = D / 64;  // 16-byte V vectors per token per lane
  constexpr int NS = AttnStages<D>::value;  // cp.async ring depth per warp
  constexpr int VPT = D / 8;   // 16-byte vectors per lane per 16-token tile (K + V)
  extern __shared__ float smem[];
  // [warps][NS][VPT][32 lanes] uint4: every lane reads back only what it copied
  uint4 *ring = reinterpret_cast<uint4 *>(smem);
  float *s_o = smem;                                    // [warps][GP][D], aliases the ring
  float *s_m = smem + kAttnWarps * NS * VPT * 32 * 4;   // [warps][GP]
  float *s_l = s_m + kAttnWarps * GP;                   // [warps][GP]
  T *s_p = reinterpret_cast<T *>(s_l + kAttnWarps * GP);  // [warps][hi, lo][16][GP]
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
  T *pw = s_p + warp * 2 * 16 * GP;  // hi tile; the lo tile follows

  // This warp's tiles are ts + (warp + kAttnWarps * k) * 16, k < n_my.  Each
  // is copied with cp.async into ring stage k % NS, NS - 1 tiles ahead of the
  // one being computed; masked tokens are zero-filled without a read.
  const int first = ts + warp * 16;
  const int n_my = (first < te) ? (te - first + kAttnWarps * 16 - 1) / (kAttnWarps * 16) : 0;
  uint4 *wring = ring + (size_t)warp * NS * VPT * 32 + lane;
  auto issue = [&](int k) {
    const int base = first + k * kAttnWarps * 16;
    uint4 *st = wring + (size_t)(k % NS) * VPT * 32;
    const int ta = base + g, tb = base + g + 8;
    const T *ra = (ta == pos) ? nk : ((ta < te) ? wk + (int64_t)ta * D : nk);
    const T *rb = (tb == pos) ? nk : ((tb < te) ? wk + (int64_t)tb * D : nk);
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      cp_async16_zfill(st + j * 32, ra + 8 * (4 * j + t), ta < te);
      cp_async16_zfill(st + (D / 32 + j) * 32, rb + 8 * (4 * j + t), tb < te);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int tv = base + 2 * t + (q & 1) + (q >> 1) * 8;
      const T *rv = (tv == pos) ? nv : ((tv < te) ? wv + (int64_t)tv * D : nv);
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        cp_async16_zfill(st + (D / 16 + q * VPL + j) * 32, rv + 8 * (8 * j + g), tv < te);
    }
  };
#pragma unroll
  for (int k = 0; k < NS - 1; ++k) {
    if (k < n_my) issue(k);
    cp_async_commit();
  }

  for (int k = 0; k < n_my; ++k) {
    if (k + NS - 1 < n_my) issue(k + NS - 1);
    cp_async_commit();
    cp_async_wait<NS - 1>();
    const int base = first + k * kAttnWarps * 16;
    uint4 ka[D / 32], kb[D / 32], vv[4][VPL];
    {
      const uint4 *st = wring + (size_t)(k % NS) * VPT * 32;
#pragma unroll
      for (int j = 0; j < D / 32; ++j) {
        ka[j] = st[j * 32];
        kb[j] = st[(D / 32 + j) * 32];
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int j = 0; j < VPL; ++j) vv[q][j] = st[(D / 16 + q * VPL + j) * 32];
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
      uint32_t *prow_lo = prow + 16 * GP / 2;
      pack2_split<T>(p[0], p[1], prow[(g * GP + nt * 8 + 2 * t) / 2],
                     prow_lo[(g * GP + nt * 8 + 2 * t) / 2]);
      pack2_split<T>(p[2], p[3], prow[((g + 8) * GP + nt * 8 + 2 * t) / 2],
                     prow_lo[((g + 8) * GP + nt * 8 + 2 * t) / 2]);
    }
    __syncwarp();
    uint32_t pb[NT][2], pl[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      ldsm_x2_trans(pb[nt], pw + (lane & 15) * GP + nt * 8);
      ldsm_x2_trans(pl[nt], pw + 16 * GP + (lane & 15) * GP + nt * 8);
    }
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
      for (int nt = 0; nt < NT; ++nt) {
        Mma<T>::run(o[nt][i], af, pb[nt]);
        Mma<T>::run(o[nt][i], af, pl[nt]);
      }
    }
  }

  // ---- merge the warps of this CTA (the O staging reuses the ring)
  cp_async_wait<0>();
  __syncthreads();
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

  merge_and_store<T, D, GP, kAttnWarps>(a, s_o, s_m, s_l, out, row, kvh, split, active, group,
                                        &s_last);
}


// ===========================================================================
// TMA-fed variant (the default on sm_100a): K/V stages of 8 * W tokens (W
// consumer warps in two groups) are copied by cp.async.bulk.tensor as
// 64-column boxes with 128-byte swizzle into a CTA-wide ring of NS stages,
// completion tracked by mbarriers; a producer warp issues all copies.
// Fragments come from the swizzled tiles with ldmatrix (conflict-free; V^T
// directly via ldmatrix.trans).  The two warp groups take alternate stages and
// each warp owns 16 tokens of its group's stages, so the two warps sharing a
// scheduler work on different stages.  The online softmax rescales O only
// when a running max grows by more than 2^8, so steady-state tiles skip the
// rescale.  All mbarrier waits are bounded: a wait that runs out sets
// DSB_FLAG_TIMEOUT, no further stage is issued, and the producer waits
// (bounded again) for the copies already issued before the ring is reused or
// the CTA exits.
// ===========================================================================
constexpr float kLazyRescale = 8.0f;  // log2 headroom before O is rescaled

// W consumer warps in kGroups groups; a warp owns 16 tokens of each of its
// group's stages, so stages are 16 * W / kGroups tokens, copied as D/64 boxes
// of [kStageTok rows x 128 bytes] for K and for V.
template <int D, int NS, int W> struct TmaCfg {
  static constexpr int kGroups = 2;
  static constexpr int kGroupWarps = W / kGroups;
  static constexpr int kStageTok = 16 * kGroupWarps;
  static_assert(W % kGroups == 0 && NS % kGroups == 0, "groups must split warps and ring evenly");
  static constexpr int kBoxBytes = 128 * kStageTok;
  static constexpr int kBoxes = D / 64;                       // boxes per K (or V) row
  static constexpr int kStageBytes = 2 * kBoxes * kBoxBytes;  // K + V
  static constexpr int kRingBytes = NS * kStageBytes;
  static constexpr int kBarBytes = (16 * NS + 15) / 16 * 16;  // full + empty mbarriers, padded
};

template <typename T, int D, int NT, int NS, int W>
constexpr size_t tma_smem_bytes() {
  return 1024 /* alignment slack */ + TmaCfg<D, NS, W>::kRingBytes + TmaCfg<D, NS, W>::kBarBytes +
         sizeof(float) * 2 * W * NT * 8 + sizeof(T) * W * 2 * 16 * NT * 8;
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// Byte address of (row, column) inside a stage half (K or V) stored as D/64
// boxes of [rows x 128 bytes] (box_bytes apart) with the 128-byte TMA swizzle.
__device__ __forceinline__ uint32_t swz(uint32_t base, int box_bytes, int row, int col) {
  const int box = col >> 6, chunk = (col & 63) >> 3;
  return base + box * box_bytes + row * 128 + (((chunk ^ (row & 7)) << 4) | ((col & 7) << 1));
}

// Shared-memory layout of the TMA kernel's epilogue: the per-warp O rows,
// padded to D + 4 floats (conflict-free fragment stores), reuse the then idle
// ring.  The cluster merge adds an exchange area after the kernel's other
// shared memory, used in rank 0: one (O, m, l) slot per cluster rank.
template <int D, int GP, int W> struct TmaEpi {
  static constexpr int DP = D + 4;
  static constexpr int kO = 0;  // [W][GP][DP] floats at the ring's start
  static constexpr size_t ring_bytes() { return sizeof(float) * (size_t)W * GP * DP; }
  static constexpr size_t exchange_bytes(int ranks) {
    return sizeof(float) * (size_t)ranks * GP * (D + 2);
  }
};

// Tail shared by the TMA-fed kernels: `fold(it, h, d, acc, M, L)` yields
// the CTA's partial for output item `it` (head h, dims d..d+3): unnormalised
// O, running max M and sum L.  A single split stores O / L; the cluster merge
// (CL) gathers every rank's partial in rank 0's exchange area `x_base`
// (distributed shared memory) and rank 0 merges; otherwise partials go to
// global scratch and the last split by atomic ticket merges them (`buf` is
// shared scratch for that merge).
template <typename T, int D, int GP, bool CL, typename Fold>
__device__ __forceinline__ void finish_split(const AttnArgs &a, Fold &fold, T *out, int row, int kvh,
                                             int split, int active, int group, float *x_base,
                                             float *buf, int *s_last) {
  T *orow = out + ((int64_t)row * a.Hq + kvh * group) * D;
  constexpr int kItems = GP * D / 4;  // float4 items of the CTA's [GP][D] output
  if (CL) {
    // Cluster merge: every rank writes (M, L, O) into its slot of rank 0's
    // exchange area (outside the ring, so no rank waits for another's loop
    // before writing); rank 0 merges the slots and stores.
    const uint32_t rank = cluster_rank(), ranks = gridDim.x;
    float *x_o = x_base;                                 // [ranks][GP][D]
    float *x_ml = x_o + (size_t)ranks * GP * D;                        // [ranks][2][GP]
    const uint32_t x_o0 = cluster_map(smem_u32(x_o), 0), x_ml0 = cluster_map(smem_u32(x_ml), 0);
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");  // every rank is running
    for (int it = threadIdx.x; it < kItems; it += blockDim.x) {
      int h, d;
      float4 acc;
      float M, L;
      fold(it, h, d, acc, M, L);
      st_cluster(x_o0 + 4u * (uint32_t)((rank * GP + h) * D + d), acc);
      if (d == 0) {
        st_cluster(x_ml0 + 4u * (rank * 2 * GP + h), M);
        st_cluster(x_ml0 + 4u * (rank * 2 * GP + GP + h), L);
      }
    }
    cluster_sync_all();  // every slot written
    if (rank != 0) return;
    for (int it = threadIdx.x; it < kItems; it += blockDim.x) {
      const int h = it / (D / 4), d = (it % (D / 4)) * 4;
      if (h >= group) continue;
      float M = -INFINITY;
      for (uint32_t r = 0; r < ranks; ++r) M = fmaxf(M, x_ml[r * 2 * GP + h]);
      float L = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (uint32_t r = 0; r < ranks; ++r) {
        const float mr = x_ml[r * 2 * GP + h];
        const float f = (mr == -INFINITY) ? 0.f : exp2f(mr - M);
        L += x_ml[r * 2 * GP + GP + h] * f;
        const float4 v = *reinterpret_cast<const float4 *>(x_o + (r * GP + h) * D + d);
        acc.x += v.x * f;
        acc.y += v.y * f;
        acc.z += v.z * f;
        acc.w += v.w * f;
      }
      const float inv = 1.f / L;
      store4<T>(orow + h * D + d, make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
    }
    return;
  }

  const int64_t part_floats = (int64_t)GP * (2 + D);
  float *part_base = a.scratch + ((int64_t)row * a.Hk + kvh) * a.num_splits * part_floats;
  float *part = part_base + (int64_t)split * part_floats;
  for (int it = threadIdx.x; it < kItems; it += blockDim.x) {
    int h, d;
    float4 acc;
    float M, L;
    fold(it, h, d, acc, M, L);
    if (active == 1) {
      if (h < group) {
        const float inv = 1.f / L;
        store4<T>(orow + h * D + d, make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
      }
    } else {
      *reinterpret_cast<float4 *>(part + 2 * GP + h * D + d) = acc;
      if (d == 0) {
        part[h] = M;
        part[GP + h] = L;
      }
    }
  }
  if (active == 1) return;
  // Publish and take a ticket; the last split of the (row, kv head) merges
  // every partial.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&a.counters[row * a.Hk + kvh], 1);
    *s_last = (prev == active - 1);
  }
  __syncthreads();
  if (!*s_last) return;
  __threadfence();
  merge_published<T, D, GP>(part_base, part_floats, active, orow, group * D, buf);
  if (threadIdx.x == 0) a.counters[row * a.Hk + kvh] = 0;
}

// Warp roles: kTmaWarps consumer warps each own 16 tokens of every stage; the
// last warp (the producer) issues every copy.  Consumers release a stage on
// its "empty" mbarrier instead of a CTA barrier, so they never wait for one
// another inside the loop: warps sharing a scheduler drift into different
// phases (one in the products while the other is in the softmax), which keeps
// the mma pipe busy.  The producer refills a slot as soon as every consumer
// has released it.
template <typename T, int D, int NT, int NS, int kTmaWarps, bool CL>
__global__ void __launch_bounds__((kTmaWarps + 1) * 32)
draft_attention_tma_kernel(const __grid_constant__ CUtensorMap tmk,
                           const __grid_constant__ CUtensorMap tmv, const AttnArgs a) {
  constexpr int kProducer = kTmaWarps;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool producer = warp == kProducer;
  using Cfg = TmaCfg<D, NS, kTmaWarps>;
  constexpr int KS = D / 16, NM = D / 16, GP = NT * 8;
  constexpr int kStageTok = Cfg::kStageTok, kBoxBytes = Cfg::kBoxBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *ring = smem;  // [NS][K boxes | V boxes], 1024-byte aligned
  uint64_t *bars = reinterpret_cast<uint64_t *>(ring + Cfg::kRingBytes);  // full[NS], empty[NS]
  float *s_m = reinterpret_cast<float *>(ring + Cfg::kRingBytes + Cfg::kBarBytes);
  float *s_l = s_m + kTmaWarps * GP;                     // [warps][GP]
  T *s_p = reinterpret_cast<T *>(s_l + kTmaWarps * GP);  // [warps][hi, lo][16][GP], 16-B aligned
  __shared__ int s_last, s_abort, s_first_unwaited;

  const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const int g = lane >> 2, t = lane & 3;
  const int group = a.Hq / a.Hk;
  T *out = static_cast<T *>(a.out);
  const uint32_t ring_u32 = smem_u32(ring);
  const uint32_t full_u32 = smem_u32(bars), empty_u32 = full_u32 + 8 * NS;
  // Independent of any global data, so it overlaps the previous kernel: the
  // descriptor prefetch and the mbarrier set-up, made visible to every warp.
  if (producer && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmv)) : "memory");
    for (int s = 0; s < NS; ++s) {
      mbar_init(full_u32 + 8 * s);                             // one expect_tx arrival + the bytes
      mbar_init_count(empty_u32 + 8 * s, Cfg::kGroupWarps);  // one arrival per warp of the group
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
    s_first_unwaited = INT_MAX;
  }
  __syncthreads();
  pdl_begin();
  // Cluster merge: arrive on the "all ranks started" phase right away; the
  // matching wait comes just before the first remote shared-memory store.
  if (CL) asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
  if (row >= a.rows) {
    if (split == 0) zero_heads<T, D>(out, row, a.Hq, kvh * group, group);
    return;
  }
  // Q^T B-fragments in natural head-dim order: lane (g, t) holds head
  // nt*8+g, dims 16s + 2t, 2t+1 and 16s + 8 + 2t, 2t+1.  Loaded before the
  // slot is known so their latency overlaps the slot / position reads.
  uint32_t qf[NT][KS][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int h = nt * 8 + g;
    const uint32_t *qp = reinterpret_cast<const uint32_t *>(
        static_cast<const T *>(a.query) + ((int64_t)row * a.Hq + kvh * group + min(h, group - 1)) * D);
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      qf[nt][s][0] = (!producer && h < group) ? qp[8 * s + t] : 0u;
      qf[nt][s][1] = (!producer && h < group) ? qp[8 * s + 4 + t] : 0u;
    }
  }
  // the producer also fetches the step's new K / V rows (written below if
  // this split owns the new position)
  constexpr int VE = 16 / sizeof(T), kNewVecs = 2 * (D / VE), kNewPerLane = (kNewVecs + 31) / 32;
  uint4 new_kv[kNewPerLane];
  if (producer) {
#pragma unroll
    for (int j = 0; j < kNewPerLane; ++j) {
      const int i = lane + 32 * j;
      const T *src = static_cast<const T *>(i < D / VE ? a.key : a.value) +
                     ((int64_t)row * a.Hk + kvh) * D + (i % (D / VE)) * VE;
      new_kv[j] = (i < kNewVecs) ? *reinterpret_cast<const uint4 *>(src) : make_uint4(0, 0, 0, 0);
    }
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
  // With the cluster merge every CTA of the cluster must reach the cluster
  // barriers, so splits past the sequence stay and contribute nothing.
  if (!CL && split >= active) return;
  const bool live = split < active;
  const int ts = live ? split * a.split_tokens : 0;
  const int te = live ? min(len, ts + a.split_tokens) : 0;
  const int64_t head_row0 = ((int64_t)slot * a.Hk + kvh) * a.W;  // tensor-map row of token 0
  const int n_stages = (te - ts + kStageTok - 1) / kStageTok;

  auto issue = [&](int k) {  // producer lane 0 only
    const int s = k % NS;
    const uint32_t kb = ring_u32 + s * Cfg::kStageBytes;
    const uint32_t vb = kb + Cfg::kBoxes * kBoxBytes;
    const int y = (int)(head_row0 + ts + k * kStageTok);
    mbar_expect_tx(full_u32 + 8 * s, Cfg::kStageBytes);
#pragma unroll
    for (int b = 0; b < Cfg::kBoxes; ++b) {
      tma_load_2d(kb + b * kBoxBytes, &tmk, 64 * b, y, full_u32 + 8 * s);
      tma_load_2d(vb + b * kBoxBytes, &tmv, 64 * b, y, full_u32 + 8 * s);
    }
  };
  int issued = 0;  // producer lane 0: stages 0 .. issued-1 have copies in flight or landed
  if (producer) {
    // Stages before the one holding the new position are issued at once; the
    // owner split then stores the new token (each lane fences its stores for
    // the async proxy) before the stage that reads it back is issued.
    const bool owner = pos >= ts && pos < te;
    const int n_first = min(NS, n_stages);
    const int k_pos = owner ? (pos - ts) / kStageTok : n_first;
    if (lane == 0)
      for (int k = 0; k < min(n_first, k_pos); ++k) issue(k);
    if (owner) {
      T *dst = static_cast<T *>(a.wk) + (head_row0 + pos) * D;
      T *dsv = static_cast<T *>(a.wv) + (head_row0 + pos) * D;
#pragma unroll
      for (int j = 0; j < kNewPerLane; ++j) {
        const int i = lane + 32 * j;
        if (i < kNewVecs)
          *reinterpret_cast<uint4 *>((i < D / VE ? dst : dsv) + (i % (D / VE)) * VE) = new_kv[j];
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __syncwarp();
    }
    if (lane == 0)
      for (int k = min(n_first, k_pos); k < n_first; ++k) issue(k);
    issued = n_first;
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
  bool ok = true;
  if (!producer) {
    T *pw = s_p + warp * 2 * 16 * GP;  // hi tile; the lo tile follows
    const int wg = warp / Cfg::kGroupWarps, wr = warp % Cfg::kGroupWarps;
    for (int k = wg; k < n_stages; k += Cfg::kGroups) {
      const int s = k % NS;
      // After a timed-out wait (here or in another warp) no stage is waited
      // for any more; the vote keeps the warp converged for the mma/ldmatrix.
      const bool got =
          __all_sync(0xffffffffu, ok && !s_abort && mbar_wait(full_u32 + 8 * s, (k / NS) & 1));
      if (!got) {
        if (ok && lane == 0) {
          atomicMin(&s_first_unwaited, k);
          s_abort = 1;
        }
        ok = false;
      }
      const int base = ts + k * kStageTok + wr * 16;  // this warp's first token
      if (ok && base < te) {
        const uint32_t kb = ring_u32 + s * Cfg::kStageBytes;
        const uint32_t vb = kb + Cfg::kBoxes * kBoxBytes;
        const int r0 = wr * 16;
        if (base + 16 > te) {  // zero V rows past the split so 0 * stale data stays 0
          uint8_t *vgen = ring + s * Cfg::kStageBytes + Cfg::kBoxes * kBoxBytes;
          for (int i = lane; i < 16 * (D / 8); i += 32) {
            const int r = i / (D / 8), col = (i % (D / 8)) * 8;
            if (base + r >= te)
              *reinterpret_cast<uint4 *>(vgen + (swz(0, kBoxBytes, r0 + r, col))) = make_uint4(0, 0, 0, 0);
          }
          __syncwarp();
        }
        // S^T = K Q^T with two accumulators per n-tile to halve the mma chain
        float cacc[NT][2][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int c = 0; c < 4; ++c) cacc[nt][h][c] = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < KS; ++s2) {
          uint32_t af[4];
          ldsm_x4(af, swz(kb, kBoxBytes, r0 + (lane & 7) + (((lane >> 3) & 1) << 3), 16 * s2 + ((lane >> 4) << 3)));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Mma<T>::run(cacc[nt][s2 & 1], af, qf[nt][s2]);
        }
        const bool va = base + g < te, vb_ok = base + g + 8 < te;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float x[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const bool valid = (c < 2) ? va : vb_ok;
            x[c] = valid ? (cacc[nt][0][c] + cacc[nt][1][c]) * a.scale_log2 : -INFINITY;
          }
          // Lazy rescale: the running max moves only when some score exceeds
          // it by more than 2^8.  One vote finds out whether any head of the
          // warp's tile does; only then are the head maxima reduced.
          const bool grow = fmaxf(x[0], x[2]) > m_run[nt][0] + kLazyRescale ||
                            fmaxf(x[1], x[3]) > m_run[nt][1] + kLazyRescale;
          if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              float mx = fmaxf(x[j], x[j + 2]);
#pragma unroll
              for (int off = 4; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
              const float m_old = m_run[nt][j];
              if (mx > m_old + kLazyRescale) {
                const float alpha = (m_old == -INFINITY) ? 0.f : exp2f(m_old - mx);
                l_run[nt][j] *= alpha;
#pragma unroll
                for (int i = 0; i < NM; ++i) {
                  o[nt][i][j] *= alpha;
                  o[nt][i][j + 2] *= alpha;
                }
                m_run[nt][j] = mx;
              }
            }
          }
          float p[4];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            p[j] = exp2f(x[j] - m_run[nt][j]);
            p[j + 2] = exp2f(x[j + 2] - m_run[nt][j]);
            l_run[nt][j] += p[j] + p[j + 2];
          }
          uint32_t *prow = reinterpret_cast<uint32_t *>(pw);
          uint32_t *prow_lo = prow + 16 * GP / 2;
          pack2_split<T>(p[0], p[1], prow[(g * GP + nt * 8 + 2 * t) / 2],
                         prow_lo[(g * GP + nt * 8 + 2 * t) / 2]);
          pack2_split<T>(p[2], p[3], prow[((g + 8) * GP + nt * 8 + 2 * t) / 2],
                         prow_lo[((g + 8) * GP + nt * 8 + 2 * t) / 2]);
        }
        __syncwarp();
        uint32_t pb[NT][2], pl[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          ldsm_x2_trans(pb[nt], pw + (lane & 15) * GP + nt * 8);
          ldsm_x2_trans(pl[nt], pw + 16 * GP + (lane & 15) * GP + nt * 8);
        }
        __syncwarp();
        // O^T += V^T P^T, V^T fragments straight from the swizzled tile
#pragma unroll
        for (int i = 0; i < NM; ++i) {
          uint32_t vf[4];
          ldsm_x4_t(vf, swz(vb, kBoxBytes, r0 + (lane & 7) + ((lane >> 4) << 3), 16 * i + (((lane >> 3) & 1) << 3)));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            Mma<T>::run(o[nt][i], vf, pb[nt]);
            Mma<T>::run(o[nt][i], vf, pl[nt]);
          }
        }
      }
      __syncwarp();  // every lane's reads of slot s are done
      if (lane == 0) mbar_arrive(empty_u32 + 8 * s);
    }
  } else if (lane == 0) {
    // Refill each slot once every consumer warp has released it; stop at the
    // first sign of an abort (a consumer's timed-out wait is published before
    // its release of the same stage, so it is seen here).
    for (int k = issued; k < n_stages; ++k) {
      const int s = k % NS;
      if (!mbar_wait(empty_u32 + 8 * s, ((k / NS) - 1) & 1)) {
        ok = false;
        s_abort = 1;
        break;
      }
      if (s_abort) break;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(k);
      ++issued;
    }
  }
  __syncthreads();  // every consumer is done with the ring
  if (!ok && lane == 0) flag_error(a.err, DSB_FLAG_TIMEOUT);
  if (s_abort) {  // CTA-uniform after the barrier
    // Let every issued copy that no consumer saw land (bounded again) before
    // the ring is reused for the O staging below or released with the CTA.
    if (producer && lane == 0)
      for (int k = min(s_first_unwaited, issued); k < issued; ++k)
        mbar_wait(full_u32 + 8 * (k % NS), (k / NS) & 1);
    __syncthreads();
  }

  // ---- combine the warps of this CTA (the ring is idle from here on)
  using Epi = TmaEpi<D, GP, kTmaWarps>;
  float *e_o = reinterpret_cast<float *>(ring) + Epi::kO;  // [warps][GP][DP], unscaled
  if (!producer) {
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
          const int d = 16 * i + g + ((c >= 2) ? 8 : 0);
          e_o[(warp * GP + h) * Epi::DP + d] = o[nt][i][c];
        }
    }
  }
  __syncthreads();
  // Item `it` (head h, dims d..d+3): fold the warps with weights
  // exp2(m_w - M) into the CTA's partial (acc, M, L).
  auto fold = [&](int it, int &h, int &d, float4 &acc, float &M, float &L) {
    h = it / (D / 4);
    d = (it % (D / 4)) * 4;
    M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTmaWarps; ++w) M = fmaxf(M, s_m[w * GP + h]);
    L = 0.f;
    acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kTmaWarps; ++w) {
      const float mw = s_m[w * GP + h];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      L += s_l[w * GP + h] * f;
      const float4 v = *reinterpret_cast<const float4 *>(e_o + (w * GP + h) * Epi::DP + d);
      acc.x += v.x * f;
      acc.y += v.y * f;
      acc.z += v.z * f;
      acc.w += v.w * f;
    }
  };

  finish_split<T, D, GP, CL>(a, fold, out, row, kvh, split, active, group,
                             reinterpret_cast<float *>(s_p + kTmaWarps * 2 * 16 * GP), e_o, &s_last);
}


bool legacy_attention_requested() {
  const char *v = getenv("DSB_ATTENTION_LEGACY");
  return v != nullptr && v[0] == '1';
}

// DSB_ATTENTION_TICKET_MERGE=1 keeps the TMA kernel but merges splits through
// global partials (the path used above 8 splits), so tests cover both merges.
bool legacy_merge_requested() {
  const char *v = getenv("DSB_ATTENTION_TICKET_MERGE");
  return v != nullptr && v[0] == '1';
}

template <typename T, int D, int NT, int NS, int W>
int launch_tma(const AttnArgs &a, int splits, cudaStream_t st) {
  CUtensorMap tmk, tmv;
  const int64_t rows_total = (int64_t)a.num_slots * a.Hk * a.W;
  const int dt = std::is_same<T, __half>::value ? DSB_F16 : DSB_BF16;
  if (!encode_kv_map(&tmk, a.wk, rows_total, D, dt, TmaCfg<D, NS, W>::kStageTok) ||
      !encode_kv_map(&tmv, a.wv, rows_total, D, dt, TmaCfg<D, NS, W>::kStageTok))
    return -1;  // no tensor map: the caller uses the register-fed kernel
  const size_t smem = tma_smem_bytes<T, D, NT, NS, W>();
  using Epi = TmaEpi<D, NT * 8, W>;
  static_assert(Epi::ring_bytes() <= TmaCfg<D, NS, W>::kRingBytes,
                "the epilogue staging must fit in the ring");
  const dim3 grid(splits, a.Hk, a.out_rows);
  const dim3 block((W + 1) * 32);  // W consumer warps + the producer warp
  // 2..8 splits: merge through distributed shared memory inside a cluster of
  // the (row, kv head)'s splits; otherwise through global partials and an
  // atomic ticket.  The ticket merge is also taken when the clusters would
  // need a second wave while the plain grid fits in one (one CTA per SM).
  constexpr size_t kMaxSmem = 227 * 1024;
  const size_t smem_cl = smem + Epi::exchange_bytes(splits);
  if (splits >= 2 && splits <= 8 && smem_cl <= kMaxSmem && !legacy_merge_requested()) {
    auto kern = draft_attention_tma_kernel<T, D, NT, NS, W, true>;
    if (int e = ensure_smem((const void *)kern, smem_cl); e != DSB_OK) return e;
    const int64_t clusters = (int64_t)a.Hk * a.out_rows;
    const int fit = max_active_clusters((const void *)kern, splits, block.x, smem_cl);
    if (fit > 0 && (clusters <= fit || clusters * splits > sm_count())) {
      launch_kernel_cluster(kern, grid, block, smem_cl, st, splits, tmk, tmv, a);
      return check_launch("draft_attention_tma_kernel (cluster merge)");
    }
  }
  auto kern = draft_attention_tma_kernel<T, D, NT, NS, W, false>;
  if (int e = ensure_smem((const void *)kern, smem); e != DSB_OK) return e;
  launch_kernel(kern, grid, block, smem, st, tmk, tmv, a);
  return check_launch("draft_attention_tma_kernel");
}

// Geometry of the TMA kernel: 8 consumer warps and 64-token stages up to
// head_dim 128 (a 192 KB ring at 128, one CTA per SM), 4 warps and 32-token
// stages at 256 (128 KB).
template <int D> struct TmaGeom {
  static constexpr int W = D >= 256 ? 4 : 8;
  static constexpr int NS = D >= 256 ? 4 : (D >= 128 ? 6 : 8);
};

template <typename T, int D, int NT>
int launch_attention_typed(const AttnArgs &a, int splits, cudaStream_t st) {
  if (!legacy_attention_requested()) {
    const int e = launch_tma<T, D, NT, TmaGeom<D>::NS, TmaGeom<D>::W>(a, splits, st);
    if (e != -1) return e;
  }
  const size_t smem = attn_smem_bytes<T, D, NT>();
  auto kern = draft_attention_kernel<T, D, NT>;
  if (int e = ensure_smem((const void *)kern, smem); e != DSB_OK) return e;
  launch_kernel(kern, dim3(splits, a.Hk, a.out_rows), dim3(kAttnWarps * 32), smem, st, a);
  return check_launch("draft_attention_kernel");
}

int launch_attention(const AttnArgs &a, int dtype, int head_dim, int group, int splits,
                     cudaStream_t st) {
  const int nt = group <= 8 ? 1 : 2;
#define DSB_LA(TT, DD, NN) \
  if (head_dim == DD && nt == NN) return launch_attention_typed<TT, DD, NN>(a, splits, st);
  if (dtype == DSB_BF16) {
    DSB_LA(__nv_bfloat16, 64, 1) DSB_LA(__nv_bfloat16, 64, 2)
    DSB_LA(__nv_bfloat16, 128, 1) DSB_LA(__nv_bfloat16, 128, 2)
    DSB_LA(__nv_bfloat16, 256, 1) DSB_LA(__nv_bfloat16, 256, 2)
  } else {
    DSB_LA(__half, 64, 1) DSB_LA(__half, 64, 2)
    DSB_LA(__half, 128, 1) DSB_LA(__half, 128, 2)
    DSB_LA(__half, 256, 1) DSB_LA(__half, 256, 2)
  }
#undef DSB_LA
  return fail(DSB_ERR_UNSUPPORTED, "no draft attention kernel for this shape");
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int32_t dsb_draft_attention_default_splits(int32_t rows, int32_t num_kv_heads,
                                                      int32_t working_budget, int32_t sm_count) {
  if (rows <= 0 || num_kv_heads <= 0 || working_budget <= 0) return 1;
  if (sm_count <= 0) sm_count = 148;
  const int64_t pairs = (int64_t)rows * num_kv_heads;
  int64_t splits = (int64_t)sm_count / pairs;  // about one resident CTA per SM
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
  return launch_attention(a, dtype, head_dim, group, splits, st);
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
  return launch_attention(a, dtype, head_dim, group, splits, st);
}
