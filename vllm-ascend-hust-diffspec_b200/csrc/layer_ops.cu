// Elementwise ops of one draft decoder layer: RMSNorm, NeoX RoPE of the
// step's queries and keys, and the SwiGLU activation.
//
// Reference: the draft model of diffspec is a vLLM Eagle3 Llama layer (its
// qkv input is the embedding concatenated with the target hidden state,
// diffspec/vllm_patch.py:189-225) whose RoPE positions are the working
// cache's local positions (diffspec/runtime.py:1767-1794).  Between the
// GEMMs a decode step of that layer runs three elementwise stages; each is a
// handful of small tensor ops in eager PyTorch (one launch per op, ~2-3 us
// each for a 16-row step), here one launch apiece:
//   * rms_norm:   out = round(round(x * rsqrt(mean(x^2) + eps)) * w), fp32
//                 math, rounded where vLLM's rms_norm rounds (the normalised
//                 value to the weight dtype, then the product);
//   * rope_qk:    queries of the step rotated in place and keys rotated
//                 out of the K/V projection's packed rows into the
//                 contiguous rows the draft attention reads, values copied
//                 beside them (NeoX halves, products rounded before the add,
//                 as in the working-cache rebuild);
//   * silu_mul:   out = round(round(silu(gate)) * up) over a [rows, 2 * inter]
//                 GEMM output holding gate then up (vLLM SiluAndMul's rounding
//                 points).
// All three are latency bound at decode sizes (tens of KB per launch): one
// CTA per row (norm), one warp per (token, head) (RoPE), a grid-stride loop
// of 16-byte vectors (activation), with programmatic dependent launch so a
// launch overlaps the previous kernel's tail.
#include <algorithm>

#include "common.cuh"
#include "peer.cuh"

namespace dsb {
namespace {

constexpr int kNormThreads = 256;

template <typename T>
__device__ __forceinline__ void load8(const T *p, float (&v)[8]) {
  const uint4 w = *reinterpret_cast<const uint4 *>(p);
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack2<T>(u[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T *p, const float (&v)[8]) {
  uint4 w;
  w.x = pack2<T>(v[0], v[1]);
  w.y = pack2<T>(v[2], v[3]);
  w.z = pack2<T>(v[4], v[5]);
  w.w = pack2<T>(v[6], v[7]);
  *reinterpret_cast<uint4 *>(p) = w;
}

// One CTA per row; cols is a multiple of 8 and rows are 16-byte aligned.
template <typename T>
__global__ void __launch_bounds__(kNormThreads)
    rms_norm_kernel(const T *__restrict__ x, int64_t x_stride, const T *__restrict__ w,
                    T *__restrict__ out, int64_t out_stride, int cols, float eps) {
  __shared__ float part[kNormThreads / 32];
  pdl_begin();
  const T *row = x + blockIdx.x * x_stride;
  const int vecs = cols / 8;
  float ss = 0.f;
  for (int v = threadIdx.x; v < vecs; v += kNormThreads) {
    float f[8];
    load8(row + 8 * v, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) total += part[i];
  const float inv = rsqrtf(total / static_cast<float>(cols) + eps);
  T *orow = out + blockIdx.x * out_stride;
  for (int v = threadIdx.x; v < vecs; v += kNormThreads) {
    float f[8], g[8];
    load8(row + 8 * v, f);
    load8(w + 8 * v, g);
#pragma unroll
    for (int i = 0; i < 8; ++i)  // normalised value rounded to T, then times the weight
      f[i] = __fmul_rn(Elem<T>::to_f(Elem<T>::from_f(__fmul_rn(f[i], inv))), g[i]);
    store8(orow + 8 * v, f);
  }
}

// x = round(partial + residual) per element (fp32 add, one rounding: what a
// residual epilogue of one whole linear gives), stored to x_out; then, when
// w is set, norm_out = rms_norm(x) with exactly rms_norm_kernel's arithmetic
// (same per-thread vectors, reduction tree and rounding points), so a
// tensor-parallel layer whose linears all-reduce fp32 partials reaches the
// same values as the single-GPU layer up to the partials' summation order.
// One CTA per row; cols a multiple of 8.
// The peer variant's view of this rank's exchange buffer (peer.cuh).
struct PeerIn {
  const uint8_t *data;  // [2][world][tokens_max][cols] (value, tag) words
  uint32_t *sync;       // epoch, consumer ticket
  int world, tmax;
};

// PEER: the fp32 partial of (row, c) is the sum, in rank order, of every
// rank's partial in this rank's exchange buffer, each read once it carries
// the call's tag (bounded wait); the last CTA advances the epoch.
template <typename T, bool PEER>
__global__ void __launch_bounds__(kNormThreads)
    add_rms_norm_kernel(const float *__restrict__ part, int64_t p_stride,
                        const T *__restrict__ res, int64_t r_stride, const T *__restrict__ w,
                        T *__restrict__ x_out, int64_t x_stride, T *__restrict__ out,
                        int64_t out_stride, int cols, float eps, PeerIn pin, int32_t *err) {
  __shared__ float red[kNormThreads / 32];
  pdl_begin();
  uint32_t epoch = 0;
  const uint8_t *prow8 = nullptr;  // PEER: this row of rank 0's words of the call
  if (PEER) {
    epoch = *reinterpret_cast<volatile const uint32_t *>(pin.sync);
    prow8 = pin.data +
            (((int64_t)(epoch & 1u) * pin.world * pin.tmax + blockIdx.x) * cols) * 8;
  }
  const float *prow = PEER ? nullptr : part + blockIdx.x * p_stride;
  const int64_t rank_stride = PEER ? (int64_t)pin.tmax * cols * 8 : 0;  // bytes
  const T *rrow = res + blockIdx.x * r_stride;
  T *xrow = x_out + blockIdx.x * x_stride;
  const int vecs = cols / 8;
  float ss = 0.f;
  bool late = false;
  auto sum8 = [&](int v, float (&f)[8]) {
    float pv[8];
    if (PEER) {
      late |= !ld_tagged8(prow8 + (int64_t)v * 64, epoch + 1u, pv, !late);
      for (int q = 1; q < pin.world; ++q) {
        float pq[8];
        late |= !ld_tagged8(prow8 + q * rank_stride + (int64_t)v * 64, epoch + 1u, pq, !late);
#pragma unroll
        for (int i = 0; i < 8; ++i) pv[i] = __fadd_rn(pv[i], pq[i]);
      }
    } else {
      const float4 a = *reinterpret_cast<const float4 *>(prow + 8 * v);
      const float4 b = *reinterpret_cast<const float4 *>(prow + 8 * v + 4);
      pv[0] = a.x, pv[1] = a.y, pv[2] = a.z, pv[3] = a.w;
      pv[4] = b.x, pv[5] = b.y, pv[6] = b.z, pv[7] = b.w;
    }
    float r[8];
    load8(rrow + 8 * v, r);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = Elem<T>::to_f(Elem<T>::from_f(__fadd_rn(pv[i], r[i])));
  };
  for (int v = threadIdx.x; v < vecs; v += kNormThreads) {
    float f[8];
    sum8(v, f);
    store8(xrow + 8 * v, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
  }
  if (w != nullptr) {
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) total += red[i];
    const float inv = rsqrtf(total / static_cast<float>(cols) + eps);
    T *orow = out + blockIdx.x * out_stride;
    for (int v = threadIdx.x; v < vecs; v += kNormThreads) {
      float f[8], g[8];
      sum8(v, f);
      load8(w + 8 * v, g);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        f[i] = __fmul_rn(Elem<T>::to_f(Elem<T>::from_f(__fmul_rn(f[i], inv))), g[i]);
      store8(orow + 8 * v, f);
    }
  }
  if (PEER) {
    if (late) flag_error(err, DSB_FLAG_TIMEOUT);
    // every CTA has read the call's epoch and data: the last one advances it
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(pin.sync + 1, 1u) == gridDim.x - 1) {
      pin.sync[1] = 0;
      pin.sync[0] = epoch + 1u;
    }
  }
}

struct RopeArgs {
  void *q;
  const void *k, *v;
  void *k_out, *v_out;
  int64_t q_stride, k_stride, v_stride;  // elements between tokens
  const void *cos_sin;
  int64_t cs_stride;
  const int32_t *positions;
  int pos_offset;
  int tokens, hq, hk, hv, head_dim, half, rotary_rows;
  int32_t *error_flag;
};

// One warp per (token, head) over hq query heads (rotated in place), hk key
// heads (rotated from k into k_out) and hv value heads (copied from v into
// v_out): element i of a head pairs with element i + half.  A position
// outside the table leaves the token's rows unrotated (keys still copied)
// and sets DSB_FLAG_POSITION.
template <typename T, typename CS>
__global__ void __launch_bounds__(256) rope_qk_kernel(RopeArgs a) {
  pdl_begin();
  const int warp = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = a.hq + a.hk + a.hv;
  if (warp >= a.tokens * heads) return;
  const int t = warp / heads, h = warp % heads;
  const int64_t hd = a.head_dim;
  if (h >= a.hq + a.hk) {  // value head: plain copy into the contiguous layout
    const T *src = static_cast<const T *>(a.v) + t * a.v_stride + (h - a.hq - a.hk) * hd;
    T *dst = static_cast<T *>(a.v_out) + (static_cast<int64_t>(t) * a.hv + h - a.hq - a.hk) * hd;
    for (int i = lane; i < a.head_dim; i += 32) dst[i] = src[i];
    return;
  }
  const T *src = h < a.hq ? static_cast<const T *>(a.q) + t * a.q_stride + h * hd
                          : static_cast<const T *>(a.k) + t * a.k_stride + (h - a.hq) * hd;
  T *dst = h < a.hq ? static_cast<T *>(a.q) + t * a.q_stride + h * hd
                    : static_cast<T *>(a.k_out) + (static_cast<int64_t>(t) * a.hk + h - a.hq) * hd;
  const int pos = a.positions[t] + a.pos_offset;
  if (pos < 0 || pos >= a.rotary_rows) {
    if (lane == 0 && h == 0) flag_error(a.error_flag, DSB_FLAG_POSITION);
    if (src != dst)
      for (int i = lane; i < a.head_dim; i += 32) dst[i] = src[i];
    return;
  }
  const CS *cs = static_cast<const CS *>(a.cos_sin) + pos * a.cs_stride;
  for (int i = lane; i < a.half; i += 32) {
    const float x1 = Elem<T>::to_f(src[i]), x2 = Elem<T>::to_f(src[i + a.half]);
    const float c = Elem<CS>::to_f(cs[i]), s = Elem<CS>::to_f(cs[i + a.half]);
    dst[i] = Elem<T>::from_f(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
    dst[i + a.half] = Elem<T>::from_f(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
  }
}

// silu(g) = g / (1 + e^-g) in fp32, rounded, times up, rounded; inter % 8 == 0.
template <typename T>
__global__ void __launch_bounds__(256)
    silu_mul_kernel(const T *__restrict__ gate_up, int64_t gu_stride, T *__restrict__ out,
                    int64_t out_stride, int rows, int inter) {
  pdl_begin();
  const int vpr = inter / 8;
  const int64_t total = static_cast<int64_t>(rows) * vpr;
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = v / vpr;
    const int c = static_cast<int>(v % vpr) * 8;
    float g[8], u[8];
    load8(gate_up + r * gu_stride + c, g);
    load8(gate_up + r * gu_stride + inter + c, u);
#pragma unroll
    for (int i = 0; i < 8; ++i)  // silu(gate) rounded to T, then times up
      g[i] = __fmul_rn(Elem<T>::to_f(Elem<T>::from_f(__fdiv_rn(g[i], 1.f + expf(-g[i])))), u[i]);
    store8(out + r * out_stride + c, g);
  }
}

bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int dsb_rms_norm(const void *x, int64_t x_row_stride, const void *weight, void *out,
                            int64_t out_row_stride, int32_t rows, int32_t cols, float eps,
                            int32_t dtype, void *stream) {
  if (rows < 0 || cols <= 0) return fail(DSB_ERR_INVALID, "rows must be >= 0 and cols > 0");
  if (rows == 0) return DSB_OK;
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_INVALID, "rms_norm rows and weight must be BF16 or FP16");
  if (!x || !weight || !out) return fail(DSB_ERR_INVALID, "null pointer argument");
  if (!(eps >= 0.f)) return fail(DSB_ERR_INVALID, "eps must be >= 0");
  if (cols % 8 || x_row_stride % 8 || out_row_stride % 8 || x_row_stride < cols ||
      out_row_stride < cols || !aligned16(x) || !aligned16(weight) || !aligned16(out))
    return fail(DSB_ERR_UNSUPPORTED,
                "rms_norm needs cols and row strides that are multiples of 8 (>= cols) and "
                "16-byte aligned rows");
  const cudaStream_t st = as_stream(stream);
  if (dtype == DSB_BF16)
    launch_kernel(rms_norm_kernel<__nv_bfloat16>, dim3(rows), dim3(kNormThreads), 0, st,
                  static_cast<const __nv_bfloat16 *>(x), x_row_stride,
                  static_cast<const __nv_bfloat16 *>(weight), static_cast<__nv_bfloat16 *>(out),
                  out_row_stride, (int)cols, eps);
  else
    launch_kernel(rms_norm_kernel<__half>, dim3(rows), dim3(kNormThreads), 0, st,
                  static_cast<const __half *>(x), x_row_stride, static_cast<const __half *>(weight),
                  static_cast<__half *>(out), out_row_stride, (int)cols, eps);
  return check_launch("rms_norm_kernel");
}

extern "C" int dsb_add_rms_norm(const float *partial, int64_t partial_row_stride,
                                const void *residual, int64_t residual_row_stride,
                                const void *weight, void *x_out, int64_t x_row_stride, void *out,
                                int64_t out_row_stride, int32_t rows, int32_t cols, float eps,
                                int32_t dtype, void *stream) {
  if (rows < 0 || cols <= 0) return fail(DSB_ERR_INVALID, "rows must be >= 0 and cols > 0");
  if (rows == 0) return DSB_OK;
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_INVALID, "add_rms_norm rows and weight must be BF16 or FP16");
  if (!partial || !residual || !x_out || (weight && !out))
    return fail(DSB_ERR_INVALID, "null pointer argument");
  if (!(eps >= 0.f)) return fail(DSB_ERR_INVALID, "eps must be >= 0");
  const bool strides_ok = cols % 8 == 0 && partial_row_stride % 8 == 0 &&
                          residual_row_stride % 8 == 0 && x_row_stride % 8 == 0 &&
                          partial_row_stride >= cols && residual_row_stride >= cols &&
                          x_row_stride >= cols &&
                          (!weight || (out_row_stride % 8 == 0 && out_row_stride >= cols));
  if (!strides_ok || !aligned16(partial) || !aligned16(residual) || !aligned16(x_out) ||
      (weight && (!aligned16(weight) || !aligned16(out))))
    return fail(DSB_ERR_UNSUPPORTED,
                "add_rms_norm needs cols and row strides that are multiples of 8 (>= cols) and "
                "16-byte aligned rows");
  const cudaStream_t st = as_stream(stream);
  const PeerIn none{};
  if (dtype == DSB_BF16)
    launch_kernel(add_rms_norm_kernel<__nv_bfloat16, false>, dim3(rows), dim3(kNormThreads), 0, st,
                  partial, partial_row_stride, static_cast<const __nv_bfloat16 *>(residual),
                  residual_row_stride, static_cast<const __nv_bfloat16 *>(weight),
                  static_cast<__nv_bfloat16 *>(x_out), x_row_stride,
                  static_cast<__nv_bfloat16 *>(out), out_row_stride, (int)cols, eps, none,
                  (int32_t *)nullptr);
  else
    launch_kernel(add_rms_norm_kernel<__half, false>, dim3(rows), dim3(kNormThreads), 0, st,
                  partial, partial_row_stride, static_cast<const __half *>(residual),
                  residual_row_stride, static_cast<const __half *>(weight),
                  static_cast<__half *>(x_out), x_row_stride, static_cast<__half *>(out),
                  out_row_stride, (int)cols, eps, none, (int32_t *)nullptr);
  return check_launch("add_rms_norm_kernel");
}

extern "C" int dsb_peer_add_rms_norm(void *own_base, int32_t world, int32_t tokens_max,
                                     const void *residual, int64_t residual_row_stride,
                                     const void *weight, void *x_out, int64_t x_row_stride,
                                     void *out, int64_t out_row_stride, int32_t rows,
                                     int32_t cols, float eps, int32_t dtype, int32_t *error_flag,
                                     void *stream) {
  if (rows < 0 || cols <= 0) return fail(DSB_ERR_INVALID, "rows must be >= 0 and cols > 0");
  if (world < 1 || world > kPeerMaxWorld || rows > tokens_max)
    return fail(DSB_ERR_INVALID, "world must be in [1, 8] and rows at most the buffer's tokens");
  if (rows == 0) return DSB_OK;
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_INVALID, "add_rms_norm rows and weight must be BF16 or FP16");
  if (!own_base || !residual || !x_out || (weight && !out))
    return fail(DSB_ERR_INVALID, "null pointer argument");
  if (!(eps >= 0.f)) return fail(DSB_ERR_INVALID, "eps must be >= 0");
  const bool strides_ok = cols % 8 == 0 && residual_row_stride % 8 == 0 && x_row_stride % 8 == 0 &&
                          residual_row_stride >= cols && x_row_stride >= cols &&
                          (!weight || (out_row_stride % 8 == 0 && out_row_stride >= cols));
  if (!strides_ok || !aligned16(own_base) || !aligned16(residual) || !aligned16(x_out) ||
      (weight && (!aligned16(weight) || !aligned16(out))))
    return fail(DSB_ERR_UNSUPPORTED,
                "add_rms_norm needs cols and row strides that are multiples of 8 (>= cols) and "
                "16-byte aligned rows");
  const PeerLayout L(world, tokens_max, cols);
  uint8_t *b = static_cast<uint8_t *>(own_base);
  const PeerIn pin{b, reinterpret_cast<uint32_t *>(b + L.sync_off), (int)world, (int)tokens_max};
  const cudaStream_t st = as_stream(stream);
  if (dtype == DSB_BF16)
    launch_kernel(add_rms_norm_kernel<__nv_bfloat16, true>, dim3(rows), dim3(kNormThreads), 0, st,
                  (const float *)nullptr, (int64_t)0, static_cast<const __nv_bfloat16 *>(residual),
                  residual_row_stride, static_cast<const __nv_bfloat16 *>(weight),
                  static_cast<__nv_bfloat16 *>(x_out), x_row_stride,
                  static_cast<__nv_bfloat16 *>(out), out_row_stride, (int)cols, eps, pin,
                  error_flag);
  else
    launch_kernel(add_rms_norm_kernel<__half, true>, dim3(rows), dim3(kNormThreads), 0, st,
                  (const float *)nullptr, (int64_t)0, static_cast<const __half *>(residual),
                  residual_row_stride, static_cast<const __half *>(weight),
                  static_cast<__half *>(x_out), x_row_stride, static_cast<__half *>(out),
                  out_row_stride, (int)cols, eps, pin, error_flag);
  return check_launch("add_rms_norm_kernel (peer)");
}

extern "C" int dsb_rope_qk(void *query, int64_t query_row_stride, int32_t num_query_heads,
                           const void *key, int64_t key_row_stride, void *key_out,
                           const void *value, int64_t value_row_stride, void *value_out,
                           int32_t num_kv_heads, int32_t head_dim, const int32_t *positions,
                           int32_t position_offset, int32_t tokens, const void *cos_sin,
                           int64_t cos_sin_row_stride,
                           int32_t rotary_rows, int32_t cos_sin_dtype, int32_t dtype,
                           int32_t *error_flag, void *stream) {
  if (tokens < 0) return fail(DSB_ERR_INVALID, "negative token count");
  if (tokens == 0) return DSB_OK;
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_INVALID, "queries and keys must be BF16 or FP16");
  if (cos_sin_dtype != DSB_BF16 && cos_sin_dtype != DSB_F16 && cos_sin_dtype != DSB_F32)
    return fail(DSB_ERR_INVALID, "cos_sin must be BF16, FP16 or FP32");
  if (num_query_heads < 0 || num_kv_heads < 0 || num_query_heads + num_kv_heads <= 0)
    return fail(DSB_ERR_INVALID, "head counts must be >= 0 with at least one head");
  if (head_dim <= 0 || head_dim % 2 || rotary_rows <= 0 || cos_sin_row_stride < head_dim)
    return fail(DSB_ERR_INVALID,
                "head_dim must be even and positive; cos_sin rows hold [cos | sin] of head_dim");
  if (!positions || !cos_sin) return fail(DSB_ERR_INVALID, "null pointer argument");
  if (num_query_heads && (!query || query_row_stride < (int64_t)num_query_heads * head_dim))
    return fail(DSB_ERR_INVALID, "null query or query row stride shorter than its heads");
  const int64_t kv_row = (int64_t)num_kv_heads * head_dim;
  if (num_kv_heads && (!key || !key_out || key_row_stride < kv_row))
    return fail(DSB_ERR_INVALID, "null key / key_out or key row stride shorter than its heads");
  if (value && (!value_out || !num_kv_heads || value_row_stride < kv_row))
    return fail(DSB_ERR_INVALID, "value needs value_out and a row stride covering its heads");
  if (key_out && key_out != key && key_row_stride < kv_row)
    return fail(DSB_ERR_INVALID, "key row stride shorter than its heads");
  // key_out is contiguous [tokens, num_kv_heads, head_dim]: in place needs
  // the key rows to be that layout too.
  if (num_kv_heads && key_out == key && key_row_stride != kv_row)
    return fail(DSB_ERR_INVALID, "in-place keys must be contiguous");
  const int hv = value ? num_kv_heads : 0;
  const int64_t warps = (int64_t)tokens * (num_query_heads + num_kv_heads + hv);
  if ((warps + 7) / 8 > INT32_MAX) return fail(DSB_ERR_UNSUPPORTED, "grid too large");
  RopeArgs a{query, key, value, key_out, value_out, query_row_stride, key_row_stride,
             value_row_stride, cos_sin, cos_sin_row_stride, positions, position_offset, tokens,
             num_query_heads,
             num_kv_heads, hv, head_dim, head_dim / 2, rotary_rows, error_flag};
  const cudaStream_t st = as_stream(stream);
  const dim3 grid(static_cast<unsigned>((warps + 7) / 8)), block(256);
  auto go = [&](auto tag_t) {
    using T = decltype(tag_t);
    if (cos_sin_dtype == DSB_BF16)
      launch_kernel(rope_qk_kernel<T, __nv_bfloat16>, grid, block, 0, st, a);
    else if (cos_sin_dtype == DSB_F16)
      launch_kernel(rope_qk_kernel<T, __half>, grid, block, 0, st, a);
    else
      launch_kernel(rope_qk_kernel<T, float>, grid, block, 0, st, a);
  };
  if (dtype == DSB_BF16)
    go(__nv_bfloat16());
  else
    go(__half());
  return check_launch("rope_qk_kernel");
}

extern "C" int dsb_silu_mul(const void *gate_up, int64_t gate_up_row_stride, void *out,
                            int64_t out_row_stride, int32_t rows, int32_t intermediate,
                            int32_t dtype, void *stream) {
  if (rows < 0 || intermediate <= 0)
    return fail(DSB_ERR_INVALID, "rows must be >= 0 and intermediate > 0");
  if (rows == 0) return DSB_OK;
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_INVALID, "silu_mul rows must be BF16 or FP16");
  if (!gate_up || !out) return fail(DSB_ERR_INVALID, "null pointer argument");
  if (intermediate % 8 || gate_up_row_stride % 8 || out_row_stride % 8 ||
      gate_up_row_stride < 2 * (int64_t)intermediate || out_row_stride < intermediate ||
      !aligned16(gate_up) || !aligned16(out))
    return fail(DSB_ERR_UNSUPPORTED,
                "silu_mul needs intermediate and row strides that are multiples of 8 and "
                "16-byte aligned rows");
  const int64_t vecs = (int64_t)rows * (intermediate / 8);
  const int blocks = static_cast<int>(std::min<int64_t>((vecs + 255) / 256, 4L * sm_count()));
  const cudaStream_t st = as_stream(stream);
  if (dtype == DSB_BF16)
    launch_kernel(silu_mul_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st,
                  static_cast<const __nv_bfloat16 *>(gate_up), gate_up_row_stride,
                  static_cast<__nv_bfloat16 *>(out), out_row_stride, (int)rows, (int)intermediate);
  else
    launch_kernel(silu_mul_kernel<__half>, dim3(blocks), dim3(256), 0, st,
                  static_cast<const __half *>(gate_up), gate_up_row_stride,
                  static_cast<__half *>(out), out_row_stride, (int)rows, (int)intermediate);
  return check_launch("silu_mul_kernel");
}
