// Shared device helpers for the DiffSpec sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "diffspec_b200.h"

namespace dsb {

// ---------------------------------------------------------------- host side
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int check_launch(const char *what);

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

int sm_count();

// Raise a kernel's dynamic shared-memory limit once per (device, kernel), so
// repeated launches (and launches during CUDA-graph capture) only enqueue.
int ensure_smem(const void *kernel, size_t bytes);

// Launch with programmatic dependent launch allowed: the kernel's CTAs may be
// scheduled while the previous kernel in the stream is finishing, and block in
// pdl_begin() (griddepcontrol.wait) until that kernel has completed and its
// memory is visible.  Every kernel of this library calls pdl_begin() before
// its first global memory access, so the overlap only hides launch latency.
// Errors surface through cudaGetLastError (check_launch).
template <typename... Params, typename... Args>
void launch_kernel(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t st, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  (void)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Same, with thread-block clusters of `cluster_x` CTAs along x.
template <typename... Params, typename... Args>
void launch_kernel_cluster(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                           cudaStream_t st, int cluster_x, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  (void)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Resident CTAs of `kernel` with this block size and dynamic shared memory on
// the current device (occupancy x SMs, at least one per SM), cached.
int resident_ctas(const void *kernel, int threads, size_t smem);

// How many clusters of `cluster_x` CTAs with this block size and shared
// memory can be resident on the device at once (0 if none can; cached per
// device, kernel, cluster size and smem).
int max_active_clusters(const void *kernel, int cluster_x, int threads, size_t smem);

// ------------------------------------------------------------ element types
template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};

// Programmatic dependent launch: wait for the previous kernel in the stream
// (a no-op when the launch had no programmatic dependency), then let the next
// kernel's CTAs start launching.
__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void flag_error(int32_t *flag, int32_t bit) {
  if (flag != nullptr) atomicOr(flag, bit);
}

// 16-byte global load that bypasses L1 allocation (streamed once).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// cp.async groups: close the current group; wait until at most N are pending.
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// L2 policy for data read once per pass (the paged target K of the chunk
// scores, the raw caches a rebuild gathers from): its lines are evicted
// first, so the working cache that the draft steps re-read keeps its lines in
// L2.  Without side effects, so the compiler may hoist it.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
#ifdef DSB_NO_L2_HINTS
  asm("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
#else
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
#endif
  return pol;
}

// ldg_stream with an L2 cache policy.
__device__ __forceinline__ uint4 ldg_stream(const void *p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ void stg_stream(void *p, const uint4 &v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// ------------------------------------------------------------- tensor cores
// D = A(16x16) * B(16x8) + D, fp32 accumulate (mma.sync m16n8k16).
template <typename T> struct Mma;
template <> struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4],
                                             const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
};
template <> struct Mma<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4],
                                             const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
};

// Pack two floats into one 32-bit register of two 16-bit elements
// (first argument in the low half).
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// The two floats of a packed 16-bit pair (low half first).
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t w);
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2 *>(&w));
}

// Softmax weights for a 16-bit P.V product as two 16-bit terms, hi + lo:
// hi = round(p), lo = round(p - hi).  Both feed the tensor cores, so the
// weights carry ~16 mantissa bits instead of 8 (bf16) and the output error
// stays at the output's own rounding even for sums over thousands of tokens.
template <typename T>
__device__ __forceinline__ void pack2_split(float a, float b, uint32_t &hi, uint32_t &lo) {
  hi = pack2<T>(a, b);
  const float2 h = unpack2<T>(hi);
  lo = pack2<T>(a - h.x, b - h.y);
}

// ldmatrix .x2 .trans of two 8x8 16-bit matrices.
__device__ __forceinline__ void ldsm_x2_trans(uint32_t (&r)[2], const void *smem_row) {
  uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr float kLog2e = 1.4426950408889634f;

// ------------------------------------------------- mbarriers (async copies)
constexpr int kWaitSpins = 1 << 26;          // poll backstop
constexpr uint64_t kWaitNs = 200000000ull;  // 0.2 s per wait

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}
// An mbarrier whose phase completes after `count` plain arrivals.
__device__ __forceinline__ void mbar_init_count(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// One arrival (release semantics: this thread's earlier shared-memory reads
// and writes are ordered before the phase completes).
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// Bounded wait on an mbarrier phase; false when the bound ran out.  The bound
// is wall-clock (kWaitNs on %globaltimer, checked every 64 polls) with a poll
// count as a backstop, so a lost copy costs a fraction of a second, not a hang.
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  uint64_t t0 = 0;
  for (int i = 0; i < kWaitSpins; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 63) == 0) {
      const uint64_t now = global_ns();
      if (i == 0) t0 = now;
      else if (now - t0 > kWaitNs) return false;
    }
  }
  return false;
}
// 1-D bulk copy (TMA, no tensor map) of `bytes` from global memory into this
// CTA's shared memory, completion counted on `bar`.  Both addresses 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
// bulk_load with an L2 cache policy for the source lines.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}

}  // namespace dsb
