// Draft-layer KV projection with the canonical raw-KV write in its epilogue.
//
// Reference: the draft layer's qkv projection (vLLM QKVParallelLinear) whose
// K/V the DiffSpec sink op hands, before RoPE, to the canonical cache
// (diffspec/vllm_patch.py:132-178 -> DiffSpecDraftCache.capture_raw_kv /
// _write_raw, diffspec/runtime.py:1602-1618, 1797-1877): the projection
// writes K/V to a temporary and _write_raw copies them to [slot, position].
// Here one launch computes the K/V rows and stores them both to `out` (the
// tensor the draft attention consumes after RoPE) and to the raw cache rows
// the rebuild later gathers from.
//
// B200 design: out[t, f] = sum_k hidden[t, k] * weight[f, k] on the
// 5th-generation tensor cores in swap-AB form,
//   D^T[128 features x 16 tokens] = W[128 x K] . H^T[K x 16],
// A = a 128-row weight tile and B = the 16 token rows, both K-major with the
// 128-byte swizzle, brought in by TMA; fp32 accumulators in tensor memory
// (tcgen05.mma issued by one thread, tcgen05.commit to an mbarrier).  A decode
// step is weight-streaming bound (16 tokens against a [2 Hk D, K] weight), so
// K is split over a cluster of 16 CTAs (8 where 16 cannot be scheduled): each
// loads all of its k-blocks at once and reduces into its own accumulator; the
// partials meet in distributed shared memory, each rank summing 16 / ranks
// of the tile's tokens over the ranks in rank order (deterministic), and
// writes them.
// Every wait is bounded; a wait that runs out sets DSB_FLAG_TIMEOUT, and the
// CTA still frees its tensor memory and takes part in the cluster barriers.
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "tma_umma.cuh"

namespace dsb {
namespace {

constexpr int kPjThreads = 128;           // 4 warps: one TMEM lane per thread
constexpr int kPjTok = 16;                // tokens per tile (the MMA's N)
constexpr int kPjMaxK = 4096;             // hidden size limit: 64 k-blocks over the ranks
constexpr int kPjABytes = 128 * 64 * 2;   // weight box [128 rows][64 cols]
constexpr int kPjBBytes = kPjTok * 64 * 2;  // hidden box [16 rows][64 cols]

// Split-K over a cluster of RANKS CTAs (16 where the device schedules such
// clusters, else 8): every rank holds all of its k-blocks at once and, after
// the exchange, sums 16 / RANKS of the tile's tokens.
template <int RANKS> struct PjCfg {
  static constexpr int kMaxKb = kPjMaxK / 64 / RANKS;  // k-blocks per rank
  static constexpr int kTpr = kPjTok / RANKS;          // tokens each rank sums
  static constexpr int kBarOff = kMaxKb * (kPjABytes + kPjBBytes);
  static constexpr int kXchOff = kBarOff + 8 * (kMaxKb + 1) + 16;  // [ranks][128][kTpr] fp32
  static constexpr size_t kSmem = 1024 + kXchOff + sizeof(float) * RANKS * 128 * kTpr;
};

struct PjArgs {
  const int32_t *slots;
  const int64_t *positions;
  void *raw_k, *raw_v, *out;
  int T, K, N, kv_feats, num_slots;
  int64_t max_len;
  int32_t *err;
};

// DSB_KV_PROJECTION_RANKS8=1 keeps the 8-CTA clusters (both are tested).
bool pj_ranks8_requested() {
  const char *v = std::getenv("DSB_KV_PROJECTION_RANKS8");
  return v != nullptr && v[0] == '1';
}

template <typename T, int RANKS>
__global__ void __launch_bounds__(kPjThreads)
kv_projection_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap th,
                     const PjArgs a) {
  using Cfg = PjCfg<RANKS>;
  constexpr int kPjMaxKb = Cfg::kMaxKb, kPjRanks = RANKS, kTpr = Cfg::kTpr;
  extern __shared__ uint8_t pj_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(pj_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t s_a = smem_u32(smem), s_b = s_a + kPjMaxKb * kPjABytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kBarOff);  // full[kPjMaxKb], done
  const uint32_t full0 = smem_u32(bars), done = full0 + 8 * kPjMaxKb;
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(bars + kPjMaxKb + 1);
  float *xch = reinterpret_cast<float *>(smem + Cfg::kXchOff);
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5;

  // No global data yet: descriptor prefetch, barriers and tensor memory
  // overlap the previous kernel.
  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&th)) : "memory");
    for (int kb = 0; kb <= kPjMaxKb; ++kb) mbar_init(full0 + 8 * kb);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 32;" ::"r"(
                     smem_u32(s_tmem))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_begin();
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");

  const int rank = (int)cluster_rank();
  const int f0 = blockIdx.y * 128, t0 = blockIdx.z * kPjTok;
  const int nkb_all = a.K / 64;
  const int per = (nkb_all + kPjRanks - 1) / kPjRanks;  // <= kPjMaxKb (host check)
  const int kb0 = rank * per;
  const int nkb = max(0, min(per, nkb_all - kb0));
  if (tid == 0) {
    for (int kb = 0; kb < nkb; ++kb) {
      mbar_expect_tx(full0 + 8 * kb, kPjABytes + kPjBBytes);
      tma_load_2d(s_a + kb * kPjABytes, &tw, (kb0 + kb) * 64, f0, full0 + 8 * kb);
      tma_load_2d(s_b + kb * kPjBBytes, &th, (kb0 + kb) * 64, t0, full0 + 8 * kb);
    }
    const uint32_t idesc = umma_idesc<T, kPjTok>(false);
    int kb = 0;
    for (; kb < nkb; ++kb) {
      if (!mbar_wait(full0 + 8 * kb, 0)) break;
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma(tmem, umma_desc(s_a + kb * kPjABytes + ks * 32, 16, 1024),
             umma_desc(s_b + kb * kPjBBytes + ks * 32, 16, 1024), idesc, kb > 0 || ks > 0);
    }
    if (kb < nkb) {  // a copy did not land in time: let the rest land, skip the products
      flag_error(a.err, DSB_FLAG_TIMEOUT);
      for (int k2 = kb + 1; k2 < nkb; ++k2) mbar_wait(full0 + 8 * k2, 0);
      s_abort = 1;
    }
    if (nkb > 0) umma_commit(done);  // arrives once the issued products are done
  }
  __syncthreads();

  // This rank's partial: thread = feature row (TMEM lane), 16 token columns.
  float acc[kPjTok];
#pragma unroll
  for (int j = 0; j < kPjTok; ++j) acc[j] = 0.f;
  if (nkb > 0) {
    const bool got = mbar_wait(done, 0);
    if (__syncthreads_and(got) && !s_abort) {
      tc_fence_after();
      tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16), acc);
    } else if (tid == 0) {
      flag_error(a.err, DSB_FLAG_TIMEOUT);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 32;" ::"r"(tmem) : "memory");

  // Rank q sums tokens q * kTpr .. q * kTpr + kTpr - 1 over the ranks: send
  // them there.
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");  // every rank is running
  const uint32_t x0 = smem_u32(xch);
#pragma unroll
  for (int q = 0; q < kPjRanks; ++q) {
    const uint32_t remote = cluster_map(x0, (uint32_t)q) + 4u * (uint32_t)((rank * 128 + tid) * kTpr);
#pragma unroll
    for (int j = 0; j < kTpr; ++j) st_cluster(remote + 4u * j, acc[q * kTpr + j]);
  }
  cluster_sync_all();  // every partial delivered

  T *out = static_cast<T *>(a.out);
  T *raw_k = static_cast<T *>(a.raw_k), *raw_v = static_cast<T *>(a.raw_v);
  const int g = f0 + tid;  // output feature
#pragma unroll
  for (int j = 0; j < kTpr; ++j) {
    const int t = t0 + kTpr * rank + j;
    if (t >= a.T) continue;
    float v = 0.f;
#pragma unroll
    for (int r = 0; r < kPjRanks; ++r) v += xch[(r * 128 + tid) * kTpr + j];
    const T y = Elem<T>::from_f(v);
    if (out != nullptr) out[(int64_t)t * a.N + g] = y;
    const int slot = a.slots[t];
    if (slot < 0) continue;  // padding row: no cache row
    const int64_t pos = a.positions[t];
    if (slot >= a.num_slots || pos < 0 || pos >= a.max_len) {
      if (tid == 0) flag_error(a.err, slot >= a.num_slots ? DSB_FLAG_SLOT : DSB_FLAG_POSITION);
      continue;
    }
    const int64_t row = ((int64_t)slot * a.max_len + pos) * a.kv_feats;
    if (g < a.kv_feats) raw_k[row + g] = y;
    else raw_v[row + g - a.kv_feats] = y;
  }
}

// 16-CTA clusters are beyond the portable size: allowed per kernel once, and
// used only if the device can schedule one.
bool allow_cluster16(const void *kernel) {
  static std::mutex mu;
  static std::map<std::pair<int, const void *>, bool> known;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(dev, kernel);
  auto it = known.find(key);
  if (it != known.end()) return it->second;
  const bool ok =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
  if (!ok) (void)cudaGetLastError();
  known[key] = ok;
  return ok;
}

template <typename T, int RANKS>
int launch_ranks(const CUtensorMap &tw, const CUtensorMap &th, const PjArgs &a, cudaStream_t st,
                 bool &launched) {
  launched = false;
  auto kern = kv_projection_kernel<T, RANKS>;
  constexpr size_t smem = PjCfg<RANKS>::kSmem;
  if (RANKS > 8 && !allow_cluster16((const void *)kern)) return DSB_OK;
  if (int e = ensure_smem((const void *)kern, smem); e != DSB_OK) return e;
  if (max_active_clusters((const void *)kern, RANKS, kPjThreads, smem) <= 0) return DSB_OK;
  const dim3 grid(RANKS, a.N / 128, (a.T + kPjTok - 1) / kPjTok);
  launch_kernel_cluster(kern, grid, dim3(kPjThreads), smem, st, RANKS, tw, th, a);
  launched = true;
  return check_launch("kv_projection_kernel");
}

template <typename T>
int launch_kv_projection(const void *hidden, const void *weight, const PjArgs &a, int dtype,
                         cudaStream_t st) {
  CUtensorMap tw, th;
  if (!encode_kv_map(&tw, weight, a.N, a.K, dtype, 128) ||
      !encode_kv_map(&th, hidden, a.T, a.K, dtype, kPjTok))
    return fail(DSB_ERR_UNSUPPORTED, "no tensor map for the weight or hidden rows");
  bool launched = false;
  if (!pj_ranks8_requested()) {
    if (int e = launch_ranks<T, 16>(tw, th, a, st, launched); e != DSB_OK || launched) return e;
  }
  if (int e = launch_ranks<T, 8>(tw, th, a, st, launched); e != DSB_OK || launched) return e;
  return fail(DSB_ERR_UNSUPPORTED, "a cluster of 8 projection CTAs does not fit on this device");
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int dsb_kv_projection_write_raw(const void *hidden, int32_t tokens, int32_t hidden_size,
                                           const void *weight, int32_t num_kv_heads,
                                           int32_t head_dim, const int32_t *slots,
                                           const int64_t *positions, void *raw_key,
                                           void *raw_value, int32_t num_slots,
                                           int64_t max_model_len, int32_t dtype, void *out,
                                           int32_t *error_flag, void *stream) {
  if (tokens < 0) return fail(DSB_ERR_INVALID, "negative token count");
  if (tokens == 0) return DSB_OK;
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_INVALID, "hidden rows, weight and caches must be BF16 or FP16");
  if (num_kv_heads <= 0 || head_dim <= 0 || num_slots <= 0 || max_model_len <= 0)
    return fail(DSB_ERR_INVALID, "kv heads, head_dim, slots and max_model_len must be positive");
  const int64_t kv_feats = (int64_t)num_kv_heads * head_dim;
  if (kv_feats % 128)
    return fail(DSB_ERR_UNSUPPORTED, "num_kv_heads * head_dim must be a multiple of 128");
  if (hidden_size <= 0 || hidden_size % 64 || hidden_size > kPjMaxK)
    return fail(DSB_ERR_UNSUPPORTED, "hidden_size must be a multiple of 64 and at most 4096");
  if ((tokens + kPjTok - 1) / kPjTok > 65535 || 2 * kv_feats / 128 > 65535)
    return fail(DSB_ERR_UNSUPPORTED, "grid too large");
  if (!hidden || !weight || !slots || !positions || !raw_key || !raw_value)
    return fail(DSB_ERR_INVALID, "null pointer argument");
  if (reinterpret_cast<uintptr_t>(hidden) % 16 || reinterpret_cast<uintptr_t>(weight) % 16)
    return fail(DSB_ERR_UNSUPPORTED, "hidden rows and weight must be 16-byte aligned");
  PjArgs a{};
  a.slots = slots;
  a.positions = positions;
  a.raw_k = raw_key;
  a.raw_v = raw_value;
  a.out = out;
  a.T = tokens;
  a.K = hidden_size;
  a.N = (int)(2 * kv_feats);
  a.kv_feats = (int)kv_feats;
  a.num_slots = num_slots;
  a.max_len = max_model_len;
  a.err = error_flag;
  cudaStream_t st = as_stream(stream);
  return dtype == DSB_BF16 ? launch_kv_projection<__nv_bfloat16>(hidden, weight, a, dtype, st)
                           : launch_kv_projection<__half>(hidden, weight, a, dtype, st);
}
