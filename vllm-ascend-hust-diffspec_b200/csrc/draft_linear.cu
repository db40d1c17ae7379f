// Weight-streaming linear layers of a draft decode step on the tensor cores,
// with the epilogues the draft layer needs: the K/V projection that also
// writes the canonical raw-KV rows, the query + K/V projection in one launch,
// a residual add, and SwiGLU.
//
// Reference: the draft layer's projections (vLLM QKVParallelLinear,
// RowParallelLinear, MergedColumnParallelLinear + SiluAndMul of the Eagle3
// Llama layer whose qkv input diffspec builds at diffspec/vllm_patch.py:
// 189-225) and the sink op that hands the pre-RoPE K/V to the canonical cache
// (diffspec/vllm_patch.py:132-178 -> DiffSpecDraftCache.capture_raw_kv /
// _write_raw, diffspec/runtime.py:1602-1618, 1797-1877): the projection
// writes K/V to a temporary and _write_raw copies them to [slot, position].
// Here the epilogue stores the rows to their consumers directly.
//
// B200 design: out[t, f] = sum_k x[t, k] * weight[f, k] on the
// 5th-generation tensor cores in swap-AB form,
//   D^T[128 features x 16 tokens] = W[128 x K] . X^T[K x 16],
// A = a 128-row weight tile and B = the 16 token rows, both K-major with the
// 128-byte swizzle, brought in by TMA; fp32 accumulators in tensor memory
// (tcgen05.mma issued by one thread, tcgen05.commit to mbarriers).  A decode
// step is weight-streaming bound (16 tokens against a [N, K] weight), so K is
// split over a cluster of 1-16 CTAs (the widest whose grid holds about one
// CTA per SM); in each rank a producer warp streams its k-blocks through a
// 4-slot ring (a slot is refilled once the products reading it have
// completed) while one thread issues the products, and the partials meet in
// distributed shared memory, each rank summing 16 / ranks of the tile's
// tokens over the ranks in rank order (deterministic).  With DSB_LINEAR_PREFETCH_WEIGHT the
// first ring slots' weight tiles are requested before the wait on the
// previous kernel in the stream (programmatic dependent launch), so the
// weight stream starts while that kernel is finishing.
// Every wait is bounded; a wait that runs out sets DSB_FLAG_TIMEOUT, and the
// CTA still lets its copies land, frees its tensor memory and takes part in
// the cluster barriers.
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "peer.cuh"
#include "tma_umma.cuh"

namespace dsb {
namespace {

constexpr int kLnThreads = 128;             // 4 warps: one TMEM lane per thread
constexpr int kLnTok = 16;                  // tokens per tile (the MMA's N)
constexpr int kLnStages = 4;                // ring slots per CTA (two CTAs fit an SM)
constexpr int kLnL2Ahead = 4;               // k-blocks past the ring requested into L2
constexpr int kLnABytes = 128 * 64 * 2;     // weight box [128 rows][64 cols]
constexpr int kLnBBytes = kLnTok * 64 * 2;  // activation box [16 rows][64 cols]
constexpr int kLnMaxK = 1 << 16;

// kPeerF32: the fp32 sums go to every rank's peer exchange buffer (peer.cuh)
enum Epilogue : int { kPlain = 0, kResidual = 1, kSwiglu = 2, kPartialF32 = 3, kPeerF32 = 4 };

template <int RANKS> struct LnCfg {
  static constexpr int kTpr = kLnTok / RANKS;  // tokens each rank sums
  static constexpr int kBarOff = kLnStages * (kLnABytes + kLnBBytes);
  // full[stages], empty[stages], done, exchange, then the TMEM address word
  // 16-byte aligned: the partials arrive as 16-byte (or 8-byte) stores
  static constexpr int kXchOff = (kBarOff + 8 * (2 * kLnStages + 2) + 16 + 15) / 16 * 16;
  static constexpr int kSwOff = kXchOff + 4 * RANKS * 128 * kTpr;  // [kTpr][128] fp32 (SwiGLU)
  static constexpr size_t kSmem = 1024 + kSwOff + 4 * 128 * kTpr;
};

struct LnArgs {
  // features [0, split) -> out[t * ldo + f] (epilogue applied);
  // features [split, N) -> out2[t * ldo2 + f - split] and, when raw_k is
  // set, the raw caches (first kv_feats features K, the rest V).
  void *out, *out2;
  int64_t ldo, ldo2;
  int split;
  const void *residual;
  int64_t ldr;
  int mode;
  int prefetch;
  int prefetch_l2;  // with prefetch: the rest of the weight into L2 as well
  int packed;  // weight in the tile-packed layout (DSB_LINEAR_PACKED_WEIGHT)
  const void *wpacked;  // that weight's base (bulk-copied block by block)
  const int32_t *slots;
  const int64_t *positions;
  void *raw_k, *raw_v;
  int kv_feats, num_slots;
  int64_t max_len;
  int T, K, N;
  int32_t *err;
  // kPeerF32: base of every rank's exchange buffer as mapped here ([world]),
  // this rank, the buffers' token capacity and this rank's own epoch word
  const uint64_t *peers;
  int pworld, prank, ptmax;
  uint32_t *psync;
};

// Cluster size forced by the environment (0: chosen per launch):
// DSB_LINEAR_RANKS=1|2|4|8|16, or DSB_KV_PROJECTION_RANKS8=1 for 8.
int ranks_requested() {
  if (const char *v = std::getenv("DSB_LINEAR_RANKS")) {
    const int r = std::atoi(v);
    if (r == 1 || r == 2 || r == 4 || r == 8 || r == 16) return r;
  }
  const char *v = std::getenv("DSB_KV_PROJECTION_RANKS8");
  return v != nullptr && v[0] == '1' ? 8 : 0;
}

__device__ __forceinline__ float silu_f(float g) { return __fdiv_rn(g, 1.f + expf(-g)); }

template <typename T, int RANKS>
__global__ void __launch_bounds__(kLnThreads)
draft_linear_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
                    const LnArgs a) {
  using Cfg = LnCfg<RANKS>;
  constexpr int kTpr = Cfg::kTpr, S = kLnStages;
  extern __shared__ uint8_t ln_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(ln_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t s_a = smem_u32(smem), s_b = s_a + S * kLnABytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kBarOff);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * S, done = full0 + 16 * S;
  const uint32_t xbar = done + 8;  // the partials sent to this rank
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(bars + 2 * S + 2);
  float *xch = reinterpret_cast<float *>(smem + Cfg::kXchOff);
  float *sw = reinterpret_cast<float *>(smem + Cfg::kSwOff);
  __shared__ int s_abort, s_consumed, s_issued;
  const int tid = threadIdx.x, warp = tid >> 5;

  const int rank = (int)cluster_rank();
  const int f0 = blockIdx.y * 128, t0 = blockIdx.z * kLnTok;
  const int nkb_all = a.K / 64;
  const int per = (nkb_all + RANKS - 1) / RANKS;
  const int kb0 = rank * per;
  const int nkb = max(0, min(per, nkb_all - kb0));
  const int first = min(nkb, S);
  // weights are streamed once per step: evicted first, so the working cache
  // the draft attention re-reads keeps its L2 lines
  const uint64_t wpol = l2_evict_first();
  // Weight block of k-block kb into slot `dst`: row-major [N, K] by a 2-D
  // TMA box (x = 64 kb, y = f0, swizzled on the way in); tile-packed (the
  // block already in its swizzled shared-memory image, contiguous) by one
  // 1-D bulk copy of 16 KB.
  const uint8_t *wpacked = static_cast<const uint8_t *>(a.wpacked);
  auto load_w = [&](uint32_t dst, int kb, uint32_t bar) {
    if (a.packed)
      bulk_load(dst, wpacked + ((int64_t)blockIdx.y * nkb_all + kb) * kLnABytes, kLnABytes, bar,
                wpol);
    else
      tma_load_2d_hint(dst, &tw, kb * 64, f0, bar, wpol);
  };

  // No activations yet: descriptor prefetch, barriers, tensor memory and
  // (when allowed) the first weight tiles overlap the previous kernel.
  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tx)) : "memory");
    for (int b = 0; b <= 2 * S + 1; ++b) mbar_init(full0 + 8 * b);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
    s_consumed = 0;
    s_issued = 0;
    if (a.prefetch) {
      for (int kb = 0; kb < first; ++kb) {
        mbar_expect_tx(full0 + 8 * kb, kLnABytes + kLnBBytes);
        load_w(s_a + kb * kLnABytes, kb0 + kb, full0 + 8 * kb);
      }
      // the next kLnL2Ahead of this rank's weight blocks into L2, so that
      // HBM keeps streaming while the previous kernel finishes and the
      // ring's next loads hit L2 (a bounded run: the whole weight measured
      // slower and holds more of L2)
      for (int kb = first; kb < min(nkb, first + kLnL2Ahead) && a.prefetch_l2; ++kb) {
        if (a.packed)
          bulk_prefetch_l2_hint(wpacked + ((int64_t)blockIdx.y * nkb_all + kb0 + kb) * kLnABytes,
                                kLnABytes, wpol);
        else
          tma_prefetch_2d_hint(&tw, (kb0 + kb) * 64, f0, wpol);
      }
    }
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

  // The epilogue's global operands (written by earlier kernels, valid once
  // the wait above has returned) are loaded now, so their latency passes
  // while the weights stream: this thread's residual values, or the slot and
  // position of each token it stores.
  const int g = f0 + tid;  // output feature of this thread in the epilogue
  const uint32_t pepoch = a.mode == kPeerF32 ? *reinterpret_cast<volatile const uint32_t *>(a.psync) : 0u;
  float res[kTpr];
  int32_t tslot[kTpr];
  int64_t tpos[kTpr];
#pragma unroll
  for (int j = 0; j < kTpr; ++j) {
    const int t = t0 + kTpr * rank + j;
    res[j] = 0.f;
    tslot[j] = -1;
    tpos[j] = 0;
    if (t >= a.T) continue;
    if (a.mode == kResidual && g < a.split)
      res[j] = Elem<T>::to_f(static_cast<const T *>(a.residual)[(int64_t)t * a.ldr + g]);
    if (a.raw_k != nullptr && g >= a.split) {
      tslot[j] = a.slots[t];
      tpos[j] = a.positions[t];
    }
  }

  if (tid == 32) {
    // Producer: fill slot kb % S once the products of its previous fill
    // (k-block kb - S) have completed.
    int kb = 0;
    for (; kb < nkb; ++kb) {
      const int s = kb % S;
      if (kb >= S) {
        if (!mbar_wait(empty0 + 8 * s, (uint32_t)(kb / S - 1) & 1u) ||
            *reinterpret_cast<volatile int *>(&s_abort))
          break;
      }
      if (!(a.prefetch && kb < first)) {
        mbar_expect_tx(full0 + 8 * s, kLnABytes + kLnBBytes);
        load_w(s_a + s * kLnABytes, kb0 + kb, full0 + 8 * s);
      }
      tma_load_2d(s_b + s * kLnBBytes, &tx, (kb0 + kb) * 64, t0, full0 + 8 * s);
    }
    if (kb < nkb) atomicExch(&s_abort, 1);
    s_issued = kb;
  } else if (tid == 0) {
    // Products: one k-block (4 MMAs of K = 16) per filled slot; each slot is
    // released to the producer by a commit once its products are done.
    const uint32_t idesc = umma_idesc<T, kLnTok>(false);
    int kb = 0;
    for (; kb < nkb; ++kb) {
      const int s = kb % S;
      if (!mbar_wait(full0 + 8 * s, (uint32_t)(kb / S) & 1u)) break;
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma(tmem, umma_desc(s_a + s * kLnABytes + ks * 32, 16, 1024),
             umma_desc(s_b + s * kLnBBytes + ks * 32, 16, 1024), idesc, kb > 0 || ks > 0);
      if (kb + S < nkb) umma_commit(empty0 + 8 * s);
    }
    if (kb < nkb) atomicExch(&s_abort, 1);
    s_consumed = kb;
    if (nkb > 0) umma_commit(done);  // arrives once every issued product is done
  }
  __syncthreads();
  if (tid == 32 && s_abort) {  // a wait ran out: let the requested copies land
    flag_error(a.err, DSB_FLAG_TIMEOUT);
    for (int k2 = s_consumed; k2 < s_issued; ++k2)
      mbar_wait(full0 + 8 * (k2 % S), (uint32_t)(k2 / S) & 1u);
  }
  __syncthreads();

  // This rank's partial: thread = feature row (TMEM lane), 16 token columns.
  float acc[kLnTok];
#pragma unroll
  for (int j = 0; j < kLnTok; ++j) acc[j] = 0.f;
  if (nkb > 0) {
    const bool got = mbar_wait(done, 0);
    if (__syncthreads_and(got) && !s_abort) {
      tc_fence_after();
      tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16), acc);
    } else {
      // `done` is committed after the last product that was issued (a wait
      // that ran out above stops the issuing, it never leaves a product
      // half-issued), so it arrives once those few MMAs finish; wait for it
      // once more (bounded) so no product still writes the tensor memory
      // freed below.  The partial stays zero and the launch is flagged.
      if (tid == 0) {
        flag_error(a.err, DSB_FLAG_TIMEOUT);
        if (!got) mbar_wait(done, 0);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 32;" ::"r"(tmem) : "memory");

  // Rank q sums tokens q * kTpr .. q * kTpr + kTpr - 1 over the ranks: send
  // them there, as asynchronous 16-byte stores where kTpr allows (the
  // exchange costs per transaction) that complete on the receiver's `xbar`.
  // Each rank then waits only for the bytes addressed to it (thread 0 arms
  // the barrier with their count; stores that land first are counted all
  // the same), and leaves only once all of them have landed, so no rank
  // exits while a peer still writes into its shared memory.
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");  // every rank is running
  if (tid == 0) mbar_expect_tx(xbar, (uint32_t)(RANKS * 128 * kTpr * 4));
  const uint32_t x0 = smem_u32(xch);
#pragma unroll
  for (int q = 0; q < RANKS; ++q) {
    const uint32_t remote = cluster_map(x0, (uint32_t)q) + 4u * (uint32_t)((rank * 128 + tid) * kTpr);
    const uint32_t rbar = cluster_map(xbar, (uint32_t)q);
    if constexpr (kTpr % 4 == 0) {
#pragma unroll
      for (int j = 0; j < kTpr; j += 4)
        st_async(remote + 4u * j, make_float4(acc[q * kTpr + j], acc[q * kTpr + j + 1],
                                              acc[q * kTpr + j + 2], acc[q * kTpr + j + 3]),
                 rbar);
    } else if constexpr (kTpr == 2) {
      st_async(remote, make_float2(acc[q * 2], acc[q * 2 + 1]), rbar);
    } else {
      st_async(remote, acc[q], rbar);
    }
  }
  if (!mbar_wait_cluster(xbar, 0) && tid == 0) flag_error(a.err, DSB_FLAG_TIMEOUT);

  // (read as the 16- or 8-byte vectors they arrived in; the sum over the
  // ranks runs in rank order either way)
  float v[kTpr];
#pragma unroll
  for (int j = 0; j < kTpr; ++j) v[j] = 0.f;
#pragma unroll
  for (int r = 0; r < RANKS; ++r) {
    const float *row = xch + (r * 128 + tid) * kTpr;
    if constexpr (kTpr % 4 == 0) {
#pragma unroll
      for (int j = 0; j < kTpr; j += 4) {
        const float4 x4 = *reinterpret_cast<const float4 *>(row + j);
        v[j] += x4.x;
        v[j + 1] += x4.y;
        v[j + 2] += x4.z;
        v[j + 3] += x4.w;
      }
    } else if constexpr (kTpr == 2) {
      const float2 x2 = *reinterpret_cast<const float2 *>(row);
      v[0] += x2.x;
      v[1] += x2.y;
    } else {
      v[0] += row[0];
    }
  }

  if (a.mode == kSwiglu) {
    // Tile rows 0..63 are gate rows and 64..127 the up rows of output
    // features f0 / 2 .. f0 / 2 + 63: both rounded to the storage type, as a
    // gate_up GEMM output is, then round(round(silu(gate)) * up) as vLLM's
    // SiluAndMul computes it.
#pragma unroll
    for (int j = 0; j < kTpr; ++j) sw[j * 128 + tid] = Elem<T>::to_f(Elem<T>::from_f(v[j]));
    __syncthreads();
    // 64 output features x kTpr tokens over all 128 threads
    T *out = static_cast<T *>(a.out);
    const int f = tid & 63;
    for (int j = tid >> 6; j < kTpr; j += 2) {
      const int t = t0 + kTpr * rank + j;
      if (t >= a.T) continue;
      const float gt = sw[j * 128 + f], u = sw[j * 128 + f + 64];
      const float sg = Elem<T>::to_f(Elem<T>::from_f(silu_f(gt)));  // SiluAndMul rounds silu
      out[(int64_t)t * a.ldo + f0 / 2 + f] = Elem<T>::from_f(__fmul_rn(sg, u));
    }
    return;
  }

  if (a.mode == kPeerF32) {
    // Fused all-reduce: this rank's fp32 sums into its slot of every rank's
    // buffer (peer stores over NVLink, own buffer included), each with the
    // call's tag in the same 8-byte store, so the readers need no flag.
    const uint32_t tag = pepoch + 1u;
    const int64_t slot0 = (int64_t)((int)(pepoch & 1u) * a.pworld + a.prank) * a.ptmax;
#pragma unroll
    for (int j = 0; j < kTpr; ++j) {
      const int t = t0 + kTpr * rank + j;
      if (t >= a.T) continue;
      for (int q = 0; q < a.pworld; ++q)
        st_tagged(reinterpret_cast<uint8_t *>(a.peers[q]) + ((slot0 + t) * a.N + g) * 8, v[j], tag);
    }
    return;
  }

  T *raw_k = static_cast<T *>(a.raw_k), *raw_v = static_cast<T *>(a.raw_v);
#pragma unroll
  for (int j = 0; j < kTpr; ++j) {
    const int t = t0 + kTpr * rank + j;
    if (t >= a.T) continue;
    if (g < a.split) {
      if (a.mode == kPartialF32) {  // the fp32 sums themselves (no rounding)
        static_cast<float *>(a.out)[(int64_t)t * a.ldo + g] = v[j];
        continue;
      }
      float y = v[j];
      if (a.mode == kResidual) y = __fadd_rn(y, res[j]);
      static_cast<T *>(a.out)[(int64_t)t * a.ldo + g] = Elem<T>::from_f(y);
      continue;
    }
    const T y = Elem<T>::from_f(v[j]);
    const int gk = g - a.split;
    if (a.out2 != nullptr) static_cast<T *>(a.out2)[(int64_t)t * a.ldo2 + gk] = y;
    if (raw_k == nullptr) continue;
    const int slot = tslot[j];
    if (slot < 0) continue;  // padding row: no cache row
    const int64_t pos = tpos[j];
    if (slot >= a.num_slots || pos < 0 || pos >= a.max_len) {
      if (tid == 0) flag_error(a.err, slot >= a.num_slots ? DSB_FLAG_SLOT : DSB_FLAG_POSITION);
      continue;
    }
    const int64_t row = ((int64_t)slot * a.max_len + pos) * a.kv_feats;
    if (gk < a.kv_feats) raw_k[row + gk] = y;
    else raw_v[row + gk - a.kv_feats] = y;
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

template <typename T, int RANKS> const void *kernel_of() {
  return (const void *)draft_linear_kernel<T, RANKS>;
}

// Resident CTAs of the RANKS-wide kernel (0 if no such cluster can be
// scheduled); enables the non-portable size 16 on first use.
template <typename T, int RANKS> int64_t resident_slots() {
  const void *kern = kernel_of<T, RANKS>();
  constexpr size_t smem = LnCfg<RANKS>::kSmem;
  if (RANKS > 8 && !allow_cluster16(kern)) return 0;
  if (ensure_smem(kern, smem) != DSB_OK) {
    (void)cudaGetLastError();
    return 0;
  }
  return (int64_t)max_active_clusters(kern, RANKS, kLnThreads, smem) * RANKS;
}

template <typename T, int RANKS>
int launch_ranks(const CUtensorMap &tw, const CUtensorMap &tx, const LnArgs &a, cudaStream_t st) {
  auto kern = draft_linear_kernel<T, RANKS>;
  constexpr size_t smem = LnCfg<RANKS>::kSmem;
  const dim3 grid(RANKS, a.N / 128, (a.T + kLnTok - 1) / kLnTok);
  launch_kernel_cluster(kern, grid, dim3(kLnThreads), smem, st, RANKS, tw, tx, a);
  return check_launch("draft_linear_kernel");
}

// The K split: the widest cluster (16, 8, 4, 2, 1 CTAs) whose grid holds at
// most 4/3 CTAs per SM and leaves no rank without k-blocks.  Measured on
// B200 for 16 tokens (qkv 5120 x 4096, o 2048 x 4096, gate_up 12288 x 2048,
// down 2048 x 6144), this is the fastest size of every shape: wider clusters
// add CTAs whose fixed set-up and exchange cost more than their shorter
// k-runs save, narrower ones leave SMs idle.
template <typename T> int pick_ranks(const LnArgs &a) {
  const int forced = ranks_requested();
  const int64_t tiles = (int64_t)(a.N / 128) * ((a.T + kLnTok - 1) / kLnTok);
  const int nkb = a.K / 64;
  const int ranks[5] = {16, 8, 4, 2, 1};
  const int64_t sms = sm_count();
  int pick = 0;
  for (int i = 0; i < 5 && !pick; ++i)
    if ((forced ? ranks[i] == forced : 3 * tiles * ranks[i] <= 4 * sms && ranks[i] <= nkb))
      pick = ranks[i];
  if (!pick) pick = 1;
  const int64_t slots = pick == 16 ? resident_slots<T, 16>() : pick == 8 ? resident_slots<T, 8>()
                        : pick == 4 ? resident_slots<T, 4>() : pick == 2 ? resident_slots<T, 2>()
                                                             : resident_slots<T, 1>();
  if (slots > 0) return pick;
  return resident_slots<T, 8>() > 0 ? 8 : resident_slots<T, 1>() > 0 ? 1 : 0;
}

template <typename T>
int launch_linear(const void *x, const void *weight, const LnArgs &a, int dtype, cudaStream_t st) {
  CUtensorMap tw, tx;
  // packed weights are bulk-copied (the map is unused; encoded over the
  // first block so the launch argument stays valid)
  const bool wmap = a.packed ? encode_kv_map(&tw, weight, 128, 64, dtype, 128)
                             : encode_kv_map(&tw, weight, a.N, a.K, dtype, 128);
  if (!wmap ||
      !encode_kv_map(&tx, x, a.T, a.K, dtype, kLnTok))
    return fail(DSB_ERR_UNSUPPORTED, "no tensor map for the weight or activation rows");
  switch (pick_ranks<T>(a)) {
    case 16: return launch_ranks<T, 16>(tw, tx, a, st);
    case 8: return launch_ranks<T, 8>(tw, tx, a, st);
    case 4: return launch_ranks<T, 4>(tw, tx, a, st);
    case 2: return launch_ranks<T, 2>(tw, tx, a, st);
    case 1: return launch_ranks<T, 1>(tw, tx, a, st);
    default: return fail(DSB_ERR_UNSUPPORTED, "no linear-layer CTA fits on this device");
  }
}

int check_common(const void *x, int32_t tokens, int32_t in_features, const void *weight,
                 int64_t out_features, int32_t dtype) {
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_INVALID, "activations, weight and outputs must be BF16 or FP16");
  if (in_features <= 0 || in_features % 64 || in_features > kLnMaxK)
    return fail(DSB_ERR_UNSUPPORTED, "in_features must be a multiple of 64 and at most 65536");
  if (out_features <= 0 || out_features % 128)
    return fail(DSB_ERR_UNSUPPORTED, "the weight's row count must be a multiple of 128");
  if ((tokens + kLnTok - 1) / kLnTok > 65535 || out_features / 128 > 65535 ||
      out_features * (in_features / 64) > INT_MAX)
    return fail(DSB_ERR_UNSUPPORTED, "grid too large");
  if (!x || !weight) return fail(DSB_ERR_INVALID, "null pointer argument");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(weight) % 16)
    return fail(DSB_ERR_UNSUPPORTED, "activation rows and weight must be 16-byte aligned");
  return DSB_OK;
}

int dispatch(const void *x, const void *weight, const LnArgs &a, int32_t dtype, void *stream) {
  cudaStream_t st = as_stream(stream);
  return dtype == DSB_BF16 ? launch_linear<__nv_bfloat16>(x, weight, a, dtype, st)
                           : launch_linear<__half>(x, weight, a, dtype, st);
}

// out[m][kb][r][...] = weight[128 m + r][64 kb .. 64 kb + 63] with the
// 16-byte pieces of row r in the 128-byte-swizzle order (piece p stored at
// p ^ (r % 8)), i.e. each 16 KB block is byte for byte the shared-memory
// image a 2-D TMA load with CU_TENSOR_MAP_SWIZZLE_128B would produce, so one
// 1-D bulk copy stages it.  One thread per 16-byte piece.
// Launched without programmatic dependent launch and never releasing its
// dependents early: the next kernel in the stream may be a linear that
// requests this very weight before its own dependency wait, so it must not
// start before these writes are complete.
template <typename T>
__global__ void pack_weight_kernel(const T *__restrict__ w, int64_t rows, int cols,
                                   T *__restrict__ out) {
  const int64_t pieces = rows * (cols / 8);
  const int nkb = cols / 64;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < pieces;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t blk = i / (128 * 8);  // m * nkb + kb
    const int rem = (int)(i % (128 * 8)), r = rem / 8, p = rem % 8;
    const int64_t m = blk / nkb, kb = blk % nkb;
    const int64_t src = (m * 128 + r) * cols + kb * 64 + p * 8;
    const int64_t dst = (blk * 128 + r) * 64 + (int64_t)(p ^ (r & 7)) * 8;
    *reinterpret_cast<uint4 *>(out + dst) = *reinterpret_cast<const uint4 *>(w + src);
  }
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" int dsb_qkv_projection_write_raw(
    const void *hidden, int32_t tokens, int32_t hidden_size, const void *weight,
    int32_t q_features, int32_t num_kv_heads, int32_t head_dim, const int32_t *slots,
    const int64_t *positions, void *raw_key, void *raw_value, int32_t num_slots,
    int64_t max_model_len, int32_t dtype, void *q_out, void *kv_out, int32_t flags,
    int32_t *error_flag, void *stream) {
  if (tokens < 0) return fail(DSB_ERR_INVALID, "negative token count");
  if (tokens == 0) return DSB_OK;
  if (num_kv_heads <= 0 || head_dim <= 0 || num_slots <= 0 || max_model_len <= 0 || q_features < 0)
    return fail(DSB_ERR_INVALID,
                "kv heads, head_dim, slots and max_model_len must be positive, q_features >= 0");
  const int64_t kv_feats = (int64_t)num_kv_heads * head_dim;
  if (kv_feats % 128 || q_features % 128)
    return fail(DSB_ERR_UNSUPPORTED,
                "num_kv_heads * head_dim and q_features must be multiples of 128");
  if (int e = check_common(hidden, tokens, hidden_size, weight, q_features + 2 * kv_feats, dtype))
    return e;
  if (!slots || !positions || !raw_key || !raw_value || (q_features > 0 && !q_out))
    return fail(DSB_ERR_INVALID, "null pointer argument");
  LnArgs a{};
  a.out = q_out;
  a.ldo = q_features;
  a.out2 = kv_out;
  a.ldo2 = 2 * kv_feats;
  a.split = q_features;
  a.mode = kPlain;
  a.prefetch = (flags & DSB_LINEAR_PREFETCH_WEIGHT) != 0;
  a.prefetch_l2 = a.prefetch && (flags & DSB_LINEAR_PREFETCH_L2) != 0;
  a.packed = (flags & DSB_LINEAR_PACKED_WEIGHT) != 0;
  a.wpacked = weight;
  a.slots = slots;
  a.positions = positions;
  a.raw_k = raw_key;
  a.raw_v = raw_value;
  a.kv_feats = (int)kv_feats;
  a.num_slots = num_slots;
  a.max_len = max_model_len;
  a.T = tokens;
  a.K = hidden_size;
  a.N = (int)(q_features + 2 * kv_feats);
  a.err = error_flag;
  return dispatch(hidden, weight, a, dtype, stream);
}

extern "C" int dsb_kv_projection_write_raw(const void *hidden, int32_t tokens, int32_t hidden_size,
                                           const void *weight, int32_t num_kv_heads,
                                           int32_t head_dim, const int32_t *slots,
                                           const int64_t *positions, void *raw_key,
                                           void *raw_value, int32_t num_slots,
                                           int64_t max_model_len, int32_t dtype, void *out,
                                           int32_t *error_flag, void *stream) {
  return dsb_qkv_projection_write_raw(hidden, tokens, hidden_size, weight, 0, num_kv_heads,
                                      head_dim, slots, positions, raw_key, raw_value, num_slots,
                                      max_model_len, dtype, nullptr, out, 0, error_flag, stream);
}

extern "C" int dsb_draft_linear(const void *x, int32_t tokens, int32_t in_features,
                                const void *weight, int32_t weight_rows, int32_t epilogue,
                                const void *residual, int64_t residual_row_stride, void *out,
                                int64_t out_row_stride, int32_t dtype, int32_t flags,
                                int32_t *error_flag, void *stream) {
  if (tokens < 0) return fail(DSB_ERR_INVALID, "negative token count");
  if (tokens == 0) return DSB_OK;
  if (epilogue != DSB_LINEAR_PLAIN && epilogue != DSB_LINEAR_RESIDUAL &&
      epilogue != DSB_LINEAR_SWIGLU && epilogue != DSB_LINEAR_PARTIAL_F32)
    return fail(DSB_ERR_INVALID, "unknown epilogue");
  if (int e = check_common(x, tokens, in_features, weight, weight_rows, dtype)) return e;
  const int64_t out_cols = epilogue == DSB_LINEAR_SWIGLU ? weight_rows / 2 : weight_rows;
  if (!out || out_row_stride < out_cols)
    return fail(DSB_ERR_INVALID, "null output or output row stride shorter than its row");
  if (epilogue == DSB_LINEAR_RESIDUAL && (!residual || residual_row_stride < out_cols))
    return fail(DSB_ERR_INVALID, "null residual or residual row stride shorter than its row");
  LnArgs a{};
  a.out = out;
  a.ldo = out_row_stride;
  a.split = weight_rows;  // every feature goes to `out`
  a.residual = residual;
  a.ldr = residual_row_stride;
  a.mode = epilogue == DSB_LINEAR_PLAIN      ? kPlain
           : epilogue == DSB_LINEAR_RESIDUAL ? kResidual
           : epilogue == DSB_LINEAR_SWIGLU   ? kSwiglu
                                             : kPartialF32;
  a.prefetch = (flags & DSB_LINEAR_PREFETCH_WEIGHT) != 0;
  a.prefetch_l2 = a.prefetch && (flags & DSB_LINEAR_PREFETCH_L2) != 0;
  a.packed = (flags & DSB_LINEAR_PACKED_WEIGHT) != 0;
  a.wpacked = weight;
  a.T = tokens;
  a.K = in_features;
  a.N = weight_rows;
  a.err = error_flag;
  return dispatch(x, weight, a, dtype, stream);
}

extern "C" int dsb_draft_linear_peer(const void *x, int32_t tokens, int32_t in_features,
                                     const void *weight, int32_t weight_rows,
                                     const uint64_t *peer_bases, int32_t world, int32_t rank,
                                     int32_t tokens_max, void *own_base, int32_t dtype,
                                     int32_t flags, int32_t *error_flag, void *stream) {
  if (tokens < 0) return fail(DSB_ERR_INVALID, "negative token count");
  if (world < 1 || world > kPeerMaxWorld || rank < 0 || rank >= world)
    return fail(DSB_ERR_INVALID, "world must be in [1, 8] and rank in [0, world)");
  if (tokens > tokens_max) return fail(DSB_ERR_INVALID, "more tokens than the exchange buffer holds");
  if (!peer_bases || !own_base) return fail(DSB_ERR_INVALID, "null pointer argument");
  if (tokens == 0) return DSB_OK;
  if (int e = check_common(x, tokens, in_features, weight, weight_rows, dtype)) return e;
  const PeerLayout L(world, tokens_max, weight_rows);
  LnArgs a{};
  a.split = weight_rows;
  a.mode = kPeerF32;
  a.prefetch = (flags & DSB_LINEAR_PREFETCH_WEIGHT) != 0;
  a.prefetch_l2 = a.prefetch && (flags & DSB_LINEAR_PREFETCH_L2) != 0;
  a.packed = (flags & DSB_LINEAR_PACKED_WEIGHT) != 0;
  a.wpacked = weight;
  a.T = tokens;
  a.K = in_features;
  a.N = weight_rows;
  a.err = error_flag;
  a.peers = peer_bases;
  a.pworld = world;
  a.prank = rank;
  a.ptmax = tokens_max;
  a.psync = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(own_base) + L.sync_off);
  return dispatch(x, weight, a, dtype, stream);
}

extern "C" int dsb_pack_linear_weight(const void *weight, int64_t rows, int32_t cols,
                                      int32_t dtype, void *out, void *stream) {
  if (dtype != DSB_BF16 && dtype != DSB_F16)
    return fail(DSB_ERR_INVALID, "the weight must be BF16 or FP16");
  if (rows <= 0 || rows % 128 || cols <= 0 || cols % 64)
    return fail(DSB_ERR_UNSUPPORTED, "rows must be a multiple of 128 and cols of 64");
  if (!weight || !out || weight == out) return fail(DSB_ERR_INVALID, "null or aliased buffers");
  if (reinterpret_cast<uintptr_t>(weight) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail(DSB_ERR_UNSUPPORTED, "weight and out must be 16-byte aligned");
  const int64_t pieces = rows * (cols / 8);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((pieces + threads - 1) / threads, 8 * sm_count());
  cudaStream_t st = as_stream(stream);
  if (dtype == DSB_BF16)
    pack_weight_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, st>>>(
        static_cast<const __nv_bfloat16 *>(weight), rows, (int)cols,
        static_cast<__nv_bfloat16 *>(out));
  else
    pack_weight_kernel<__half><<<(unsigned)blocks, threads, 0, st>>>(
        static_cast<const __half *>(weight), rows, (int)cols, static_cast<__half *>(out));
  return check_launch("pack_weight_kernel");
}
