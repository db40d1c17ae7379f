// Buffers of the fused row-split linear + all-reduce (layout in peer.cuh):
// allocation and the CUDA IPC handles that map one rank's buffer into the
// other ranks' processes.  The reduction itself is the epilogue of
// draft_linear_kernel (dsb_draft_linear_peer) and the peer variant of the
// add + RMSNorm kernel (dsb_peer_add_rms_norm).  Reference: the tensor-parallel
// all-reduce of vLLM's RowParallelLinear in the Eagle3 draft layer
// (diffspec/proposer.py:97-119 drafts through it).
#include <algorithm>
#include <climits>
#include <cstring>

#include "common.cuh"
#include "peer.cuh"

using namespace dsb;

extern "C" int64_t dsb_peer_buffer_bytes(int32_t world, int32_t tokens_max, int32_t features) {
  if (world < 1 || world > kPeerMaxWorld || tokens_max < 1 || features < 1) return -1;
  return PeerLayout(world, tokens_max, features).total;
}

extern "C" int dsb_peer_buffer_create(int32_t world, int32_t tokens_max, int32_t features,
                                      void **base) {
  if (!base) return fail(DSB_ERR_INVALID, "null pointer argument");
  *base = nullptr;
  if (world < 1 || world > kPeerMaxWorld || tokens_max < 1 || tokens_max > 65535 || features < 8 ||
      features % 8)
    return fail(DSB_ERR_INVALID,
                "world must be in [1, 8], tokens_max in [1, 65535] and features a multiple of 8");
  const PeerLayout L(world, tokens_max, features);
  void *p = nullptr;
  if (cudaMalloc(&p, (size_t)L.total) != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(DSB_ERR_CUDA, "cudaMalloc of the peer exchange buffer failed");
  }
  if (cudaMemset(p, 0, (size_t)L.total) != cudaSuccess) {
    (void)cudaGetLastError();
    cudaFree(p);
    return fail(DSB_ERR_CUDA, "cudaMemset of the peer exchange buffer failed");
  }
  *base = p;
  return DSB_OK;
}

extern "C" int dsb_peer_buffer_destroy(void *base) {
  if (!base) return DSB_OK;
  if (cudaFree(base) != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(DSB_ERR_CUDA, "cudaFree of the peer exchange buffer failed");
  }
  return DSB_OK;
}

extern "C" int dsb_ipc_handle(void *base, void *handle) {
  if (!base || !handle) return fail(DSB_ERR_INVALID, "null pointer argument");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, base) != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(DSB_ERR_CUDA, "cudaIpcGetMemHandle failed");
  }
  static_assert(sizeof(h) == DSB_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return DSB_OK;
}

extern "C" int dsb_ipc_open(const void *handle, void **base) {
  if (!handle || !base) return fail(DSB_ERR_INVALID, "null pointer argument");
  *base = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    (void)cudaGetLastError();
    *base = nullptr;
    return fail(DSB_ERR_CUDA, "cudaIpcOpenMemHandle failed (no peer access to that GPU?)");
  }
  return DSB_OK;
}

extern "C" int dsb_ipc_close(void *base) {
  if (!base) return DSB_OK;
  if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(DSB_ERR_CUDA, "cudaIpcCloseMemHandle failed");
  }
  return DSB_OK;
}

// All-gather over the same buffers (one "token" row of count_max features):
// each rank stores its `count` floats, tagged, into its slot of every rank's
// buffer; each rank then unpacks the world slots of its own buffer into a
// plain [world][count] array once their tags show the call's values arrived.
// Two launches (send, then receive), so ranks emulated on one GPU can run
// every send before any receive.
namespace dsb {
namespace {

__global__ void peer_send_kernel(const float *__restrict__ src, int64_t count,
                                 const uint64_t *__restrict__ peers, int world, int rank,
                                 int64_t count_max, const uint32_t *sync) {
  pdl_begin();
  const uint32_t epoch = *reinterpret_cast<volatile const uint32_t *>(sync);
  const int64_t slot = (int64_t)((int)(epoch & 1u) * world + rank) * count_max;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = src[i];
    for (int q = 0; q < world; ++q)
      st_tagged(reinterpret_cast<uint8_t *>(peers[q]) + (slot + i) * 8, v, epoch + 1u);
  }
}

__global__ void peer_recv_kernel(const uint8_t *__restrict__ own, int world, int64_t count,
                                 int64_t count_max, float *__restrict__ out, uint32_t *sync,
                                 int32_t *err) {
  pdl_begin();
  const uint32_t epoch = *reinterpret_cast<volatile const uint32_t *>(sync);
  const int64_t groups = count / 8, base = (int64_t)(epoch & 1u) * world * count_max;
  bool late = false;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < world * groups;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t q = k / groups, i = (k % groups) * 8;
    float v[8];
    late |= !ld_tagged8(own + (base + q * count_max + i) * 8, epoch + 1u, v, !late);
    float4 *o = reinterpret_cast<float4 *>(out + q * count + i);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
  if (late) flag_error(err, DSB_FLAG_TIMEOUT);
  // every CTA has read the call's epoch and words: the last one advances it
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(sync + 1, 1u) == gridDim.x - 1) {
      sync[1] = 0;
      sync[0] = epoch + 1u;
    }
  }
}

int gather_grid(int64_t items) {
  const int64_t ctas = (items + 255) / 256;
  return (int)std::min<int64_t>(std::max<int64_t>(ctas, 1), 4 * (int64_t)sm_count());
}

}  // namespace
}  // namespace dsb

extern "C" int dsb_peer_all_gather_send(const float *src, int64_t count,
                                        const uint64_t *peer_bases, int32_t world, int32_t rank,
                                        int64_t count_max, void *own_base, void *stream) {
  if (world < 1 || world > kPeerMaxWorld || rank < 0 || rank >= world)
    return fail(DSB_ERR_INVALID, "world must be in [1, 8] and rank in [0, world)");
  if (count < 0 || count > count_max || count % 8 || count_max % 8 || count_max > INT32_MAX)
    return fail(DSB_ERR_INVALID,
                "count must be a multiple of 8 within the buffer's row (count_max, a multiple of 8)");
  if (!src || !peer_bases || !own_base) return fail(DSB_ERR_INVALID, "null pointer argument");
  if (count == 0) return DSB_OK;
  const PeerLayout L(world, 1, (int)count_max);
  const uint32_t *sync =
      reinterpret_cast<const uint32_t *>(static_cast<uint8_t *>(own_base) + L.sync_off);
  launch_kernel(peer_send_kernel, dim3(gather_grid(count)), dim3(256), 0, as_stream(stream), src,
                count, peer_bases, (int)world, (int)rank, count_max, sync);
  return check_launch("peer_send_kernel");
}

extern "C" int dsb_peer_all_gather_recv(void *own_base, int32_t world, int64_t count,
                                        int64_t count_max, float *out, int32_t *error_flag,
                                        void *stream) {
  if (world < 1 || world > kPeerMaxWorld)
    return fail(DSB_ERR_INVALID, "world must be in [1, 8]");
  if (count < 0 || count > count_max || count % 8 || count_max % 8 || count_max > INT32_MAX)
    return fail(DSB_ERR_INVALID,
                "count must be a multiple of 8 within the buffer's row (count_max, a multiple of 8)");
  if (!own_base || !out) return fail(DSB_ERR_INVALID, "null pointer argument");
  if (reinterpret_cast<uintptr_t>(out) % 16) return fail(DSB_ERR_UNSUPPORTED, "out must be 16-byte aligned");
  if (count == 0) return DSB_OK;
  const PeerLayout L(world, 1, (int)count_max);
  uint8_t *b = static_cast<uint8_t *>(own_base);
  launch_kernel(peer_recv_kernel, dim3(gather_grid(world * count / 8)), dim3(256), 0,
                as_stream(stream), (const uint8_t *)b, (int)world, count, count_max, out,
                reinterpret_cast<uint32_t *>(b + L.sync_off), error_flag);
  return check_launch("peer_recv_kernel");
}
