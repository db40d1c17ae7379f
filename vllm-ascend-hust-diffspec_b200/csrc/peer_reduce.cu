// Buffers of the fused row-split linear + all-reduce (layout in peer.cuh):
// allocation and the CUDA IPC handles that map one rank's buffer into the
// other ranks' processes.  The reduction itself is the epilogue of
// draft_linear_kernel (dsb_draft_linear_peer) and the peer variant of the
// add + RMSNorm kernel (dsb_peer_add_rms_norm).  Reference: the tensor-parallel
// all-reduce of vLLM's RowParallelLinear in the Eagle3 draft layer
// (diffspec/proposer.py:97-119 drafts through it).
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
