// Status reporting shared by every C-ABI entry point.
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "common.cuh"

namespace dsb {

static thread_local std::string g_last_error;

void set_error(const std::string &msg) { g_last_error = msg; }

int fail(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(DSB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return DSB_OK;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

int ensure_smem(const void *kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return DSB_OK;
  static std::mutex mu;
  static std::map<std::pair<int, const void *>, size_t> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(DSB_ERR_CUDA, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(dev, kernel);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return DSB_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess)
    return fail(DSB_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  done[key] = bytes;
  return DSB_OK;
}

}  // namespace dsb

extern "C" const char *dsb_last_error(void) { return dsb::g_last_error.c_str(); }

extern "C" int dsb_abi_version(void) { return 1; }
