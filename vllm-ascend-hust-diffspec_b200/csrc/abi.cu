// Status reporting shared by every C-ABI entry point.
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
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

int resident_ctas(const void *kernel, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void *, int, size_t>, int> known;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return sm_count();
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(dev, kernel, threads, smem);
  auto it = known.find(key);
  if (it != known.end()) return it->second;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess ||
      per_sm <= 0) {
    (void)cudaGetLastError();
    per_sm = 1;
  }
  return known[key] = per_sm * sm_count();
}

int max_active_clusters(const void *kernel, int cluster_x, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void *, int, size_t>, int> known;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(dev, kernel, cluster_x, smem);
  auto it = known.find(key);
  if (it != known.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster_x, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();  // a refused query is an answer, not an error
    n = 0;
  }
  known[key] = n;
  return n;
}

}  // namespace dsb

extern "C" const char *dsb_last_error(void) { return dsb::g_last_error.c_str(); }

extern "C" int dsb_abi_version(void) { return 2; }
