// Cached device facts for the launch paths (see launch_cache.h).
#include "launch_cache.h"

#include <map>
#include <mutex>
#include <tuple>

namespace attnres {

namespace {

constexpr int kMaxDevices = 64;

struct DeviceFacts {
  bool known = false;
  int sm_count = 0;
  int smem_optin = 0;
};

std::mutex g_mu;
DeviceFacts g_dev[kMaxDevices];
std::map<std::pair<int, const void*>, int> g_smem;                            // (device, fn) -> bytes set
std::map<std::tuple<int, const void*, int, size_t>, int> g_occupancy;         // -> blocks per SM

cudaError_t facts(DeviceFacts** out, int* dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  *dev_out = dev;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceFacts& f = g_dev[dev];
  if (!f.known) {
    if ((e = cudaDeviceGetAttribute(&f.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&f.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
      return e;
    f.known = true;
  }
  *out = &f;
  return cudaSuccess;
}

}  // namespace

cudaError_t cached_sm_count(int* n) {
  DeviceFacts* f = nullptr;
  int dev = 0;
  const cudaError_t e = facts(&f, &dev);
  if (e == cudaSuccess) *n = f->sm_count;
  return e;
}

cudaError_t cached_smem_optin(int* bytes) {
  DeviceFacts* f = nullptr;
  int dev = 0;
  const cudaError_t e = facts(&f, &dev);
  if (e == cudaSuccess) *bytes = f->smem_optin;
  return e;
}

cudaError_t ensure_dynamic_smem(const void* fn, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_smem.find({dev, fn});
  if (it != g_smem.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) g_smem[{dev, fn}] = bytes;
  return e;
}

cudaError_t cached_occupancy(int* per_sm, const void* fn, int block, size_t smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_tuple(dev, fn, block, smem);
  {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_occupancy.find(key);
    if (it != g_occupancy.end()) {
      *per_sm = it->second;
      return cudaSuccess;
    }
  }
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, fn, block, smem);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_mu);
  g_occupancy[key] = *per_sm;
  return cudaSuccess;
}

}  // namespace attnres
