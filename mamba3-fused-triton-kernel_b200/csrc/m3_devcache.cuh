// Per-device launch configuration caches, safe under concurrent host threads.
//
// A dynamic-shared-memory opt-in (cudaFuncSetAttribute) applies to the
// device that is current when it is made, and an occupancy answer belongs to
// one device, so every cache here is indexed by the current device.  Each
// kernel instantiation owns one LaunchCache (a function-local static of its
// launcher); a mutex guards it, so two host threads that launch the same
// kernel, on the same or on different GPUs, neither race on it nor skip the
// opt-in on a device that has not had it.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <mutex>

namespace m3 {

constexpr int kMaxCachedDevices = 64;

inline cudaError_t current_device(int *dev) {
  const cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return e;
  if (*dev < 0 || *dev >= kMaxCachedDevices) return cudaErrorInvalidDevice;
  return cudaSuccess;
}

// SM count of the current device (148 on a B200; 148 if it cannot be read).
inline int sm_count_current() {
  static std::atomic<int> cached[kMaxCachedDevices] = {};
  int dev = 0;
  if (current_device(&dev) != cudaSuccess) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

struct LaunchCache {
  std::mutex mu;
  int smem_optin[kMaxCachedDevices] = {};  // dynamic smem granted on each device (0: not yet)
  size_t occ_smem[kMaxCachedDevices] = {};  // key of the cached occupancy: smem bytes ...
  int occ_threads[kMaxCachedDevices] = {};  // ... and threads (0: nothing cached)
  int occ[kMaxCachedDevices] = {};
};

// Opts `kern` in to `bytes` of dynamic shared memory on the current device,
// once per device (again only if a later call asks for more).
template <typename K>
cudaError_t ensure_smem_optin(LaunchCache &c, K kern, int bytes) {
  int dev = 0;
  cudaError_t e = current_device(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(c.mu);
  if (c.smem_optin[dev] >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  c.smem_optin[dev] = bytes;
  return cudaSuccess;
}

// CTAs of `threads` threads and `smem` dynamic bytes resident per SM of the
// current device (the last (threads, smem) asked for is cached per device).
template <typename K>
cudaError_t occupancy_per_sm(LaunchCache &c, K kern, int threads, size_t smem, int *per_sm) {
  int dev = 0;
  cudaError_t e = current_device(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(c.mu);
  if (c.occ_threads[dev] == threads && c.occ_smem[dev] == smem) {
    *per_sm = c.occ[dev];
    return cudaSuccess;
  }
  int n = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, smem);
  if (e != cudaSuccess) return e;
  c.occ[dev] = n;
  c.occ_threads[dev] = threads;
  c.occ_smem[dev] = smem;
  *per_sm = n;
  return cudaSuccess;
}

}  // namespace m3
