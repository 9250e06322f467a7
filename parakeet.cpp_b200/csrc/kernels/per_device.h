// Thread-safe per-device cache for one-time launch set-up (kernel attributes,
// occupancy figures). Several host threads may launch on different devices at
// once (the multi-device dispatcher runs one per device), so the first launch
// of a kernel on each device runs its set-up under a lock; later launches
// read the cached value. Any device index is accepted.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <mutex>

namespace pkc {

struct PerDevice {
  std::mutex mu;
  std::map<int, int> val;  // device -> value recorded by the set-up
};

// The value recorded for the current device, running init(value) first if
// this is the device's first call. A failing init records nothing.
template <typename F>
cudaError_t per_device(PerDevice& pd, int* out, F&& init) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> g(pd.mu);
  auto it = pd.val.find(dev);
  if (it != pd.val.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  int v = 0;
  e = init(dev, v);
  if (e != cudaSuccess) return e;
  pd.val[dev] = v;
  *out = v;
  return cudaSuccess;
}

// Raise kernel `kern`'s dynamic shared memory allowance on the current device
// to at least `bytes`; the largest allowance granted is kept per device.
template <typename K>
cudaError_t allow_smem(PerDevice& pd, K kern, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> g(pd.mu);
  auto it = pd.val.find(dev);
  if (it != pd.val.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) pd.val[dev] = bytes;
  return e;
}

}  // namespace pkc
