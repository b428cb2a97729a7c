// Per-device launch set-up shared by the host code of every kernel file.
//
// Kernel attributes such as the dynamic shared-memory limit belong to one device's context:
// a process that launches the same kernel on two GPUs (evaluation on cuda:1, a tool that
// drives several devices from one process) has to set them on each GPU. These helpers key
// every one-time step by (kernel, device) instead of by process, and are safe to call from
// several host threads.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <set>
#include <tuple>

namespace hrm {

constexpr int kMaxDevices = 64;

inline int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

// Number of SMs of the current device (looked up once per device).
inline int device_sm_count() {
  static std::atomic<int> cache[kMaxDevices];
  const int dev = current_device();
  int n = dev < kMaxDevices ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (n == 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (dev < kMaxDevices) cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Raises the dynamic shared-memory limit of `func` to `bytes` on the current device, once per
// (kernel, device, size). Returns the error of the attribute call (cudaSuccess once done).
inline cudaError_t ensure_dynamic_smem(const void* func, int bytes) {
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, int>> done;
  const auto key = std::make_tuple(func, current_device(), bytes);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert(key);
  return e;
}

}  // namespace hrm
