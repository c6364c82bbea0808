// Kernel launch with optional programmatic dependent launch (PDL), so the decode step's chain of
// kernels overlaps each launch and prologue with the previous kernel's tail. HCP_PDL=0 turns it
// off. Kernels launched this way call pdl_wait() before reading anything a predecessor writes.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

namespace hcp {

inline bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = std::getenv("HCP_PDL");
    v = (s && *s) ? (std::atoi(s) != 0) : 1;
  }
  return v != 0;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Kernel function attributes (dynamic shared-memory opt-in, carveout) belong to a device's
// context, so a process that launches on several GPUs has to set them on each. `once_per_device`
// runs `set` the first time a call site meets the current device (devices 0-63 are remembered in
// `done`; higher ones set it on every call) and returns its result; afterwards cudaSuccess. Two
// host threads that race both run `set`, which is harmless: the attribute calls are idempotent.
template <typename F>
cudaError_t once_per_device(std::atomic<unsigned long long>& done, F&& set) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = set();
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// The same for a call site shared by several kernels (one launch helper for every batch size or
// kernel variant): remembered per (device, kernel address), so each kernel gets its attributes.
template <typename F>
cudaError_t once_per_device_kernel(const void* kernel, F&& set) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({dev, kernel})) return cudaSuccess;
  }
  e = set();
  if (e == cudaSuccess) {
    std::lock_guard<std::mutex> lock(mu);
    done.insert({dev, kernel});
  }
  return e;
}

}  // namespace hcp
