// Kernel launch with optional programmatic dependent launch (PDL), so the decode step's chain of
// kernels overlaps each launch and prologue with the previous kernel's tail. HCP_PDL=0 turns it
// off. Kernels launched this way call pdl_wait() before reading anything a predecessor writes.
#pragma once

#include <cuda_runtime.h>

#include <cstdlib>

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

}  // namespace hcp
