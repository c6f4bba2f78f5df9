// Kernel launches of the library: every kernel is launched with programmatic
// stream serialisation (programmatic dependent launch), so its launch and
// prologue overlap the tail of the previous kernel in the stream. Each kernel
// calls pdl_wait() (eir_common.cuh) before its first global memory access and
// pdl_launch_dependents() once all of its CTAs are running. EIR_PDL=0 turns
// the attribute off (plain stream order).
#pragma once

#include <cuda_runtime.h>
#include <cstdlib>

namespace eir {

inline bool pdl_enabled() {
  static const bool on = [] {
    char const *v = std::getenv("EIR_PDL");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t st, Args const &...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace eir
