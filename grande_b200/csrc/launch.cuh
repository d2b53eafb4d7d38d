// Kernel launches with programmatic dependent launch (PDL): the next kernel
// in the stream may be scheduled while this one drains, runs its prologue
// (barrier init, TMEM allocation, tensor-map prefetch), and then waits in
// griddep_wait() until this grid has completed and its writes are visible.
// Every kernel launched this way calls griddep_wait() before its first read
// of memory an earlier kernel wrote (and before any global write), and
// griddep_launch() after its last global write.
#pragma once
#include <cuda_runtime.h>

namespace omg {

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace omg
