// launch.cuh - programmatic dependent launch (PDL) for the kernel chains.
//
// A kernel launched with launch_pdl may start while the previous kernel on
// the stream is still finishing; it runs its independent prologue (shared
// memory tables, mbarrier init, tensor-map prefetch) and then calls
// pdl_wait(), which returns once every prerequisite grid has completed and
// its memory is visible. pdl_trigger() lets the next kernel start launching
// early. Both are no-ops for a kernel launched the ordinary way. Every
// kernel calls pdl_wait() before its first read of data another kernel
// produced.
#pragma once
#include <utility>
#include <cuda_runtime.h>

namespace dsv4 {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace dsv4
