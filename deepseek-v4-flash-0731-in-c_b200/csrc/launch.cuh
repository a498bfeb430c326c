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
#include <cstdlib>
#include <mutex>
#include <utility>
#include <vector>
#include <cuda_runtime.h>

namespace dsv4 {

// Every kernel of the chains asks for the largest shared-memory carveout:
// a CTA of a small kernel (router, SwiGLU, combine) and one of a streaming
// GEMV (~150 KB of shared memory) then share an SM without the SM first
// draining to change its L1 / shared-memory split, which otherwise delays
// a kernel forked onto a side stream by several microseconds.
inline void prefer_max_shared(const void* fn) {
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& d : done)
    if (d.first == fn && d.second == dev) return;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    (void)cudaGetLastError();  // a preference only: clear the failure
  done.emplace_back(fn, dev);
}

// Raises a kernel's dynamic shared-memory limit to `bytes` once per
// (kernel, device): the attribute belongs to the device current at the call.
inline cudaError_t set_max_dynamic_smem(const void* fn, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& d : done)
    if (d.first == fn && d.second == dev) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.emplace_back(fn, dev);
  return e;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// DSV4_PDL=0 in the environment launches every kernel the ordinary way
// (each starts after the previous one has finished): a profile then shows
// each kernel's own duration.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("DSV4_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  prefer_max_shared(reinterpret_cast<const void*>(kernel));
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
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace dsv4
