// Process-wide count of the kernels this library has launched (or recorded
// into a CUDA graph under capture).  Every launch site adds its launches;
// qi_b200_launch_count reads the total.
#pragma once
#include <atomic>
#include <cuda_runtime.h>

namespace qib {

inline std::atomic<unsigned long long>& launch_counter() {
  static std::atomic<unsigned long long> n{0};
  return n;
}

inline void count_launches(int n) { launch_counter().fetch_add(static_cast<unsigned long long>(n), std::memory_order_relaxed); }

// Programmatic dependent launch: a kernel launched with launch_pdl may start
// (prologue: barriers, TMEM, descriptor prefetch) while the previous kernel in
// the stream is still running.  Every kernel launched this way calls
// griddep_wait() before it touches global memory, and then
// griddep_launch_dependents() so the next such kernel can start its prologue.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              int cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (cluster > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace qib
