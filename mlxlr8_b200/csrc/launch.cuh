// Launch helpers for the decode kernel chain: programmatic dependent launch
// and one shared-memory carveout for every kernel of the chain.
//
// Programmatic dependent launch lets a kernel be scheduled while the previous
// kernel of the stream is still running: the previous kernel calls
// pdl_launch_dependents() (at its start), the next kernel's CTAs become
// resident as SM resources free up, and each calls pdl_wait() before it
// touches memory that earlier work writes or reads.  pdl_wait() returns once
// the previous grid has completed and its memory is visible (and that grid
// itself waited for its own predecessor).  Launched without the attribute,
// both calls do nothing.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace exlr8 {

__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Prefer the largest shared-memory carveout: the stream kernel needs about
// 207 KB per SM, and kernels of the chain that asked for another L1/shared
// split would make the SM reconfigure (and flush L1) at every launch.
template <typename Kernel>
inline cudaError_t prefer_shared_carveout(Kernel kernel) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                              static_cast<int>(cudaSharedmemCarveoutMaxShared));
}

// `kernel<<<grid, block, smem, s>>>(args...)` with programmatic stream
// serialisation allowed (see above).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace exlr8
