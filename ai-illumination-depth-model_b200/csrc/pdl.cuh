// Programmatic dependent launch (PDL) for the forward's kernels.
//
// Every forward kernel is launched with programmatic stream serialization, so
// the next kernel of the chain may start while the current one still runs:
// each CTA calls pdl_trigger() as it starts, and once every CTA of a grid has
// started (or exited) its dependent grid may be scheduled onto SMs that have
// room. A dependent kernel runs only its prologue (barrier init, TMEM
// allocation, bias and weight staging, all read-only data) before
// pdl_wait(), which returns once the preceding grid has completed and its
// memory is visible; every access to activations, residuals, workspaces and
// outputs comes after it, so reuse of arena buffers stays ordered. Outside a
// programmatic dependency both calls are no-ops.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace illumina {
namespace gpu {

#ifdef __CUDACC__
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#endif

// Whether launch_pdl requests programmatic serialization on this host thread.
// The runtime enables it for small batches, where early launch overlaps each
// kernel's prologue with its predecessor's tail; at large batches the early
// CTAs only compete with the running kernel.
bool &pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
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
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace gpu
}  // namespace illumina
