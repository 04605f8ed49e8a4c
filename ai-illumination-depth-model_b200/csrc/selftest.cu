// Exhaustive device self-checks of the arithmetic helpers that stand in for
// compiler-provided operations in the tensor-core kernels (tc_common.cuh),
// over all 2^32 binary32 bit patterns except NaNs:
//   0: tcx::tf32_round(a) against cvt.rna.tf32.f32,
//   1: tcx::div6(a) against the IEEE quotient a / 6.0f.
#include <cuda_runtime.h>

#include <cstdint>

#include "illumina.h"
#include "tc_common.cuh"

namespace {

__global__ void k_selftest(int which, unsigned long long *out) {
  const uint64_t total = 1ull << 32;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  unsigned long long checked = 0, bad = 0;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t bits = (uint32_t)i;
    const float a = __uint_as_float(bits);
    if (isnan(a)) continue;
    checked++;
    const bool same = which == 0 ? illumina::gpu::tcx::tf32_round(a) == illumina::gpu::tcx::tf32_rna(a)
                                 : __float_as_uint(illumina::gpu::tcx::div6(a)) == __float_as_uint(a / 6.0f);
    if (!same) {
      bad++;
      atomicCAS(&out[2], 0xffffffffffffffffull, (unsigned long long)bits);
    }
  }
  atomicAdd(&out[0], checked);
  if (bad) atomicAdd(&out[1], bad);
}

}  // namespace

extern "C" illumina_status illumina_selftest(int which, unsigned long long *result) {
  if (!result || which < 0 || which > 1) return ILLUMINA_INVALID_ARG;
  unsigned long long *d = nullptr;
  if (cudaMalloc(&d, 3 * sizeof(unsigned long long)) != cudaSuccess) return ILLUMINA_CUDA_ERROR;
  const unsigned long long init[3] = {0, 0, 0xffffffffffffffffull};
  cudaError_t e = cudaMemcpy(d, init, sizeof(init), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    k_selftest<<<4 * 148, 256>>>(which, d);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpy(result, d, sizeof(init), cudaMemcpyDeviceToHost);
  cudaFree(d);
  return e == cudaSuccess ? ILLUMINA_OK : ILLUMINA_CUDA_ERROR;
}
