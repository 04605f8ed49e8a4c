// Exhaustive device self-checks of the arithmetic helpers that stand in for
// compiler-provided operations in the tensor-core kernels (tc_common.cuh),
// over all 2^32 binary32 bit patterns except NaNs:
//   0: tcx::tf32_round(a) against cvt.rna.tf32.f32,
//   1: div6(a) against the IEEE quotient a / 6.0f, by div6's contract
//      (arith.cuh): bitwise equal for finite a with a normal or zero
//      quotient, within 2^-149 and of the same sign for a subnormal quotient,
//      NaN for infinite a.
#include <cuda_runtime.h>

#include <cstdint>

#include "illumina.h"
#include "tc_common.cuh"

namespace {

__device__ bool div6_in_contract(float a) {
  const float got = illumina::gpu::div6(a), want = a / 6.0f;
  if (isinf(a)) return isnan(got);
  const uint32_t g = __float_as_uint(got), w = __float_as_uint(want);
  if (a == 0.0f || fabsf(a) >= 6.0f * 0x1p-126f) return g == w;
  // subnormal quotient: same sign, magnitudes at most one step apart
  const uint32_t gm = g & 0x7fffffffu, wm = w & 0x7fffffffu;
  return (g >> 31) == (w >> 31) && (gm > wm ? gm - wm : wm - gm) <= 1u;
}

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
                                 : div6_in_contract(a);
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
