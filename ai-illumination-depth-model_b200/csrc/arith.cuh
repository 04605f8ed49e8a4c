// Division by 6 for hardswish (x * relu6(x + 3) / 6) in every kernel.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace illumina {
namespace gpu {

// a / 6 in binary32 with three FMA-pipe operations and no branch, in place of
// the compiler's divide sequence (a reciprocal, its refinement and a
// slow-path branch per quotient).
//
// q0 = RN(a * c) with c = RN(1/6) is within one ulp of a / 6, so the
// remainder r = a - 6 q0 is exactly representable and one FMA computes it
// exactly; by Markstein's theorem on correction steps (c within half an ulp
// of 1/6, q0 within one ulp of the quotient) RN(q0 + r c) is the correctly
// rounded quotient whenever nothing underflows. The sign is copied from a so
// that -0 / 6 stays -0. Contract, checked over every binary32 input by
// illumina_selftest:
//   - |a| >= 6 * 2^-126 (normal quotient), finite, or a = +-0: bitwise a / 6.0f;
//   - 0 < |a| < 6 * 2^-126 (subnormal quotient): within one subnormal step
//     (2^-149) of a / 6.0f, same sign;
//   - a = +-inf: NaN (the IEEE quotient is +-inf).
__device__ __forceinline__ float div6(float a) {
  constexpr float c = 1.0f / 6.0f;
  const float q0 = a * c;
  const float r = fmaf(-q0, 6.0f, a);
  const float q = fmaf(r, c, q0);
  return __uint_as_float((__float_as_uint(q) & 0x7fffffffu) | (__float_as_uint(a) & 0x80000000u));
}

}  // namespace gpu
}  // namespace illumina
