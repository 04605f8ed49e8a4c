// Source-texture sampling in front of the network: the texture read of
// makePreprocess (src/model/kernels/io.ts:64-118) when the source is an 8-bit
// RGBA image of any size rather than frames already at network resolution.
//
// Output pixel (x, y) of the size x size network frame samples the source at
//   uv = ((x + 0.5) / size, (y + 0.5) / size) * uvScale + uvOffset
// (io.ts:76-84; createDepthModel's uvScale/uvOffset options, runner.ts:88-89,
// :181-182), optionally mirrored first (u = 1 - u, the blit's mirror,
// src/scene/blit.ts:57-60), with a linear-filtering, clamp-to-edge sampler
// (runner.ts:177): texel coordinate t = uv * extent - 0.5, the two texels
// floor(t) and floor(t) + 1 clamped to the image, weights from fract(t). The
// 8-bit texels read as unorm (value / 255). The result is the planar float
// frame illumina_forward consumes, so the sRGB decode, exposure and
// normalisation stay fused into the network's first kernel. The blit's
// aspect-preserving centre crop (cropTransform, blit.ts:80-86) is this
// transform with uvScale/uvOffset = the crop, so a camera frame is sampled
// once, directly, instead of blitted into a square texture first.
//
// All arithmetic is explicitly rounded (no FMA contraction) so texel choice and
// weights are bit-identical to a scalar float32 evaluation of the same
// expressions.
#include <cstdint>

#include "kernels.h"

namespace illumina {
namespace gpu {

namespace {

// The 256 unorm values v / 255 (correctly rounded), built once per CTA: a
// table load per texel channel instead of a division.
__global__ void __launch_bounds__(256) k_sample_source(const uchar4 *__restrict__ src, int sw, int sh, float su,
                                                       float sv, float ou, float ov, int mirror, int size,
                                                       float *__restrict__ frames) {
  __shared__ float unorm[256];
  unorm[threadIdx.y * blockDim.x + threadIdx.x] = __fdiv_rn((float)(threadIdx.y * blockDim.x + threadIdx.x), 255.0f);
  __syncthreads();
  auto unorm8 = [&](uint32_t v) { return unorm[v]; };
  const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
  if (x >= size || y >= size) return;
  const long f = blockIdx.z;
  const float fs = (float)size;
  float u = __fdiv_rn(__fadd_rn((float)x, 0.5f), fs);
  const float v = __fdiv_rn(__fadd_rn((float)y, 0.5f), fs);
  if (mirror) u = __fsub_rn(1.0f, u);
  const float uu = __fadd_rn(__fmul_rn(u, su), ou), vv = __fadd_rn(__fmul_rn(v, sv), ov);
  const float tx = __fsub_rn(__fmul_rn(uu, (float)sw), 0.5f), ty = __fsub_rn(__fmul_rn(vv, (float)sh), 0.5f);
  const float fx0 = floorf(tx), fy0 = floorf(ty);
  const float ax = __fsub_rn(tx, fx0), ay = __fsub_rn(ty, fy0);
  // clamp in float first: a uv far outside [0, 1] must not overflow the int conversion
  const int x0 = (int)fminf(fmaxf(fx0, 0.0f), (float)(sw - 1)), x1 = (int)fminf(fmaxf(fx0 + 1.0f, 0.0f), (float)(sw - 1));
  const int y0 = (int)fminf(fmaxf(fy0, 0.0f), (float)(sh - 1)), y1 = (int)fminf(fmaxf(fy0 + 1.0f, 0.0f), (float)(sh - 1));
  const uchar4 *img = src + f * (long)sw * sh;
  const uchar4 a = img[(long)y0 * sw + x0], b = img[(long)y0 * sw + x1];
  const uchar4 c = img[(long)y1 * sw + x0], d = img[(long)y1 * sw + x1];
  const float wx0 = __fsub_rn(1.0f, ax), wy0 = __fsub_rn(1.0f, ay);
  const float w00 = __fmul_rn(wx0, wy0), w10 = __fmul_rn(ax, wy0), w01 = __fmul_rn(wx0, ay), w11 = __fmul_rn(ax, ay);
  const uint32_t ca[3] = {a.x, a.y, a.z}, cb[3] = {b.x, b.y, b.z}, cc[3] = {c.x, c.y, c.z}, cd[3] = {d.x, d.y, d.z};
  const long plane = (long)size * size, o = (long)y * size + x;
#pragma unroll
  for (int k = 0; k < 3; k++) {
    float s = __fmul_rn(unorm8(ca[k]), w00);
    s = __fadd_rn(s, __fmul_rn(unorm8(cb[k]), w10));
    s = __fadd_rn(s, __fmul_rn(unorm8(cc[k]), w01));
    s = __fadd_rn(s, __fmul_rn(unorm8(cd[k]), w11));
    frames[(f * 3 + k) * plane + o] = s;
  }
}

}  // namespace

cudaError_t sample_source(const uint8_t *rgba8, int n, int sw, int sh, const float uv_scale[2],
                          const float uv_offset[2], int mirror, int size, float *frames, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const dim3 block(32, 8), grid((size + 31) / 32, (size + 7) / 8, n);
  k_sample_source<<<grid, block, 0, st>>>(reinterpret_cast<const uchar4 *>(rgba8), sw, sh, uv_scale[0], uv_scale[1],
                                          uv_offset[0], uv_offset[1], mirror, size, frames);
  return cudaGetLastError();
}

}  // namespace gpu
}  // namespace illumina
