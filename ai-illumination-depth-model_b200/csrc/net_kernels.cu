// CUDA kernels of the IlluminaDepth forward pass (sm_100a).
//
// Layout: every activation is channels-last with the batch outermost,
// (n, y, x, c), c a multiple of 4, stored as float32 or bfloat16 (`T`); all
// arithmetic accumulates in float32. The op semantics are the reference's
// (src/model/reference.ts): residual added before the activation, the
// depthwise result activated before the pointwise, bilinear taps clamped
// independently, sigmoid head broadcast, 3x3 joint-bilateral upsample.
//
// The pointwise-shaped ops (pw, dw->pw, lateral) share one register-blocked
// tile GEMM: a CTA owns BM output pixels x BN output channels, walks the input
// channels in chunks of 16 staged through shared memory, and fuses the
// operand producer (plain load, depthwise k x k + bias + activation, or the
// skip tensor) and the epilogue (bias, residual / bilinear-upsampled coarse,
// activation) so no intermediate reaches HBM.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "arith.cuh"
#include "kernels.h"
#include "pdl.cuh"

namespace illumina {
namespace gpu {

// ---------------------------------------------------------------------------
// helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ float act_apply(int act, float v) {
  switch (act) {
    case 1: return fmaxf(v, 0.0f);
    case 2: return fminf(fmaxf(v, 0.0f), 6.0f);
    case 3: return div6(v * fminf(fmaxf(v + 3.0f, 0.0f), 6.0f));
    default: return v;
  }
}

template <typename T>
struct Io;

template <>
struct Io<float> {
  static __device__ __forceinline__ float4 load4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
  static __device__ __forceinline__ void store4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
  static __device__ __forceinline__ float2 load2(const float *p) { return *reinterpret_cast<const float2 *>(p); }
  static __device__ __forceinline__ void store2(float *p, float2 v) { *reinterpret_cast<float2 *>(p) = v; }
  static __device__ __forceinline__ float4 round4(float4 v) { return v; }
};

template <>
struct Io<__nv_bfloat16> {
  static __device__ __forceinline__ float4 load4(const __nv_bfloat16 *p) {
    uint2 r = *reinterpret_cast<const uint2 *>(p);
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162 *>(&r.x), b = *reinterpret_cast<__nv_bfloat162 *>(&r.y);
    float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
  }
  static __device__ __forceinline__ void store4(__nv_bfloat16 *p, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 r;
    r.x = *reinterpret_cast<uint32_t *>(&a);
    r.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = r;
  }
  static __device__ __forceinline__ float2 load2(const __nv_bfloat16 *p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(p));
  }
  static __device__ __forceinline__ void store2(__nv_bfloat16 *p, float2 v) {
    *reinterpret_cast<__nv_bfloat162 *>(p) = __floats2bfloat162_rn(v.x, v.y);
  }
  // the value a store4 + load4 round trip gives back
  static __device__ __forceinline__ float4 round4(float4 v) {
    const float2 a = __bfloat1622float2(__floats2bfloat162_rn(v.x, v.y));
    const float2 b = __bfloat1622float2(__floats2bfloat162_rn(v.z, v.w));
    return make_float4(a.x, a.y, b.x, b.y);
  }
};

__device__ __forceinline__ float4 f4add(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 f4fma(float4 a, float4 b, float4 c) {
  return make_float4(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y), fmaf(a.z, b.z, c.z), fmaf(a.w, b.w, c.w));
}

// The power is exp2(2.4 * log2(x)) on the hardware approximations (__powf,
// within ~1e-6 relative here): the accuracy WGSL defines for the reference
// shader's pow, at a small fraction of powf's instruction count. The
// divisions by constants are products with the rounded reciprocals (within
// 1.5 ulp of the quotient; WGSL gives its division 2.5 ulp).
__device__ __forceinline__ float srgb_to_linear(float c) {
  return c <= 0.04045f ? c * (1.0f / 12.92f) : __powf((c + 0.055f) * (1.0f / 1.055f), 2.4f);
}

static inline unsigned blocks_for(long n, int threads) { return (unsigned)((n + threads - 1) / threads); }

// idx = (b * H + y) * W + x, split with 32-bit division (64-bit division is a
// long software sequence); launches check that their index range is below 2^31.
__device__ __forceinline__ void unflatten3(long idx, int W, int H, int &x, int &y, int &b) {
  const uint32_t u = (uint32_t)idx, uw = (uint32_t)W, uh = (uint32_t)H;
  const uint32_t t = u / uw;
  x = (int)(u - t * uw);
  const uint32_t bb = t / uh;
  y = (int)(t - bb * uh);
  b = (int)bb;
}
constexpr long kMaxIndex = 0x7fffffffL;

bool &pdl_enabled() {
  static thread_local bool on = false;
  return on;
}

// ---------------------------------------------------------------------------
// preprocess (src/model/kernels/io.ts:64-118 semantics, refPreprocess)
// ---------------------------------------------------------------------------

// One pixel: sRGB decode (optional), exposure, then the normalised network
// input (r, g, b standardised with the rounded reciprocal of std; w = linear
// luma). r, g, bl come back as the
// exposed linear colour (the scene colour).
__device__ __forceinline__ float4 preprocess_px(float &r, float &g, float &bl, const PreprocessParams &p) {
  if (p.decode_srgb) r = srgb_to_linear(r), g = srgb_to_linear(g), bl = srgb_to_linear(bl);
  r *= p.exposure, g *= p.exposure, bl *= p.exposure;
  const float l = 0.2126f * r + 0.7152f * g + 0.0722f * bl;
  return make_float4((r - p.mean[0]) * p.inv_std[0], (g - p.mean[1]) * p.inv_std[1], (bl - p.mean[2]) * p.inv_std[2],
                     l);
}

// Parameter list mirrored by kPreprocessArgCount / kPreprocessFramesArg.
template <typename T>
__global__ void k_preprocess(const float *__restrict__ frames, int layout, long total, int S, PreprocessParams p,
                             T *__restrict__ input, float *__restrict__ luma, float *__restrict__ scene) {
  pdl_wait();
  pdl_trigger();
  long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  long plane = (long)S * S;
  const uint32_t ub = (uint32_t)idx / (uint32_t)plane;
  long b = ub, pix = idx - b * plane;
  float r, g, bl;
  if (layout == 0) {
    const float *f = frames + b * 3 * plane + pix;
    r = __ldg(f), g = __ldg(f + plane), bl = __ldg(f + 2 * plane);
  } else {
    float4 v = __ldg(reinterpret_cast<const float4 *>(frames) + idx);
    r = v.x, g = v.y, bl = v.z;
  }
  const float4 o = preprocess_px(r, g, bl, p);
  const float l = o.w;
  Io<T>::store4(input + idx * 4, o);
  if (luma) luma[idx] = l;
  if (scene) reinterpret_cast<float4 *>(scene)[idx] = make_float4(r, g, bl, 1.0f);
}

cudaError_t preprocess(int T, const float *frames, int layout, int n, int S, const PreprocessParams &p, void *input,
                       float *luma, float *scene, cudaStream_t st) {
  long total = (long)n * S * S;
  if (total > kMaxIndex) return cudaErrorInvalidValue;
  if (total == 0) return cudaSuccess;
  if (T == F32)
    return launch_pdl(k_preprocess<float>, dim3(blocks_for(total, 256)), dim3(256), 0, st, frames, layout, total, S, p,
                      (float *)input, luma, scene);
  return launch_pdl(k_preprocess<__nv_bfloat16>, dim3(blocks_for(total, 256)), dim3(256), 0, st, frames, layout, total,
                    S, p, (__nv_bfloat16 *)input, luma, scene);
}

// ---------------------------------------------------------------------------
// dense k x k conv (stem): one thread = one output pixel x 16 channels
// ---------------------------------------------------------------------------

template <typename T>
__global__ void k_conv(const T *__restrict__ src, int n, int H, int W, int Cin, const float *__restrict__ wpk,
                       const float *__restrict__ bias, int Cout, int k, int stride, int act, int OH, int OW,
                       T *__restrict__ dst) {
  pdl_wait();
  pdl_trigger();
  long pix = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long total = (long)n * OH * OW;
  if (pix >= total) return;
  int og = blockIdx.y;  // group of 16 output channels
  int ox, oy, b;
  unflatten3(pix, OW, OH, ox, oy, b);
  int pad = (k - 1) >> 1;
  int cout4 = Cout >> 2, cin4 = Cin >> 2;
  int g0 = og * 4;
  float4 acc[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    int g = g0 + j;
    acc[j] = g < cout4 ? __ldg(reinterpret_cast<const float4 *>(bias) + g) : make_float4(0, 0, 0, 0);
  }
  for (int ky = 0; ky < k; ky++) {
    int iy = oy * stride + ky - pad;
    if (iy < 0 || iy >= H) continue;
    for (int kx = 0; kx < k; kx++) {
      int ix = ox * stride + kx - pad;
      if (ix < 0 || ix >= W) continue;
      const T *px = src + (((long)b * H + iy) * W + ix) * Cin;
      const float4 *wk = reinterpret_cast<const float4 *>(wpk) + (long)(ky * k + kx) * Cin * cout4;
      for (int c4 = 0; c4 < cin4; c4++) {
        float4 x = Io<T>::load4(px + c4 * 4);
        float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float4 *wr = wk + (long)(c4 * 4 + q) * cout4;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            int g = g0 + j;
            if (g < cout4) acc[j] = f4fma(make_float4(xs[q], xs[q], xs[q], xs[q]), __ldg(wr + g), acc[j]);
          }
        }
      }
    }
  }
  T *o = dst + pix * Cout;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    int g = g0 + j;
    if (g < cout4) {
      float4 v = acc[j];
      v = make_float4(act_apply(act, v.x), act_apply(act, v.y), act_apply(act, v.z), act_apply(act, v.w));
      Io<T>::store4(o + g * 4, v);
    }
  }
}

// Same op with the 16-channel group's weights staged in shared memory
// ([k*k*Cin] x 4 float4, broadcast reads) and two output pixels per thread,
// so each weight read serves eight FMAs. Accumulation order per output is
// that of k_conv (bias, then ky, kx, input channel).
template <typename T>
__global__ void k_conv_sw(const T *__restrict__ src, int n, int H, int W, int Cin, const float *__restrict__ wpk,
                          const float *__restrict__ bias, int Cout, int k, int stride, int act, int OH, int OW,
                          T *__restrict__ dst) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float4 wsm[];
  const int og = blockIdx.y, cout4 = Cout >> 2, cin4 = Cin >> 2, g0 = og * 4;
  const int rows = k * k * Cin;
  for (int i = threadIdx.x; i < rows * 4; i += blockDim.x) {
    const int r = i >> 2, g = g0 + (i & 3);
    wsm[i] = g < cout4 ? __ldg(reinterpret_cast<const float4 *>(wpk) + (long)r * cout4 + g) : make_float4(0, 0, 0, 0);
  }
  __syncthreads();
  const long total = (long)n * OH * OW;
  const long pix0 = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (pix0 >= total) return;
  const int npx = pix0 + 1 < total ? 2 : 1;
  const int pad = (k - 1) >> 1;
  int ox[2], oy[2], ob[2];
#pragma unroll
  for (int u = 0; u < 2; u++) unflatten3(u < npx ? pix0 + u : pix0, OW, OH, ox[u], oy[u], ob[u]);
  float4 acc[2][4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int g = g0 + j;
    const float4 bj = g < cout4 ? __ldg(reinterpret_cast<const float4 *>(bias) + g) : make_float4(0, 0, 0, 0);
    acc[0][j] = bj, acc[1][j] = bj;
  }
  for (int ky = 0; ky < k; ky++) {
    for (int kx = 0; kx < k; kx++) {
      const T *px[2];
      bool ok[2];
#pragma unroll
      for (int u = 0; u < 2; u++) {
        const int iy = oy[u] * stride + ky - pad, ix = ox[u] * stride + kx - pad;
        ok[u] = u < npx && iy >= 0 && iy < H && ix >= 0 && ix < W;
        px[u] = src + (((long)ob[u] * H + (ok[u] ? iy : 0)) * W + (ok[u] ? ix : 0)) * Cin;
      }
      const float4 *wk = wsm + (ky * k + kx) * Cin * 4;
      for (int c4 = 0; c4 < cin4; c4++) {
        float xs[2][4];
#pragma unroll
        for (int u = 0; u < 2; u++) {
          const float4 x = ok[u] ? Io<T>::load4(px[u] + c4 * 4) : make_float4(0, 0, 0, 0);
          xs[u][0] = x.x, xs[u][1] = x.y, xs[u][2] = x.z, xs[u][3] = x.w;
        }
#pragma unroll
        for (int qq = 0; qq < 4; qq++) {
          const float4 *wr = wk + (c4 * 4 + qq) * 4;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const float4 wv = wr[j];
#pragma unroll
            for (int u = 0; u < 2; u++)
              if (ok[u]) acc[u][j] = f4fma(make_float4(xs[u][qq], xs[u][qq], xs[u][qq], xs[u][qq]), wv, acc[u][j]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < 2; u++) {
    if (u >= npx) break;
    T *o = dst + (pix0 + u) * Cout;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int g = g0 + j;
      if (g < cout4) {
        float4 v = acc[u][j];
        v = make_float4(act_apply(act, v.x), act_apply(act, v.y), act_apply(act, v.z), act_apply(act, v.w));
        Io<T>::store4(o + g * 4, v);
      }
    }
  }
}

cudaError_t conv(int T, const void *src, int n, int H, int W, int Cin, const float *wpk, const float *bias, int Cout,
                 int k, int stride, int act, void *dst, cudaStream_t st) {
  int pad = (k - 1) >> 1;
  int OH = (H + 2 * pad - k) / stride + 1, OW = (W + 2 * pad - k) / stride + 1;
  long total = (long)n * OH * OW;
  if (total > kMaxIndex) return cudaErrorInvalidValue;
  if (total <= 0) return cudaSuccess;
  const size_t wsm = (size_t)k * k * Cin * 4 * sizeof(float4);
  if (wsm <= 32 * 1024) {
    dim3 grid(blocks_for((total + 1) / 2, 128), (Cout / 4 + 3) / 4);
    if (T == F32)
      return launch_pdl(k_conv_sw<float>, grid, dim3(128), wsm, st, (const float *)src, n, H, W, Cin, wpk, bias, Cout,
                        k, stride, act, OH, OW, (float *)dst);
    return launch_pdl(k_conv_sw<__nv_bfloat16>, grid, dim3(128), wsm, st, (const __nv_bfloat16 *)src, n, H, W, Cin,
                      wpk, bias, Cout, k, stride, act, OH, OW, (__nv_bfloat16 *)dst);
  }
  dim3 grid(blocks_for(total, 128), (Cout / 4 + 3) / 4);
  if (T == F32)
    return launch_pdl(k_conv<float>, grid, dim3(128), 0, st, (const float *)src, n, H, W, Cin, wpk, bias, Cout, k,
                      stride, act, OH, OW, (float *)dst);
  return launch_pdl(k_conv<__nv_bfloat16>, grid, dim3(128), 0, st, (const __nv_bfloat16 *)src, n, H, W, Cin, wpk, bias,
                    Cout, k, stride, act, OH, OW, (__nv_bfloat16 *)dst);
}

// ---------------------------------------------------------------------------
// preprocess fused into the stem (3x3 stride-2 conv, 4 -> 16 channels)
// ---------------------------------------------------------------------------
// One CTA = a 32 x 16 tile of stem outputs of one frame. Phase 1 preprocesses
// the tile's input window (65 x 33 pixels with the one-pixel halo) into shared
// memory, zero outside the frame (the conv's padding) and rounded to the
// storage type as the unfused stem would read it back, and writes the luma
// guide of the pixels the tile owns (its 64 x 32 interior; the scene colour
// and the normalised input too when asked for). The network input itself
// never reaches HBM. Phase 2: each thread computes 2 adjacent outputs x 16
// channels from the window with k_conv's accumulation order (bias, then ky,
// kx, input channel), the weights read as shared-memory broadcasts. Two
// outputs per thread keep a thread within 64 registers, so four 256-thread
// CTAs (32 warps) share an SM and one CTA's window loads overlap another's FMAs.
constexpr int kStemTW = 32, kStemTH = 16, kStemWinW = 2 * kStemTW + 1, kStemWinH = 2 * kStemTH + 1;
// one float4 of padding after every 8: a quarter-warp's reads (8 threads 4
// window columns apart) then fall into distinct banks
constexpr int kStemRow = kStemWinW + (kStemWinW + 7) / 8;
constexpr int kStemTaps = 9 * 4 * 4;  // [ky][kx][cin][4 float4 of output channels]
constexpr int kStemThreads = 256, kStemOut = 2, kStemWin = kStemWinH * kStemWinW;
constexpr int kStemBatch = (kStemWin + 2 * kStemThreads - 1) / (2 * kStemThreads);  // two batches
constexpr size_t kStemSmem = (size_t)(kStemWinH * kStemRow + kStemTaps) * sizeof(float4);
__device__ __forceinline__ int stem_col(int c) { return c + (c >> 3); }

// Parameter list mirrored by kStemArgCount / kStemFramesArg.
template <typename T>
__global__ void __launch_bounds__(kStemThreads, 4) k_stem_fused(const float *__restrict__ frames, const StemParams p) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float4 stem_sm[];
  float4 *win = stem_sm, *wsm = stem_sm + kStemWinH * kStemRow;
  const int tiles = p.tiles_x * p.tiles_y;
  const int b = blockIdx.x / tiles, tile = blockIdx.x - b * tiles;
  const int ty = tile / p.tiles_x, tx = tile - ty * p.tiles_x;
  const int ox0 = tx * kStemTW, oy0 = ty * kStemTH;
  const int ix0 = 2 * ox0 - 1, iy0 = 2 * oy0 - 1, S = p.S;
  for (int i = threadIdx.x; i < kStemTaps; i += kStemThreads) wsm[i] = __ldg(reinterpret_cast<const float4 *>(p.w) + i);
  const long plane = (long)S * S;
  // Planar frames at a 16-byte aligned address (S is a multiple of 32, so
  // every row and every 4-column group is aligned): the window's rows are read
  // as the 17 aligned float4 groups covering input columns ix0 - 3 .. ix0 + 64
  // (the first group's three leading pixels unused), three channel loads per
  // group, and the owned pixels' luma stored four at a time.
  if (p.layout == 0 && (S & 3) == 0 && (reinterpret_cast<uintptr_t>(frames) & 15) == 0) {
    constexpr int kGroupsX = (kStemWinW + 3 + 3) / 4, kGroupsW = kStemWinH * kGroupsX;
    for (int g0 = 0; g0 < kGroupsW; g0 += 2 * kStemThreads) {
      float4 c[2][3];
#pragma unroll
      for (int u = 0; u < 2; u++) {
        const int gi = g0 + u * kStemThreads + (int)threadIdx.x;
        const int ry = gi / kGroupsX, cg = gi - ry * kGroupsX;
        const int iy = iy0 + ry, gx = ix0 - 3 + 4 * cg;
        c[u][0] = c[u][1] = c[u][2] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (gi < kGroupsW && iy >= 0 && iy < S && gx >= 0 && gx < S) {
          const float4 *f = reinterpret_cast<const float4 *>(frames + b * 3 * plane + (long)iy * S + gx);
          c[u][0] = __ldg(f), c[u][1] = __ldg(f + plane / 4), c[u][2] = __ldg(f + plane / 2);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; u++) {
        const int gi = g0 + u * kStemThreads + (int)threadIdx.x;
        if (gi >= kGroupsW) break;
        const int ry = gi / kGroupsX, cg = gi - ry * kGroupsX;
        const int iy = iy0 + ry, gx = ix0 - 3 + 4 * cg;
        const bool in_frame = iy >= 0 && iy < S && gx >= 0 && gx < S;
        const float r4[4] = {c[u][0].x, c[u][0].y, c[u][0].z, c[u][0].w};
        const float g4[4] = {c[u][1].x, c[u][1].y, c[u][1].z, c[u][1].w};
        const float b4[4] = {c[u][2].x, c[u][2].y, c[u][2].z, c[u][2].w};
        float l4[4];
        const bool own_row = ry >= 1 && ry <= 2 * kStemTH;
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int rx = 4 * cg + e - 3;
          if (rx < 0 || rx >= kStemWinW) continue;
          float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          l4[e] = 0.0f;
          if (in_frame) {
            float r = r4[e], g = g4[e], bl = b4[e];
            const float4 o = preprocess_px(r, g, bl, p.pre);
            v = Io<T>::round4(o);
            l4[e] = o.w;
            if (own_row && rx >= 1 && rx <= 2 * kStemTW && (p.scene || p.input)) {
              const long idx = b * plane + (long)iy * S + gx + e;
              if (p.scene) reinterpret_cast<float4 *>(p.scene)[idx] = make_float4(r, g, bl, 1.0f);
              if (p.input) Io<T>::store4(static_cast<T *>(p.input) + idx * 4, o);
            }
          }
          win[ry * kStemRow + stem_col(rx)] = v;
        }
        // groups 1..16 hold owned columns only (rx 1..64); group 0 owns none
        if (in_frame && own_row && cg >= 1 && cg <= 2 * kStemTW / 4)
          *reinterpret_cast<float4 *>(p.luma + b * plane + (long)iy * S + gx) = make_float4(l4[0], l4[1], l4[2], l4[3]);
      }
    }
  } else
  // the window's pixels in batches of kStemBatch per thread, all loads of a
  // batch in flight before any is used
  for (int i0 = 0; i0 < kStemWin; i0 += kStemBatch * kStemThreads) {
    float r[kStemBatch], g[kStemBatch], bl[kStemBatch];
#pragma unroll
    for (int u = 0; u < kStemBatch; u++) {
      const int i = i0 + u * kStemThreads + (int)threadIdx.x;
      const int ry = i / kStemWinW, rx = i - ry * kStemWinW;
      const int iy = iy0 + ry, ix = ix0 + rx;
      r[u] = g[u] = bl[u] = 0.0f;
      if (i < kStemWin && iy >= 0 && iy < S && ix >= 0 && ix < S) {
        const long pix = (long)iy * S + ix;
        if (p.layout == 0) {
          const float *f = frames + b * 3 * plane + pix;
          r[u] = __ldg(f), g[u] = __ldg(f + plane), bl[u] = __ldg(f + 2 * plane);
        } else {
          const float4 c = __ldg(reinterpret_cast<const float4 *>(frames) + b * plane + pix);
          r[u] = c.x, g[u] = c.y, bl[u] = c.z;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kStemBatch; u++) {
      const int i = i0 + u * kStemThreads + (int)threadIdx.x;
      if (i >= kStemWin) break;
      const int ry = i / kStemWinW, rx = i - ry * kStemWinW;
      const int iy = iy0 + ry, ix = ix0 + rx;
      float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (iy >= 0 && iy < S && ix >= 0 && ix < S) {
        const long idx = b * plane + (long)iy * S + ix;
        const float4 o = preprocess_px(r[u], g[u], bl[u], p.pre);
        v = Io<T>::round4(o);
        if (ry >= 1 && rx >= 1 && ry <= 2 * kStemTH && rx <= 2 * kStemTW) {
          p.luma[idx] = o.w;
          if (p.scene) reinterpret_cast<float4 *>(p.scene)[idx] = make_float4(r[u], g[u], bl[u], 1.0f);
          if (p.input) Io<T>::store4(static_cast<T *>(p.input) + idx * 4, o);
        }
      }
      win[ry * kStemRow + stem_col(rx)] = v;
    }
  }
  __syncthreads();

  constexpr int kGroups = kStemTW / kStemOut, kCols = 2 * kStemOut + 1;
  const int ly = threadIdx.x / kGroups, xg = threadIdx.x % kGroups;
  const int oy = oy0 + ly, ox = ox0 + xg * kStemOut;
  if (oy >= p.OH || ox >= p.OW) return;
  float4 acc[kStemOut][4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const float4 bj = __ldg(reinterpret_cast<const float4 *>(p.bias) + j);
#pragma unroll
    for (int q = 0; q < kStemOut; q++) acc[q][j] = bj;
  }
#pragma unroll 1
  for (int ky = 0; ky < 3; ky++) {
    const float4 *row = win + (2 * ly + ky) * kStemRow;
    float xs[kCols][4];
#pragma unroll
    for (int c = 0; c < kCols; c++) {
      const float4 x = row[stem_col(2 * kStemOut * xg + c)];
      xs[c][0] = x.x, xs[c][1] = x.y, xs[c][2] = x.z, xs[c][3] = x.w;
    }
#pragma unroll
    for (int kx = 0; kx < 3; kx++) {
#pragma unroll
      for (int ci = 0; ci < 4; ci++) {
        const float4 *wr = wsm + ((ky * 3 + kx) * 4 + ci) * 4;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float4 wv = wr[j];
#pragma unroll
          for (int q = 0; q < kStemOut; q++) {
            const float x = xs[2 * q + kx][ci];
            acc[q][j] = f4fma(make_float4(x, x, x, x), wv, acc[q][j]);
          }
        }
      }
    }
  }
  T *o = static_cast<T *>(p.dst) + (((long)b * p.OH + oy) * p.OW + ox) * 16;
#pragma unroll
  for (int q = 0; q < kStemOut; q++) {
    if (ox + q >= p.OW) break;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float4 v = acc[q][j];
      Io<T>::store4(o + q * 16 + j * 4, make_float4(act_apply(p.act, v.x), act_apply(p.act, v.y),
                                                    act_apply(p.act, v.z), act_apply(p.act, v.w)));
    }
  }
}

cudaError_t stem_fused(int T, const float *frames, int layout, int n, int S, const PreprocessParams &pre,
                       const float *wpk, const float *bias, int act, void *dst, float *luma, float *scene, void *input,
                       cudaStream_t st) {
  const long total = (long)n * S * S;
  if (total > kMaxIndex || !luma) return cudaErrorInvalidValue;
  if (total == 0) return cudaSuccess;
  StemParams p;
  p.layout = layout, p.S = S;
  p.OH = (S - 1) / 2 + 1, p.OW = p.OH;
  p.tiles_x = (p.OW + kStemTW - 1) / kStemTW, p.tiles_y = (p.OH + kStemTH - 1) / kStemTH;
  p.act = act, p.pre = pre, p.w = wpk, p.bias = bias, p.dst = dst, p.luma = luma, p.scene = scene, p.input = input;
  const long blocks = (long)n * p.tiles_x * p.tiles_y;
  if (blocks > kMaxIndex) return cudaErrorInvalidValue;
  if (T == F32) return launch_pdl(k_stem_fused<float>, dim3((unsigned)blocks), dim3(kStemThreads), kStemSmem, st, frames, p);
  return launch_pdl(k_stem_fused<__nv_bfloat16>, dim3((unsigned)blocks), dim3(kStemThreads), kStemSmem, st, frames, p);
}

// ---------------------------------------------------------------------------
// tile GEMM for pw / dw->pw / lateral
// ---------------------------------------------------------------------------

constexpr int GBK = 16;       // input channels per chunk
constexpr int GTHREADS = 256; // 16 x 16 thread grid

struct GemmParams {
  const void *src;
  const float *w, *bias;
  const void *res;
  void *dst;
  const float *dw_w, *dw_b;
  const void *coarse;
  long M;
  int N, K, act, mid_act;
  int H, W, OH, OW, stride;  // dw input dims / output dims; lateral output dims in OH, OW
};

// MODE 0: pointwise; 1: depthwise KS x KS then pointwise; 2: lateral
template <typename T, int BM, int BN, int MODE, int KS>
__global__ void __launch_bounds__(GTHREADS) k_gemm(const GemmParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int TM = BM / 16, TN = BN / 16;
  constexpr int A_VEC = BM * 4;  // float4 groups per chunk (BM pixels x 4 channel groups)
  constexpr int A_PER = (A_VEC + GTHREADS - 1) / GTHREADS;
  constexpr int B_VEC = BN * 4;
  constexpr int B_PER = (B_VEC + GTHREADS - 1) / GTHREADS;
  __shared__ __align__(16) float As[GBK][BM + 4];
  __shared__ __align__(16) float Bs[GBK][BN + 4];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const long m0 = (long)blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  const int K4 = p.K >> 2;

  // Per-thread A-producer coordinates (fixed across chunks).
  int a_mm[A_PER], a_kq[A_PER];
  bool a_ok[A_PER];
  int a_b[A_PER], a_y[A_PER], a_x[A_PER];
#pragma unroll
  for (int i = 0; i < A_PER; i++) {
    int v = tid + i * GTHREADS;
    a_mm[i] = v >> 2;
    a_kq[i] = v & 3;
    long m = m0 + a_mm[i];
    a_ok[i] = (v < A_VEC) && (m < p.M);
    a_b[i] = a_y[i] = a_x[i] = 0;
    if (MODE == 1 && a_ok[i]) {
      a_x[i] = (int)(m % p.OW);
      long t = m / p.OW;
      a_y[i] = (int)(t % p.OH);
      a_b[i] = (int)(t / p.OH);
    }
  }

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = 0.0f;

  const T *src = reinterpret_cast<const T *>(p.src);
  for (int k0 = 0; k0 < p.K; k0 += GBK) {
    // ---- produce the A chunk (BM x 16) ----
#pragma unroll
    for (int i = 0; i < A_PER; i++) {
      float4 v = make_float4(0, 0, 0, 0);
      int c4 = (k0 >> 2) + a_kq[i];
      if (a_ok[i] && c4 < K4) {
        if (MODE != 1) {
          v = Io<T>::load4(src + (m0 + a_mm[i]) * p.K + c4 * 4);
        } else {
          constexpr int pad = (KS - 1) / 2;
          float4 s = __ldg(reinterpret_cast<const float4 *>(p.dw_b) + c4);
#pragma unroll
          for (int ky = 0; ky < KS; ky++) {
            int iy = a_y[i] * p.stride + ky - pad;
            if (iy < 0 || iy >= p.H) continue;
            const T *row = src + ((long)a_b[i] * p.H + iy) * p.W * p.K;
#pragma unroll
            for (int kx = 0; kx < KS; kx++) {
              int ix = a_x[i] * p.stride + kx - pad;
              if (ix < 0 || ix >= p.W) continue;
              float4 x = Io<T>::load4(row + (long)ix * p.K + c4 * 4);
              float4 w = __ldg(reinterpret_cast<const float4 *>(p.dw_w) + (long)(ky * KS + kx) * K4 + c4);
              s = f4fma(x, w, s);
            }
          }
          v = make_float4(act_apply(p.mid_act, s.x), act_apply(p.mid_act, s.y), act_apply(p.mid_act, s.z),
                          act_apply(p.mid_act, s.w));
        }
      }
      if (tid + i * GTHREADS < A_VEC) {
        int kk = a_kq[i] * 4, mm = a_mm[i];
        As[kk + 0][mm] = v.x;
        As[kk + 1][mm] = v.y;
        As[kk + 2][mm] = v.z;
        As[kk + 3][mm] = v.w;
      }
    }
    // ---- B chunk (BN x 16) from w[N][K] ----
#pragma unroll
    for (int i = 0; i < B_PER; i++) {
      int v = tid + i * GTHREADS;
      if (v < B_VEC) {
        int nn = v >> 2, kq = v & 3;
        int n = n0 + nn, c4 = (k0 >> 2) + kq;
        float4 w = make_float4(0, 0, 0, 0);
        if (n < p.N && c4 < K4) w = __ldg(reinterpret_cast<const float4 *>(p.w + (long)n * p.K) + c4);
        int kk = kq * 4;
        Bs[kk + 0][nn] = w.x;
        Bs[kk + 1][nn] = w.y;
        Bs[kk + 2][nn] = w.z;
        Bs[kk + 3][nn] = w.w;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < GBK; kk++) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; i += 2) {
        float2 t = *reinterpret_cast<const float2 *>(&As[kk][ty * TM + i]);
        a[i] = t.x, a[i + 1] = t.y;
      }
#pragma unroll
      for (int j = 0; j < TN; j += 2) {
        float2 t = *reinterpret_cast<const float2 *>(&Bs[kk][tx * TN + j]);
        b[j] = t.x, b[j + 1] = t.y;
      }
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

  // ---- epilogue ----
  const T *res = reinterpret_cast<const T *>(p.res);
  const T *coarse = reinterpret_cast<const T *>(p.coarse);
  T *dst = reinterpret_cast<T *>(p.dst);
#pragma unroll
  for (int i = 0; i < TM; i++) {
    long m = m0 + ty * TM + i;
    if (m >= p.M) continue;
    int ly0 = 0, ly1 = 0, lx0 = 0, lx1 = 0, lb = 0;
    float fx = 0, fy = 0;
    if (MODE == 2) {
      // refUpsample2 (reference.ts:161-193): source coord (i + 0.5) / 2 - 0.5,
      // both taps from the unclamped floor, clamped independently.
      int x = (int)(m % p.OW);
      long t = m / p.OW;
      int y = (int)(t % p.OH);
      lb = (int)(t / p.OH);
      int CH = p.OH >> 1, CW = p.OW >> 1;
      float sy = (y + 0.5f) * 0.5f - 0.5f, sx = (x + 0.5f) * 0.5f - 0.5f;
      float fy0 = floorf(sy), fx0 = floorf(sx);
      fy = sy - fy0, fx = sx - fx0;
      ly0 = min(max((int)fy0, 0), CH - 1), ly1 = min(max((int)fy0 + 1, 0), CH - 1);
      lx0 = min(max((int)fx0, 0), CW - 1), lx1 = min(max((int)fx0 + 1, 0), CW - 1);
      long rb = (long)lb * CH;
      ly0 = (int)((rb + ly0) * CW), ly1 = (int)((rb + ly1) * CW);  // row base pixel indices
    }
#pragma unroll
    for (int j = 0; j < TN; j += 2) {
      int n = n0 + tx * TN + j;
      if (n >= p.N) continue;
      float2 v = make_float2(acc[i][j] + __ldg(p.bias + n), acc[i][j + 1] + __ldg(p.bias + n + 1));
      if (MODE == 2) {
        long CW = p.OW >> 1;
        (void)CW;
        float2 a = Io<T>::load2(coarse + ((long)ly0 + lx0) * p.N + n);
        float2 b = Io<T>::load2(coarse + ((long)ly0 + lx1) * p.N + n);
        float2 c = Io<T>::load2(coarse + ((long)ly1 + lx0) * p.N + n);
        float2 d = Io<T>::load2(coarse + ((long)ly1 + lx1) * p.N + n);
        float w00 = (1 - fx) * (1 - fy), w01 = fx * (1 - fy), w10 = (1 - fx) * fy, w11 = fx * fy;
        v.x += a.x * w00 + b.x * w01 + c.x * w10 + d.x * w11;
        v.y += a.y * w00 + b.y * w01 + c.y * w10 + d.y * w11;
      }
      if (res) {
        float2 r = Io<T>::load2(res + m * p.N + n);
        v.x += r.x, v.y += r.y;
      }
      v.x = act_apply(p.act, v.x);
      v.y = act_apply(p.act, v.y);
      Io<T>::store2(dst + m * p.N + n, v);
    }
  }
}

template <typename T, int MODE, int KS>
static cudaError_t launch_gemm_t(const GemmParams &p, cudaStream_t st) {
  // Tile choice: wide N tiles amortise the dw producer; shrink BM until the
  // grid covers the 148 SMs at least twice.
  auto ctas = [&](int bm, int bn) { return ((p.M + bm - 1) / bm) * (long)((p.N + bn - 1) / bn); };
  int bn = p.N <= 32 ? 32 : 64;
  if (MODE == 1 && p.N > 64) bn = 128;
  int bm = 128;
  while (bm > 32 && ctas(bm, bn) < 296) bm >>= 1;
  dim3 grid((unsigned)((p.M + bm - 1) / bm), (unsigned)((p.N + bn - 1) / bn));
#define ILL_GEMM_CASE(BM_, BN_)                                      \
  if (bm == BM_ && bn == BN_) {                                      \
    return launch_pdl(k_gemm<T, BM_, BN_, MODE, KS>, grid, dim3(GTHREADS), 0, st, p); \
  }
  ILL_GEMM_CASE(128, 32) ILL_GEMM_CASE(64, 32) ILL_GEMM_CASE(32, 32)
  ILL_GEMM_CASE(128, 64) ILL_GEMM_CASE(64, 64) ILL_GEMM_CASE(32, 64)
  if (MODE == 1) { ILL_GEMM_CASE(128, 128) ILL_GEMM_CASE(64, 128) ILL_GEMM_CASE(32, 128) }
#undef ILL_GEMM_CASE
  return cudaErrorInvalidConfiguration;
}

template <typename T>
static cudaError_t gemm_t(const GemmOp &op, cudaStream_t st) {
  GemmParams p;
  p.src = op.src, p.w = op.w, p.bias = op.bias, p.res = op.res, p.dst = op.dst;
  p.dw_w = op.dw_w, p.dw_b = op.dw_b, p.coarse = op.coarse;
  p.M = op.M, p.N = op.N, p.K = op.K, p.act = op.act, p.mid_act = op.mid_act;
  p.H = op.H, p.W = op.W, p.OH = op.OH, p.OW = op.OW, p.stride = op.stride;
  if (p.M <= 0) return cudaSuccess;
  if (op.mode == 0) return launch_gemm_t<T, 0, 1>(p, st);
  if (op.mode == 2) return launch_gemm_t<T, 2, 1>(p, st);
  if (op.ks == 3) return launch_gemm_t<T, 1, 3>(p, st);
  if (op.ks == 5) return launch_gemm_t<T, 1, 5>(p, st);
  return cudaErrorInvalidValue;
}

cudaError_t gemm(int T, const GemmOp &op, cudaStream_t st) {
  return T == F32 ? gemm_t<float>(op, st) : gemm_t<__nv_bfloat16>(op, st);
}

// ---------------------------------------------------------------------------
// head (io.ts:141-166): sigmoid(b + w . x)
// ---------------------------------------------------------------------------

template <typename T>
__global__ void k_head(const T *__restrict__ src, long M, int C, const float *__restrict__ w, float bias,
                       float *__restrict__ dst1, float *__restrict__ dst4) {
  pdl_wait();
  pdl_trigger();
  long m = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  float s = bias;
  const T *x = src + m * C;
  for (int c = 0; c < C; c += 4) {
    float4 v = Io<T>::load4(x + c);
    float4 q = __ldg(reinterpret_cast<const float4 *>(w + c));
    s = fmaf(v.x, q.x, s);
    s = fmaf(v.y, q.y, s);
    s = fmaf(v.z, q.z, s);
    s = fmaf(v.w, q.w, s);
  }
  float d = 1.0f / (1.0f + expf(-s));
  if (dst1) dst1[m] = d;
  if (dst4) reinterpret_cast<float4 *>(dst4)[m] = make_float4(d, d, d, d);
}

cudaError_t head(int T, const void *src, long M, int C, const float *w, float bias, float *dst1, float *dst4,
                 cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (T == F32)
    return launch_pdl(k_head<float>, dim3(blocks_for(M, 256)), dim3(256), 0, st, (const float *)src, M, C, w, bias,
                      dst1, dst4);
  return launch_pdl(k_head<__nv_bfloat16>, dim3(blocks_for(M, 256)), dim3(256), 0, st, (const __nv_bfloat16 *)src, M, C,
                    w, bias, dst1, dst4);
}

// ---------------------------------------------------------------------------
// joint-bilateral upsample + temporal blend (io.ts:203-283)
// ---------------------------------------------------------------------------

// low: (n, lh, lw) with channel stride lc; guide luma either precomputed
// (luma, 1 channel) or from linear colour (guide, gc channels).
// Parameter list mirrored by kBilateralArgCount / kBilateralDstArg.
//
// Output (x, y) centres its 3x3 low-res taps on (floor((x + 0.5) / 2),
// floor((y + 0.5) / 2)), the same low pixel for the four pixels of a 2x2
// quad. A CTA covers 32 x 8 quads (64 x 16 output pixels): the (8 + 2) x
// (32 + 2) low-res disparities and guide samples its taps read, clamped to
// the map as the reference's taps are, are staged once in shared memory; each
// thread then runs its quad's four pixels. Per tap the weight
// spatial * exp(-dl^2 / 2) is one hardware exp2 of the summed log2 terms,
// log2(spatial) - (here - there)^2 * log2(e) / (2 sigma^2): the interior
// quads' 36 spatial terms are compile-time constants (the tap offsets are
// +-1/4, +-3/4, +-5/4 wherever the quad is), border quads compute theirs from
// the clamped tap positions. The normalising division is the SFU reciprocal
// product (within WGSL's 2.5 ulp division accuracy).
constexpr int kBilTX = 32, kBilTY = 8;
constexpr float kLog2e = 1.44269504088896340736f;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// log2 of the spatial weight of tap (dx, dy) for quad sub-pixel `sub` of an
// interior quad: offsets (dx - sx/2 + 1/4, dy - sy/2 + 1/4), exact in binary32.
__host__ __device__ constexpr float bil_sp2(int sub, int k) {
  return -(((float)(k % 3 - 1) - ((float)(sub & 1) * 0.5f - 0.25f)) *
               ((float)(k % 3 - 1) - ((float)(sub & 1) * 0.5f - 0.25f)) +
           ((float)(k / 3 - 1) - ((float)(sub >> 1) * 0.5f - 0.25f)) *
               ((float)(k / 3 - 1) - ((float)(sub >> 1) * 0.5f - 0.25f))) *
         0.5f * kLog2e;
}

__global__ void __launch_bounds__(kBilTX * kBilTY) k_bilateral(const float *__restrict__ low, int lc, int n, int lh,
                                                             int lw, const float *__restrict__ luma,
                                                             const float *__restrict__ guide, int gc,
                                                             BilateralParams p, float *__restrict__ dst,
                                                             const float *__restrict__ history,
                                                             float *__restrict__ out_tex) {
  pdl_wait();
  pdl_trigger();
  __shared__ float s_disp[kBilTY + 2][kBilTX + 2];
  __shared__ float s_there[kBilTY + 2][kBilTX + 2];
  const int S = lh * 2, SW = lw * 2;
  const int b = blockIdx.z;
  const int qi0 = blockIdx.x * kBilTX, qj0 = blockIdx.y * kBilTY;
  auto luma_at = [&](int gx, int gy) -> float {
    const int g = (b * S + gy) * SW + gx;
    if (luma) return __ldg(luma + g);
    const float *c = guide + (long)g * gc;
    return 0.2126f * __ldg(c) + 0.7152f * __ldg(c + 1) + 0.0722f * __ldg(c + 2);
  };
  const int tid = threadIdx.y * kBilTX + threadIdx.x;
  for (int e = tid; e < (kBilTY + 2) * (kBilTX + 2); e += kBilTX * kBilTY) {
    const int ey = e / (kBilTX + 2), ex = e - ey * (kBilTX + 2);
    const int qx = min(max(qi0 + ex - 1, 0), lw - 1), qy = min(max(qj0 + ey - 1, 0), lh - 1);
    s_disp[ey][ex] = __ldg(low + ((b * lh + qy) * lw + qx) * lc);
    s_there[ey][ex] = luma_at(qx * 2, qy * 2);
  }
  __syncthreads();
  const int qi = qi0 + threadIdx.x, qj = qj0 + threadIdx.y;
  if (qi >= lw || qj >= lh) return;
  const int tx = threadIdx.x, ty = threadIdx.y;
  float disp[9], there[9];
#pragma unroll
  for (int k = 0; k < 9; k++) {
    disp[k] = s_disp[ty + k / 3][tx + k % 3];
    there[k] = s_there[ty + k / 3][tx + k % 3];
  }
  // the four guide values of the quad's own pixels (row pairs as float2 when aligned)
  float here[4];
  const int g0 = (b * S + 2 * qj) * SW + 2 * qi;
  if (luma && ((reinterpret_cast<uintptr_t>(luma) & 7) == 0)) {
    const float2 h0 = __ldg(reinterpret_cast<const float2 *>(luma + g0));
    const float2 h1 = __ldg(reinterpret_cast<const float2 *>(luma + g0 + SW));
    here[0] = h0.x, here[1] = h0.y, here[2] = h1.x, here[3] = h1.y;
  } else {
#pragma unroll
    for (int sub = 0; sub < 4; sub++) here[sub] = luma_at(2 * qi + (sub & 1), 2 * qj + (sub >> 1));
  }
  const bool interior = qi >= 1 && qj >= 1 && qi + 1 < lw && qj + 1 < lh;
  const float inv = 1.0f / fmaxf(p.range_sigma, 1e-4f);
  const float k2 = inv * inv * (0.5f * kLog2e);
  float out[4];
#pragma unroll
  for (int sub = 0; sub < 4; sub++) {
    const int x = 2 * qi + (sub & 1), y = 2 * qj + (sub >> 1);
    float sp2[9];
    if (interior) {
#pragma unroll
      for (int k = 0; k < 9; k++) sp2[k] = bil_sp2(sub, k);
    } else {
      const float cx = (x + 0.5f) * 0.5f - 0.5f, cy = (y + 0.5f) * 0.5f - 0.5f;
#pragma unroll
      for (int k = 0; k < 9; k++) {
        const float dxs = (float)min(max(qi + k % 3 - 1, 0), lw - 1) - cx;
        const float dys = (float)min(max(qj + k / 3 - 1, 0), lh - 1) - cy;
        sp2[k] = -(dxs * dxs + dys * dys) * (0.5f * kLog2e);
      }
    }
    float weighted = 0.0f, total_w = 0.0f;
#pragma unroll
    for (int k = 0; k < 9; k++) {
      const float d = here[sub] - there[k];
      const float wgt = ex2_approx(fmaf(-d * d, k2, sp2[k]));
      weighted = fmaf(disp[k], wgt, weighted);
      total_w += wgt;
    }
    const float up = __fdividef(weighted, fmaxf(total_w, 1e-6f));
    float o = up;
    if (out_tex) {
      const int idx = (b * S + y) * SW + x;
      const float4 prev = history ? reinterpret_cast<const float4 *>(history)[idx] : make_float4(0, 0, 0, 0);
      const float change = fabsf(up - prev.x);
      const float alpha =
          prev.w < 0.5f ? 1.0f : fminf(fmaxf(p.base_alpha + change * p.sensitivity, p.base_alpha), 1.0f);
      o = prev.x + (up - prev.x) * alpha;
      reinterpret_cast<float4 *>(out_tex)[idx] = make_float4(o, up, change, 1.0f);
    }
    out[sub] = o;
  }
  if (dst) {  // paired stores when the caller's pointer allows, scalar otherwise
    if ((reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
      reinterpret_cast<float2 *>(dst + g0)[0] = make_float2(out[0], out[1]);
      reinterpret_cast<float2 *>(dst + g0 + SW)[0] = make_float2(out[2], out[3]);
    } else {
      dst[g0] = out[0], dst[g0 + 1] = out[1];
      dst[g0 + SW] = out[2], dst[g0 + SW + 1] = out[3];
    }
  }
}

namespace {
dim3 bilateral_grid(int n, int lh, int lw) { return dim3((lw + kBilTX - 1) / kBilTX, (lh + kBilTY - 1) / kBilTY, n); }
}  // namespace

cudaError_t bilateral(const float *low1, int n, int lh, int lw, const float *luma, const BilateralParams &p,
                      float *dst, const float *history, float *out_tex, cudaStream_t st) {
  long total = (long)n * lh * lw * 4;
  if (total > kMaxIndex || n > 65535) return cudaErrorInvalidValue;
  if (total == 0) return cudaSuccess;
  return launch_pdl(k_bilateral, bilateral_grid(n, lh, lw), dim3(kBilTX, kBilTY), 0, st, low1, 1, n, lh, lw, luma,
                    (const float *)nullptr, 0, p, dst, history, out_tex);
}

cudaError_t bilateral_strided(const float *low, int lh, int lw, int low_c, const float *guide, int guide_c,
                              float range_sigma, float *dst, cudaStream_t st) {
  long total = (long)lh * lw * 4;
  if (total > kMaxIndex) return cudaErrorInvalidValue;
  if (total == 0) return cudaSuccess;
  BilateralParams p{range_sigma, 0.35f, 3.0f};
  k_bilateral<<<bilateral_grid(1, lh, lw), dim3(kBilTX, kBilTY), 0, st>>>(low, low_c, 1, lh, lw, nullptr, guide,
                                                                          guide_c, p, dst, nullptr, nullptr);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// weight packing
// ---------------------------------------------------------------------------

__device__ __forceinline__ float maybe_bf16(float v, int r) {
  return r ? __bfloat162float(__float2bfloat16_rn(v)) : v;
}

// [C][k][k] -> [k*k][C]
__global__ void k_pack_dw(const float *w, int C, int k, float *out, int r) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  int kk = k * k;
  if (i >= C * kk) return;
  int c = i / kk, t = i % kk;
  out[t * C + c] = maybe_bf16(w[i], r);
}

// [O][I][k][k] -> [k][k][I][O]
__global__ void k_pack_conv(const float *w, int O, int I, int k, float *out, int r) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  int total = O * I * k * k;
  if (i >= total) return;
  int kx = i % k, ky = (i / k) % k, ic = (i / (k * k)) % I, oc = i / (k * k * I);
  out[((ky * k + kx) * I + ic) * O + oc] = maybe_bf16(w[i], r);
}

__global__ void k_copy_round(const float *w, long n, float *out, int r) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = maybe_bf16(w[i], r);
}

cudaError_t pack_dw(const float *w, int C, int k, float *out, int r, cudaStream_t st) {
  k_pack_dw<<<blocks_for((long)C * k * k, 256), 256, 0, st>>>(w, C, k, out, r);
  return cudaGetLastError();
}
cudaError_t pack_conv(const float *w, int O, int I, int k, float *out, int r, cudaStream_t st) {
  k_pack_conv<<<blocks_for((long)O * I * k * k, 256), 256, 0, st>>>(w, O, I, k, out, r);
  return cudaGetLastError();
}
cudaError_t copy_round(const float *w, long n, float *out, int r, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_copy_round<<<blocks_for(n, 256), 256, 0, st>>>(w, n, out, r);
  return cudaGetLastError();
}

__global__ void k_expand4(const float *src, long n, float *dst4) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    float v = src[i];
    reinterpret_cast<float4 *>(dst4)[i] = make_float4(v, v, v, v);
  }
}
cudaError_t expand4(const float *src, long n, float *dst4, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_expand4<<<blocks_for(n, 256), 256, 0, st>>>(src, n, dst4);
  return cudaGetLastError();
}

__global__ void k_bf16_to_f32(const __nv_bfloat16 *src, long n, float *dst) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = __bfloat162float(src[i]);
}
cudaError_t to_f32(int T, const void *src, long n, float *dst, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (T == F32) return cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, st);
  k_bf16_to_f32<<<blocks_for(n, 256), 256, 0, st>>>((const __nv_bfloat16 *)src, n, dst);
  return cudaGetLastError();
}

// Luminance guide of a given network input: its channel 3 (the unnormalised
// luminance the preprocess stores there, equal to the guide it writes).
__global__ void k_input_luma(const float4 *__restrict__ input, long px, float *__restrict__ luma) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < px) luma[i] = input[i].w;
}

cudaError_t input_luma(const float *input, long px, float *luma, cudaStream_t st) {
  if (px <= 0) return cudaSuccess;
  k_input_luma<<<blocks_for(px, 256), 256, 0, st>>>(reinterpret_cast<const float4 *>(input), px, luma);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// synthetic frames and checksums
// ---------------------------------------------------------------------------

// mulberry32 output for absolute draw index j (0-based) of the stream seeded
// with `seed`: the state after j+1 increments is seed + (j+1)*0x6d2b79f5.
__device__ __forceinline__ double mb32_at(uint32_t seed, uint32_t j) {
  uint32_t t = seed + (j + 1u) * 0x6d2b79f5u;
  t = (t ^ (t >> 15)) * (t | 1u);
  t ^= t + (t ^ (t >> 7)) * (t | 61u);
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

__global__ void k_gen_uniform(uint32_t seed0, int n, int S, float *out) {
  long per = 3L * S * S;
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= per * n) return;
  int f = (int)(i / per);
  uint32_t j = (uint32_t)(i - (long)f * per);
  out[i] = (float)mb32_at(seed0 + (uint32_t)f, j);
}

// Blob frames (smooth procedural images): per frame seed and channel c,
// 8 anisotropic Gaussian blobs from draws (c*8 + b)*6 .. +5 of the frame's
// mulberry32 stream -- centre (u0*S, u1*S), sigma_x = 20 + 100*u2,
// sigma_y = 20 + 100*u3 pixels, rotation u4*pi, amplitude u5 -- summed at
// the pixel centre, plus N(0, 0.02) Box-Muller noise on draws 144 + 2j and
// 145 + 2j (j = the value's (c, y, x) index, u clamped to 1e-9), clamped to
// [0, 1]. Every step is an IEEE double add, multiply, divide, square root or
// fused multiply-add with round-to-nearest in a fixed order (the intrinsics
// below are never contracted or reassociated), and exp / log / sin / cos are
// written out from their series: exp by Cody-Waite reduction with ln 2 split
// in two and the Taylor series to r^13/13!; log by the atanh series
// log m = 2 atanh((m-1)/(m+1)) on m in [sqrt(1/2), sqrt(2)]; sin and cos by
// their Taylor series on [-pi/2, pi/2]. A host evaluation of the same
// operations therefore gives the same bits, and the functions are within a
// few ulp of the exact ones.
namespace detm {

__device__ __constant__ double kExpC[12] = {0.5, 0.16666666666666666, 0.041666666666666664, 0.008333333333333333,
                                            0.001388888888888889, 0.0001984126984126984, 2.48015873015873e-05,
                                            2.7557319223985893e-06, 2.755731922398589e-07, 2.505210838544172e-08,
                                            2.08767569878681e-09, 1.6059043836821613e-10};
__device__ __constant__ double kLogC[12] = {0.3333333333333333, 0.2, 0.14285714285714285, 0.1111111111111111,
                                            0.09090909090909091, 0.07692307692307693, 0.06666666666666667,
                                            0.058823529411764705, 0.05263157894736842, 0.047619047619047616,
                                            0.043478260869565216, 0.04};
__device__ __constant__ double kCosC[12] = {-0.5, 0.041666666666666664, -0.001388888888888889, 2.48015873015873e-05,
                                            -2.755731922398589e-07, 2.08767569878681e-09, -1.1470745597729725e-11,
                                            4.779477332387385e-14, -1.5619206968586225e-16, 4.110317623312165e-19,
                                            -8.896791392450574e-22, 1.6117375710961184e-24};
__device__ __constant__ double kSinC[11] = {-0.16666666666666666, 0.008333333333333333, -0.0001984126984126984,
                                            2.7557319223985893e-06, -2.505210838544172e-08, 1.6059043836821613e-10,
                                            -7.647163731819816e-13, 2.8114572543455206e-15, -8.22063524662433e-18,
                                            1.9572941063391263e-20, -3.868170170630684e-23};
constexpr double kLn2Hi = 0.6931471803691238;  // 0x1.62e42feep-1: k * hi is exact
constexpr double kLn2Lo = 1.9082149292705877e-10;
constexpr double kInvLn2 = 1.4426950408889634;
constexpr double kPi = 3.141592653589793;
constexpr double kPiHalf = 1.5707963267948966;
constexpr double kTwoPi = 6.283185307179586;
constexpr double kSqrt2 = 1.4142135623730951;

// exp(x) for x <= 0 (0 below -708)
__device__ double exp_neg(double x) {
  if (x < -708.0) return 0.0;
  const double kd = floor(__fma_rn(x, kInvLn2, 0.5));
  double r = __fma_rn(-kd, kLn2Hi, x);
  r = __fma_rn(-kd, kLn2Lo, r);
  double p = kExpC[11];
#pragma unroll
  for (int i = 10; i >= 0; i--) p = __fma_rn(p, r, kExpC[i]);
  p = __fma_rn(p, r, 1.0);
  p = __fma_rn(p, r, 1.0);
  return __dmul_rn(p, __longlong_as_double((long long)((int)kd + 1023) << 52));
}

// log(u) for normal u > 0
__device__ double log_pos(double u) {
  unsigned long long b = (unsigned long long)__double_as_longlong(u);
  int e = (int)((b >> 52) & 0x7ff) - 1023;
  double m = __longlong_as_double((long long)((b & 0x000fffffffffffffull) | 0x3ff0000000000000ull));
  if (m > kSqrt2) {
    m = __dmul_rn(m, 0.5);
    e += 1;
  }
  const double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
  const double z = __dmul_rn(s, s);
  double p = kLogC[11];
#pragma unroll
  for (int i = 10; i >= 0; i--) p = __fma_rn(p, z, kLogC[i]);
  p = __fma_rn(p, z, 1.0);
  const double lm = __dmul_rn(__dadd_rn(s, s), p);
  const double ed = (double)e;
  return __fma_rn(ed, kLn2Hi, __fma_rn(ed, kLn2Lo, lm));
}

__device__ double cos_poly(double t) {  // |t| <= pi/2
  const double z = __dmul_rn(t, t);
  double p = kCosC[11];
#pragma unroll
  for (int i = 10; i >= 0; i--) p = __fma_rn(p, z, kCosC[i]);
  return __fma_rn(p, z, 1.0);
}

__device__ double sin_poly(double t) {  // |t| <= pi/2
  const double z = __dmul_rn(t, t);
  double p = kSinC[10];
#pragma unroll
  for (int i = 9; i >= 0; i--) p = __fma_rn(p, z, kSinC[i]);
  p = __fma_rn(p, z, 1.0);
  return __dmul_rn(t, p);
}

// cos(2 pi v), v in [0, 1) a multiple of 2^-32 (the reductions are exact)
__device__ double cos2pi(double v) {
  const double a = fabs(__dsub_rn(v, floor(__dadd_rn(v, 0.5))));
  if (a <= 0.25) return cos_poly(__dmul_rn(a, kTwoPi));
  return -cos_poly(__dmul_rn(__dsub_rn(0.5, a), kTwoPi));
}

}  // namespace detm

struct BlobParams {
  double cx, cy, hx, hy, cs, sn, amp;
};

// grid (ceil(S*S / 256), 3 channels, n frames); 256 threads, one value each
__global__ void __launch_bounds__(256) k_gen_blobs(uint32_t seed0, int S, float *out) {
  __shared__ BlobParams bl[8];
  const int c = blockIdx.y, f = blockIdx.z;
  const uint32_t seed = seed0 + (uint32_t)f;
  if (threadIdx.x < 8) {
    const int b = threadIdx.x;
    const uint32_t d = (uint32_t)((c * 8 + b) * 6);
    BlobParams o;
    o.cx = __dmul_rn(mb32_at(seed, d), (double)S);
    o.cy = __dmul_rn(mb32_at(seed, d + 1), (double)S);
    const double sx = __fma_rn(mb32_at(seed, d + 2), 100.0, 20.0);
    const double sy = __fma_rn(mb32_at(seed, d + 3), 100.0, 20.0);
    o.hx = __ddiv_rn(0.5, __dmul_rn(sx, sx));
    o.hy = __ddiv_rn(0.5, __dmul_rn(sy, sy));
    const double t = __dsub_rn(__dmul_rn(mb32_at(seed, d + 4), detm::kPi), detm::kPiHalf);  // theta - pi/2
    o.cs = -detm::sin_poly(t);
    o.sn = detm::cos_poly(t);
    o.amp = mb32_at(seed, d + 5);
    bl[b] = o;
  }
  __syncthreads();
  const long plane = (long)S * S;
  const long pix = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= plane) return;
  const int y = (int)(pix / S), x = (int)(pix - (long)y * S);
  const double px = (double)x + 0.5, py = (double)y + 0.5;
  double v = 0.0;
#pragma unroll 1
  for (int b = 0; b < 8; b++) {
    const BlobParams B = bl[b];
    const double dx = __dsub_rn(px, B.cx), dy = __dsub_rn(py, B.cy);
    const double u = __fma_rn(B.cs, dx, __dmul_rn(B.sn, dy));
    const double w = __fma_rn(B.cs, dy, -__dmul_rn(B.sn, dx));
    const double q = __fma_rn(__dmul_rn(u, u), B.hx, __dmul_rn(__dmul_rn(w, w), B.hy));
    v = __fma_rn(B.amp, detm::exp_neg(-q), v);
  }
  const long j = (long)c * plane + pix;
  const uint32_t nd = 144u + 2u * (uint32_t)j;
  double uu = mb32_at(seed, nd);
  if (uu < 1e-9) uu = 1e-9;
  const double g = __dmul_rn(__dsqrt_rn(__dmul_rn(-2.0, detm::log_pos(uu))), detm::cos2pi(mb32_at(seed, nd + 1)));
  v = __fma_rn(0.02, g, v);
  v = v < 0.0 ? 0.0 : (v > 1.0 ? 1.0 : v);
  out[(long)f * 3 * plane + j] = __double2float_rn(v);
}

cudaError_t generate_frames(int kind, uint32_t seed0, int n, int S, float *out, cudaStream_t st) {
  long total = 3L * S * S * n;
  if (total == 0) return cudaSuccess;
  if (kind == 0) k_gen_uniform<<<blocks_for(total, 256), 256, 0, st>>>(seed0, n, S, out);
  else {
    if (n > 65535) return cudaErrorInvalidValue;
    k_gen_blobs<<<dim3(blocks_for((long)S * S, 256), 3, (unsigned)n), 256, 0, st>>>(seed0, S, out);
  }
  return cudaGetLastError();
}

__global__ void k_checksums(const float *maps, long count, unsigned long long *sum64, double *fsum) {
  int f = blockIdx.y;
  const uint32_t *bits = reinterpret_cast<const uint32_t *>(maps + (long)f * count);
  const float *vals = maps + (long)f * count;
  unsigned long long h = 0;
  double s = 0.0;
  for (long j = (long)blockIdx.x * blockDim.x + threadIdx.x; j < count; j += (long)gridDim.x * blockDim.x) {
    h += (unsigned long long)bits[j] * (unsigned long long)(2 * j + 1);
    s += (double)vals[j];
  }
  for (int o = 16; o > 0; o >>= 1) {
    h += __shfl_down_sync(0xffffffffu, h, o);
    s += __shfl_down_sync(0xffffffffu, s, o);
  }
  __shared__ unsigned long long hs[32];
  __shared__ double ss[32];
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) hs[wid] = h, ss[wid] = s;
  __syncthreads();
  if (wid == 0) {
    int nw = blockDim.x >> 5;
    h = lane < nw ? hs[lane] : 0ull;
    s = lane < nw ? ss[lane] : 0.0;
    for (int o = 16; o > 0; o >>= 1) {
      h += __shfl_down_sync(0xffffffffu, h, o);
      s += __shfl_down_sync(0xffffffffu, s, o);
    }
    if (lane == 0) {
      atomicAdd(sum64 + f, h);
      atomicAdd(fsum + f, s);
    }
  }
}

cudaError_t checksums(const float *maps, int n, long count, uint64_t *sum64, double *fsum, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  cudaError_t e = cudaMemsetAsync(sum64, 0, sizeof(uint64_t) * n, st);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(fsum, 0, sizeof(double) * n, st);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((count + 255) / 256 < 64 ? (count + 255) / 256 : 64), n);
  if (grid.x == 0) grid.x = 1;
  k_checksums<<<grid, 256, 0, st>>>(maps, count, (unsigned long long *)sum64, fsum);
  return cudaGetLastError();
}

}  // namespace gpu
}  // namespace illumina
