// Tensor-core (tcgen05 / TMEM) kernel for the pointwise-shaped ops:
// pointwise, depthwise -> pointwise, and the FPN lateral.
//
// One CTA owns a tile of 128 output pixels (one UMMA M=128 row block) x up to
// 256 output channels (the accumulator: 128 TMEM lanes x N columns of fp32).
// The input channels are walked in slabs of 128 bytes per pixel row (32 fp32
// / 64 bf16 channels), double-buffered in shared memory:
//
//   all 8 warps      produce the A slab: plain loads (pw), the depthwise k x k
//                    + bias + activation (dw->pw), or the skip tensor
//                    (lateral), written in the UMMA canonical K-major
//                    128-byte-swizzle layout; and copy the B slab (weights,
//                    pre-swizzled on the host into the same image);
//   thread 0         issues tcgen05.mma for the slab and tcgen05.commit's to
//                    the slab buffer's mbarrier, so producers of slab s+2 wait
//                    only for the MMAs that read that buffer;
//   epilogue         tcgen05.ld of the accumulator, + bias, + residual or the
//                    bilinear-upsampled coarse tensor, activation, store.
//
// fp32 storage uses three TF32 products per slab (a_hi b_hi + a_hi b_lo +
// a_lo b_hi, with x = hi + lo split at production), which keeps products to
// ~2^-22 relative, the accuracy class of FFMA. bf16 storage uses kind::f16
// with fp32 accumulation.
//
// Every wait on an mbarrier is bounded (~2^31 cycles); on expiry the kernel
// records an error code in *err, skips the remaining work and still releases
// its TMEM.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace illumina {
namespace gpu {

namespace tc {

constexpr int kThreads = 256;
constexpr int kTileM = 128;
constexpr int kRowBytes = 128;  // one swizzle atom row: 128 bytes of K per pixel
constexpr long long kWaitCycles = 1ll << 31;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of `bar`; false when the bound expires.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return true;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// packed 1024 bytes apart (SBO), LBO unused (1), version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: D fp32, A/B format (1 bf16, 2 tf32), both K-major,
// M = 128, N = n.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t ab_format, uint32_t n) {
  return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((n >> 3) << 17) | ((uint32_t)(kTileM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 8 consecutive fp32 columns per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float v[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ float act_apply(int act, float v) {
  switch (act) {
    case 1: return fmaxf(v, 0.0f);
    case 2: return fminf(fmaxf(v, 0.0f), 6.0f);
    case 3: return (v * fminf(fmaxf(v + 3.0f, 0.0f), 6.0f)) / 6.0f;
    default: return v;
  }
}

__device__ __forceinline__ float4 ld4(const float *p) { return __ldg(reinterpret_cast<const float4 *>(p)); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16 *p) {
  uint2 r = __ldg(reinterpret_cast<const uint2 *>(p));
  float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162 *>(&r.x));
  float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162 *>(&r.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
__device__ __forceinline__ void st4(__nv_bfloat16 *p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 r;
  r.x = *reinterpret_cast<uint32_t *>(&a);
  r.y = *reinterpret_cast<uint32_t *>(&b);
  *reinterpret_cast<uint2 *>(p) = r;
}
__device__ __forceinline__ float4 f4fma(float4 a, float4 b, float4 c) {
  return make_float4(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y), fmaf(a.z, b.z, c.z), fmaf(a.w, b.w, c.w));
}

struct Params {
  const void *src;      // A source: pw/lateral [M][K]; dw (n, H, W, K)
  const uint8_t *wimg;  // B images: [n_tile][slab][term][n_tile_cols x 128 B]
  const float *bias;    // [N]
  const void *res;      // [M][N] or null
  const void *coarse;   // lateral: (n, OH/2, OW/2, N)
  void *dst;            // [M][N]
  const float *dw_w;    // packed [ks*ks][K]
  const float *dw_b;    // [K]
  int *err;             // error flag (nullable)
  long M;
  int N, K, act, mid_act;
  int H, W, OH, OW, stride;
  int n_tile;           // accumulator columns per CTA (multiple of 16, <= 256)
  int slabs;            // ceil(K / channels per slab)
  uint32_t tmem_cols;   // power of two >= n_tile
};

// Byte offset of 16-byte chunk `c` of row `r` inside a swizzled 8-row-atom image.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// MODE 0 pointwise, 1 depthwise (KS x KS) -> pointwise, 2 lateral.
template <typename T, int MODE, int KS>
__global__ void __launch_bounds__(kThreads, 1) k_tc_gemm(const Params p) {
  constexpr bool kF32 = sizeof(T) == 4;
  constexpr int kTerms = kF32 ? 2 : 1;          // hi/lo images per operand
  constexpr int kSlabC = kRowBytes / sizeof(T); // channels per slab: 32 (fp32) or 64 (bf16)
  constexpr int kChunkC = 16 / sizeof(T);       // channels per 16-byte chunk: 4 or 8
  constexpr int kChunks = kTileM * 8;           // 16-byte chunks in one A image
  constexpr uint32_t kAImage = kTileM * kRowBytes;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base_s = (raw + 1023u) & ~1023u;
  uint8_t *base = smem_raw + (base_s - raw);
  const uint32_t b_image = (uint32_t)p.n_tile * kRowBytes;
  const uint32_t stage_bytes = kTerms * kAImage + kTerms * b_image;
  uint64_t *mbar = reinterpret_cast<uint64_t *>(base + 2 * stage_bytes);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(base + 2 * stage_bytes + 16);

  const int tid = threadIdx.x, warp = tid >> 5;
  const long m0 = (long)blockIdx.x * kTileM;
  const int n0 = blockIdx.y * p.n_tile;
  const int K4 = p.K >> 2;

  if (tid == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
  }
  if (warp == 0) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  // Per-thread A chunks: row r = q / 8, chunk c = q % 8, q = tid + i * 256.
  constexpr int kPer = kChunks / kThreads;  // 4

  const T *src = reinterpret_cast<const T *>(p.src);
  const uint32_t idesc = instr_desc(kF32 ? 2u : 1u, (uint32_t)p.n_tile);

  for (int s = 0; s < p.slabs; s++) {
    const int buf = s & 1;
    if (s >= 2) {
      // every thread waits (bounded); the CTA agrees on the outcome
      const bool w = mbar_wait(&mbar[buf], (uint32_t)(((s - 2) >> 1) & 1));
      if (!__syncthreads_and(w)) {
        ok = false;
        break;
      }
    }
    uint8_t *st = base + buf * stage_bytes;
    const int c0 = s * kSlabC;  // first channel of the slab

    // ---- A: 128 rows x kSlabC channels ----
#pragma unroll(MODE == 1 ? 1 : kPer)
    for (int i = 0; i < kPer; i++) {
      const int q = tid + i * kThreads;
      const int r = q >> 3, c = q & 7;
      const long m = m0 + r;
      int rb = 0, ry = 0, rx = 0;
      if (MODE == 1 && m < p.M) {
        rx = (int)(m % p.OW);
        const long t = m / p.OW;
        ry = (int)(t % p.OH);
        rb = (int)(t / p.OH);
      }
      const int ch = c0 + c * kChunkC;  // first channel of this chunk
      float v[kChunkC];
#pragma unroll
      for (int j = 0; j < kChunkC; j++) v[j] = 0.0f;
      if (m < p.M) {
#pragma unroll
        for (int h = 0; h < kChunkC / 4; h++) {
          const int cq = (ch >> 2) + h;  // float4 group index
          if (cq >= K4) continue;
          float4 a;
          if (MODE != 1) {
            a = ld4(src + (m0 + r) * p.K + cq * 4);
          } else {
            constexpr int pad = (KS - 1) / 2;
            a = __ldg(reinterpret_cast<const float4 *>(p.dw_b) + cq);
#pragma unroll
            for (int ky = 0; ky < KS; ky++) {
              const int iy = ry * p.stride + ky - pad;
              if (iy < 0 || iy >= p.H) continue;
              const T *row = src + ((long)rb * p.H + iy) * p.W * p.K;
#pragma unroll
              for (int kx = 0; kx < KS; kx++) {
                const int ix = rx * p.stride + kx - pad;
                if (ix < 0 || ix >= p.W) continue;
                a = f4fma(ld4(row + (long)ix * p.K + cq * 4),
                          __ldg(reinterpret_cast<const float4 *>(p.dw_w) + (long)(ky * KS + kx) * K4 + cq), a);
              }
            }
            a = make_float4(act_apply(p.mid_act, a.x), act_apply(p.mid_act, a.y), act_apply(p.mid_act, a.z),
                            act_apply(p.mid_act, a.w));
          }
          v[h * 4 + 0] = a.x, v[h * 4 + 1] = a.y, v[h * 4 + 2] = a.z, v[h * 4 + 3] = a.w;
        }
      }
      const uint32_t off = swz(r, c);
      if (kF32) {
        uint4 hi, lo;
        uint32_t *ph = &hi.x, *pl = &lo.x;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          ph[j] = tf32_rna(v[j]);
          pl[j] = tf32_rna(v[j] - __uint_as_float(ph[j]));
        }
        *reinterpret_cast<uint4 *>(st + off) = hi;
        *reinterpret_cast<uint4 *>(st + kAImage + off) = lo;
      } else {
        uint4 pk;
        uint32_t *pp = &pk.x;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
          pp[j] = *reinterpret_cast<uint32_t *>(&b2);
        }
        *reinterpret_cast<uint4 *>(st + off) = pk;
      }
    }
    // ---- B: pre-swizzled weight images for (n tile, slab) ----
    {
      const uint4 *g = reinterpret_cast<const uint4 *>(p.wimg + ((size_t)blockIdx.y * p.slabs + s) * kTerms * b_image);
      uint4 *d = reinterpret_cast<uint4 *>(st + kTerms * kAImage);
      const int n16 = (int)(kTerms * b_image / 16);
      for (int q = tid; q < n16; q += kThreads) d[q] = __ldg(g + q);
    }
    fence_async_smem();
    __syncthreads();

    if (tid == 0) {
      tc_fence_after();
      const uint32_t sa = base_s + buf * stage_bytes;
      const uint32_t sb = sa + kTerms * kAImage;
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {  // 4 MMAs of K = 32 bytes per 128-byte slab row
        const uint32_t ko = kk * 32;
        if (kF32) {
          // small terms first: a_hi*b_lo, a_lo*b_hi, then a_hi*b_hi
          mma_tf32(tmem, smem_desc(sa + ko), smem_desc(sb + b_image + ko), idesc, (s | kk) ? 1u : 0u);
          mma_tf32(tmem, smem_desc(sa + kAImage + ko), smem_desc(sb + ko), idesc, 1u);
          mma_tf32(tmem, smem_desc(sa + ko), smem_desc(sb + ko), idesc, 1u);
        } else {
          mma_f16(tmem, smem_desc(sa + ko), smem_desc(sb + ko), idesc, (s | kk) ? 1u : 0u);
        }
      }
      mma_commit(&mbar[buf]);
    }
  }

  // ---- wait for the last slab's MMAs ----
  if (ok && p.slabs > 0) {
    const int s = p.slabs - 1;
    const bool w = mbar_wait(&mbar[s & 1], (uint32_t)((s >> 1) & 1));
    ok = __syncthreads_and(w);
  }
  if (!ok && p.err) atomicExch(p.err, 1);
  tc_fence_after();

  // ---- epilogue: warp w reads TMEM lanes 32*(w%4).., column half w/4 ----
  if (ok) {
    const int lane_base = (warp & 3) * 32;
    const int r = lane_base + (tid & 31);
    const long m = m0 + r;
    const int half = p.n_tile / 2;  // multiple of 8
    const int col0 = (warp >> 2) * half;
    const T *res = reinterpret_cast<const T *>(p.res);
    const T *coarse = reinterpret_cast<const T *>(p.coarse);
    T *dst = reinterpret_cast<T *>(p.dst);
    long cb00 = 0, cb01 = 0, cb10 = 0, cb11 = 0;
    float w00 = 0, w01 = 0, w10 = 0, w11 = 0;
    if (MODE == 2 && m < p.M) {
      // refUpsample2 taps (reference.ts:161-193)
      const int x = (int)(m % p.OW);
      const long t = m / p.OW;
      const int y = (int)(t % p.OH), b = (int)(t / p.OH);
      const int CH = p.OH >> 1, CW = p.OW >> 1;
      const float sy = (y + 0.5f) * 0.5f - 0.5f, sx = (x + 0.5f) * 0.5f - 0.5f;
      const float fy0 = floorf(sy), fx0 = floorf(sx), fy = sy - fy0, fx = sx - fx0;
      const int y0 = min(max((int)fy0, 0), CH - 1), y1 = min(max((int)fy0 + 1, 0), CH - 1);
      const int x0 = min(max((int)fx0, 0), CW - 1), x1 = min(max((int)fx0 + 1, 0), CW - 1);
      const long rb0 = ((long)b * CH + y0) * CW, rb1 = ((long)b * CH + y1) * CW;
      cb00 = (rb0 + x0) * p.N, cb01 = (rb0 + x1) * p.N, cb10 = (rb1 + x0) * p.N, cb11 = (rb1 + x1) * p.N;
      w00 = (1 - fx) * (1 - fy), w01 = fx * (1 - fy), w10 = (1 - fx) * fy, w11 = fx * fy;
    }
    for (int cc = 0; cc < half; cc += 8) {
      float v[8];
      tmem_ld8(tmem + ((uint32_t)lane_base << 16) + (uint32_t)(col0 + cc), v);
      if (m >= p.M) continue;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int n = n0 + col0 + cc + h * 4;
        if (n >= p.N) continue;
        float4 o = make_float4(v[h * 4] + __ldg(p.bias + n), v[h * 4 + 1] + __ldg(p.bias + n + 1),
                               v[h * 4 + 2] + __ldg(p.bias + n + 2), v[h * 4 + 3] + __ldg(p.bias + n + 3));
        if (MODE == 2) {
          const float4 a = ld4(coarse + cb00 + n), b = ld4(coarse + cb01 + n);
          const float4 c = ld4(coarse + cb10 + n), d = ld4(coarse + cb11 + n);
          o.x += a.x * w00 + b.x * w01 + c.x * w10 + d.x * w11;
          o.y += a.y * w00 + b.y * w01 + c.y * w10 + d.y * w11;
          o.z += a.z * w00 + b.z * w01 + c.z * w10 + d.z * w11;
          o.w += a.w * w00 + b.w * w01 + c.w * w10 + d.w * w11;
        }
        if (res) {
          const float4 q = ld4(res + m * p.N + n);
          o.x += q.x, o.y += q.y, o.z += q.z, o.w += q.w;
        }
        o = make_float4(act_apply(p.act, o.x), act_apply(p.act, o.y), act_apply(p.act, o.z), act_apply(p.act, o.w));
        st4(dst + m * p.N + n, o);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, p.tmem_cols);
}

}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

namespace {

// 2 stages x (2 A images + 2 B images of 256 rows) + alignment slack.
constexpr size_t kMaxSmem = 2 * (2 * 128 * 128 + 2 * 256 * 128) + 1024 + 64;

template <typename T, int MODE, int KS>
cudaError_t launch_t(const tc::Params &p, size_t smem, unsigned grid_x, unsigned grid_y, cudaStream_t st) {
  auto kern = tc::k_tc_gemm<T, MODE, KS>;
  // The largest tile's shared memory, granted once per device before first use.
  static unsigned long long granted = 0;  // bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !(granted & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    if (e != cudaSuccess) return e;
    granted |= 1ull << dev;
  }
  if (smem > kMaxSmem) return cudaErrorInvalidValue;
  kern<<<dim3(grid_x, grid_y), tc::kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

TcWeights tc_plan(int T, int N, int K) {
  TcWeights w;
  w.N = N, w.K = K;
  const int slab_c = T == F32 ? 32 : 64;
  w.slabs = (K + slab_c - 1) / slab_c;
  // at most 240 accumulator columns per tile: two fp32 ring stages of a wider
  // tile no longer fit beside the epilogue's shared-memory buffer
  int tiles = (N + 239) / 240;
  int per = (N + tiles - 1) / tiles;
  w.n_tile = (per + 15) / 16 * 16;
  w.n_tiles = (N + w.n_tile - 1) / w.n_tile;
  w.tmem_cols = 32;
  while ((int)w.tmem_cols < w.n_tile) w.tmem_cols <<= 1;
  const size_t terms = T == F32 ? 2 : 1;
  w.bytes = (size_t)w.n_tiles * w.slabs * terms * w.n_tile * 128;
  return w;
}

// [N][K] fp32 logical weights -> per (n tile, slab) swizzled images of
// n_tile rows x 128 bytes: tf32 hi and lo (fp32 storage) or bf16.
__global__ void k_tc_pack(const float *w, int N, int K, int n_tile, int n_tiles, int slabs, int is_f32,
                          uint8_t *out) {
  const int slab_c = is_f32 ? 32 : 64;
  const long total = (long)n_tiles * slabs * n_tile * slab_c;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int e = (int)(i % slab_c);
  long t = i / slab_c;
  const int r = (int)(t % n_tile);
  t /= n_tile;
  const int s = (int)(t % slabs);
  const int tile = (int)(t / slabs);
  const int n = tile * n_tile + r, k = s * slab_c + e;
  const float v = (n < N && k < K) ? w[(long)n * K + k] : 0.0f;
  const int terms = is_f32 ? 2 : 1;
  const size_t image = (size_t)n_tile * 128;
  const int byte = e * (is_f32 ? 4 : 2);
  const int c = byte >> 4, within = byte & 15;
  const size_t off = (size_t)(r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4) + within;
  uint8_t *img = out + ((size_t)(tile * slabs + s) * terms) * image;
  if (is_f32) {
    const uint32_t hi = tc::tf32_rna(v);
    const uint32_t lo = tc::tf32_rna(v - __uint_as_float(hi));
    *reinterpret_cast<uint32_t *>(img + off) = hi;
    *reinterpret_cast<uint32_t *>(img + image + off) = lo;
  } else {
    *reinterpret_cast<__nv_bfloat16 *>(img + off) = __float2bfloat16_rn(v);
  }
}

cudaError_t tc_pack(int T, const float *w, int N, int K, const TcWeights &plan, uint8_t *out, cudaStream_t st) {
  const long total = (long)plan.n_tiles * plan.slabs * plan.n_tile * (T == F32 ? 32 : 64);
  if (total <= 0) return cudaSuccess;
  k_tc_pack<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(w, N, K, plan.n_tile, plan.n_tiles, plan.slabs,
                                                             T == F32 ? 1 : 0, out);
  return cudaGetLastError();
}

size_t tc_smem_bytes(int T, const TcWeights &plan) {
  const size_t terms = T == F32 ? 2 : 1;
  const size_t stage = terms * tc::kTileM * 128 + terms * (size_t)plan.n_tile * 128;
  return 2 * stage + 1024 + 64;
}

cudaError_t tc_gemm(int T, const GemmOp &op, const TcWeights &plan, const uint8_t *wimg, int *err, cudaStream_t st) {
  if (op.M <= 0) return cudaSuccess;
  tc::Params p;
  p.src = op.src, p.wimg = wimg, p.bias = op.bias, p.res = op.res, p.coarse = op.coarse, p.dst = op.dst;
  p.dw_w = op.dw_w, p.dw_b = op.dw_b, p.err = err;
  p.M = op.M, p.N = op.N, p.K = op.K, p.act = op.act, p.mid_act = op.mid_act;
  p.H = op.H, p.W = op.W, p.OH = op.OH, p.OW = op.OW, p.stride = op.stride;
  p.n_tile = plan.n_tile, p.slabs = plan.slabs, p.tmem_cols = plan.tmem_cols;
  const size_t smem = tc_smem_bytes(T, plan);
  const unsigned gx = (unsigned)((op.M + tc::kTileM - 1) / tc::kTileM), gy = (unsigned)plan.n_tiles;
#define ILL_TC(TT, MODE_, KS_) return launch_t<TT, MODE_, KS_>(p, smem, gx, gy, st)
  if (T == F32) {
    if (op.mode == 0) ILL_TC(float, 0, 1);
    if (op.mode == 2) ILL_TC(float, 2, 1);
    if (op.ks == 3) ILL_TC(float, 1, 3);
    if (op.ks == 5) ILL_TC(float, 1, 5);
  } else {
    if (op.mode == 0) ILL_TC(__nv_bfloat16, 0, 1);
    if (op.mode == 2) ILL_TC(__nv_bfloat16, 2, 1);
    if (op.ks == 3) ILL_TC(__nv_bfloat16, 1, 3);
    if (op.ks == 5) ILL_TC(__nv_bfloat16, 1, 5);
  }
#undef ILL_TC
  return cudaErrorInvalidValue;
}

}  // namespace gpu
}  // namespace illumina
