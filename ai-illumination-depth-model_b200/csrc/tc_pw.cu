// Persistent, warp-specialised tcgen05 kernel for the pointwise and lateral
// ops (the ops whose A operand is an activation tensor read as-is).
//
// Roles inside one CTA (320 threads, one CTA per SM, tiles strided by grid):
//   warp 0        TMA producer: per (tile, K slab) waits for a free ring
//                 stage, then cp.async.bulk.tensor loads the 128-pixel x 128-byte
//                 A tile (SWIZZLE_128B, zero fill past M and K) and
//                 cp.async.bulk copies the pre-swizzled weight image, both
//                 completing on the stage's `full` mbarrier (expect_tx).
//   warps 2-5     fp32 only: split A in shared memory into exact TF32 parts,
//                 hi = rna_tf32(x) rewritten in place and lo = rna_tf32(x - hi)
//                 in a second image, then arrive on `lo_ready`.
//   warp 1        one thread issues tcgen05.mma into one of two TMEM
//                 accumulators (4 TF32 products per K step for fp32:
//                 hi*hi + hi*lo + lo*hi + lo*lo; one kind::f16 MMA for bf16),
//                 commits each stage back to `empty` and each finished tile to
//                 `acc_full`.
//   warps 6-9     epilogue: tcgen05.ld the accumulator rows (warp w owns TMEM
//                 lanes 32*(w%4)..), + bias, + residual or the bilinear
//                 upsample of the coarse tensor, activation, store; then
//                 release the accumulator (`acc_empty`), so the next tile's MMAs
//                 overlap this tile's stores.
// Every mbarrier wait is bounded (~2^31 cycles); a role that gives up records
// it in *err and leaves its loop; all roles meet before TMEM is released.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>

#include "kernels.h"

namespace illumina {
namespace gpu {
namespace tcp {

constexpr int kMmaWarp = 1, kConvWarp0 = 2, kNumConv = 4, kEpiWarp0 = 6, kNumEpi = 4;
constexpr int kThreads = 32 * (kEpiWarp0 + kNumEpi);
constexpr int kTileM = 128;
constexpr uint32_t kAImage = kTileM * 128;
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
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > kWaitCycles) return false;
  return true;
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
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
// K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart, version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
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
// x = hi + lo with hi, lo exact TF32 values (both rounded to nearest).
__device__ __forceinline__ void split(uint32_t x, uint32_t &hi, uint32_t &lo) {
  hi = tf32_rna(__uint_as_float(x));
  lo = tf32_rna(__uint_as_float(x) - __uint_as_float(hi));
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

struct Params {
  const uint8_t *wimg;  // [n tile][slab] images of b_bytes
  const float *bias;
  const void *res;      // [M][N] or null
  const void *coarse;   // lateral: (n, OH/2, OW/2, N)
  void *dst;            // [M][N]
  int *err;
  long M;
  int N, K, act, OH, OW;
  int n_tile, n_tiles, m_tiles, slabs, stages;
  uint32_t acc_stride, tmem_cols, b_bytes;
};

// MODE 0 pointwise, 2 lateral.
template <typename T, int MODE>
__global__ void __launch_bounds__(kThreads, 1) k_tc_pw(const __grid_constant__ CUtensorMap tmap_a, const Params p) {
  constexpr bool kF32 = sizeof(T) == 4;
  constexpr int kTerms = kF32 ? 2 : 1;
  constexpr int kSlabC = 128 / (int)sizeof(T);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const uint32_t stage_bytes = kTerms * kAImage + p.b_bytes;
  const int S = p.stages;
  uint64_t *full = reinterpret_cast<uint64_t *>(base + S * stage_bytes);
  uint64_t *lo_rdy = full + S;
  uint64_t *empty = lo_rdy + S;
  uint64_t *acc_full = empty + S;
  uint64_t *acc_empty = acc_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&lo_rdy[s], kNumConv);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kNumEpi);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = p.m_tiles * p.n_tiles;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const int mt = t / p.n_tiles, nt = t % p.n_tiles;
        for (int s = 0; s < p.slabs; s++) {
          if (!mbar_wait(&empty[stage], phase ^ 1u)) {
            ok = false;
            break;
          }
          uint8_t *st = base + stage * stage_bytes;
          mbar_expect_tx(&full[stage], kAImage + p.b_bytes);
          tma_load_2d(smem_u32(st), &tmap_a, s * kSlabC, mt * kTileM, &full[stage]);
          bulk_load(smem_u32(st + kTerms * kAImage), p.wimg + ((size_t)nt * p.slabs + s) * p.b_bytes, p.b_bytes,
                    &full[stage]);
          if (++stage == S) stage = 0, phase ^= 1u;
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      const uint32_t idesc = instr_desc(kF32 ? 2u : 1u, (uint32_t)p.n_tile);
      const uint32_t b_img = (uint32_t)p.n_tile * 128u;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)acc * p.acc_stride;
        for (int s = 0; s < p.slabs; s++) {
          if (!mbar_wait(&full[stage], phase) || (kF32 && !mbar_wait(&lo_rdy[stage], phase))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(base + stage * stage_bytes);
          const uint32_t sb = sa + kTerms * kAImage;
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const uint32_t ko = kk * 32;
            const uint32_t first = (s | kk) ? 1u : 0u;
            if (kF32) {
              mma_tf32(d, smem_desc(sa + kAImage + ko), smem_desc(sb + b_img + ko), idesc, first);  // lo * lo
              mma_tf32(d, smem_desc(sa + kAImage + ko), smem_desc(sb + ko), idesc, 1u);             // lo * hi
              mma_tf32(d, smem_desc(sa + ko), smem_desc(sb + b_img + ko), idesc, 1u);               // hi * lo
              mma_tf32(d, smem_desc(sa + ko), smem_desc(sb + ko), idesc, 1u);                       // hi * hi
            } else {
              mma_f16(d, smem_desc(sa + ko), smem_desc(sb + ko), idesc, first);
            }
          }
          mma_commit(&empty[stage]);
          if (++stage == S) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        mma_commit(&acc_full[acc]);
        if (++acc == 2) acc = 0, acc_phase ^= 1u;
      }
    }
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------------------ TF32 low parts
    if (kF32) {
      const int ct = tid - kConvWarp0 * 32;
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        for (int s = 0; s < p.slabs; s++) {
          if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase))) {
            ok = false;
            break;
          }
          uint8_t *st = base + stage * stage_bytes;
#pragma unroll 4
          for (int q = ct; q < (int)(kAImage / 16); q += kNumConv * 32) {
            const uint4 v = *reinterpret_cast<const uint4 *>(st + q * 16);
            uint4 hi, lo;
            split(v.x, hi.x, lo.x), split(v.y, hi.y, lo.y), split(v.z, hi.z, lo.z), split(v.w, hi.w, lo.w);
            *reinterpret_cast<uint4 *>(st + q * 16) = hi;
            *reinterpret_cast<uint4 *>(st + kAImage + q * 16) = lo;
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&lo_rdy[stage]);
          if (++stage == S) stage = 0, phase ^= 1u;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int lane_base = (warp & 3) * 32;
    const T *res = reinterpret_cast<const T *>(p.res);
    const T *coarse = reinterpret_cast<const T *>(p.coarse);
    T *dst = reinterpret_cast<T *>(p.dst);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const int mt = t / p.n_tiles, nt = t % p.n_tiles;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const long m = (long)mt * kTileM + lane_base + lane;
      long c00 = 0, c01 = 0, c10 = 0, c11 = 0;
      float w00 = 0, w01 = 0, w10 = 0, w11 = 0;
      if (MODE == 2 && m < p.M) {
        // refUpsample2 taps (reference.ts:161-193)
        const int x = (int)(m % p.OW);
        const long tt = m / p.OW;
        const int y = (int)(tt % p.OH), b = (int)(tt / p.OH);
        const int CH = p.OH >> 1, CW = p.OW >> 1;
        const float sy = (y + 0.5f) * 0.5f - 0.5f, sx = (x + 0.5f) * 0.5f - 0.5f;
        const float fy0 = floorf(sy), fx0 = floorf(sx), fy = sy - fy0, fx = sx - fx0;
        const int y0 = min(max((int)fy0, 0), CH - 1), y1 = min(max((int)fy0 + 1, 0), CH - 1);
        const int x0 = min(max((int)fx0, 0), CW - 1), x1 = min(max((int)fx0 + 1, 0), CW - 1);
        const long r0 = ((long)b * CH + y0) * CW, r1 = ((long)b * CH + y1) * CW;
        c00 = (r0 + x0) * p.N, c01 = (r0 + x1) * p.N, c10 = (r1 + x0) * p.N, c11 = (r1 + x1) * p.N;
        w00 = (1 - fx) * (1 - fy), w01 = fx * (1 - fy), w10 = (1 - fx) * fy, w11 = fx * fy;
      }
      const uint32_t tacc = tmem + (uint32_t)acc * p.acc_stride + ((uint32_t)lane_base << 16);
      for (int cc = 0; cc < p.n_tile; cc += 8) {
        float v[8];
        tmem_ld8(tacc + (uint32_t)cc, v);
        if (m >= p.M) continue;
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int n = nt * p.n_tile + cc + h * 4;
          if (n >= p.N) continue;
          float4 o = make_float4(v[h * 4] + __ldg(p.bias + n), v[h * 4 + 1] + __ldg(p.bias + n + 1),
                                 v[h * 4 + 2] + __ldg(p.bias + n + 2), v[h * 4 + 3] + __ldg(p.bias + n + 3));
          if (MODE == 2) {
            const float4 a = ld4(coarse + c00 + n), b = ld4(coarse + c01 + n);
            const float4 c = ld4(coarse + c10 + n), d = ld4(coarse + c11 + n);
            o.x += a.x * w00 + b.x * w01 + c.x * w10 + d.x * w11;
            o.y += a.y * w00 + b.y * w01 + c.y * w10 + d.y * w11;
            o.z += a.z * w00 + b.z * w01 + c.z * w10 + d.z * w11;
            o.w += a.w * w00 + b.w * w01 + c.w * w10 + d.w * w11;
          }
          if (res) {
            const float4 q = ld4(res + m * p.N + n);
            o.x += q.x, o.y += q.y, o.z += q.z, o.w += q.w;
          }
          o = make_float4(act_apply(p.act, o.x), act_apply(p.act, o.y), act_apply(p.act, o.z),
                          act_apply(p.act, o.w));
          st4(dst + m * p.N + n, o);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) acc = 0, acc_phase ^= 1u;
    }
  }

  if (!ok && p.err) atomicExch(p.err, 1);
  __syncwarp();  // lanes that idled while lane 0 worked rejoin before the block barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, p.tmem_cols);
}

}  // namespace tcp

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int sm_count() {
  static int count[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!count[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    count[dev] = n > 0 ? n : 148;
  }
  return count[dev];
}

constexpr size_t kSmemBudget = 227 * 1024;

template <typename T, int MODE>
cudaError_t launch(const CUtensorMap &map, const tcp::Params &p, size_t smem, cudaStream_t st) {
  auto kern = tcp::k_tc_pw<T, MODE>;
  static unsigned long long granted = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !(granted & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget);
    if (e != cudaSuccess) return e;
    granted |= 1ull << dev;
  }
  const long tiles = (long)p.m_tiles * p.n_tiles;
  const unsigned grid = (unsigned)(tiles < sm_count() ? tiles : sm_count());
  kern<<<grid, tcp::kThreads, smem, st>>>(map, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t tc_pw(int T, const GemmOp &op, const TcWeights &plan, const uint8_t *wimg, int *err, cudaStream_t st) {
  if (op.M <= 0) return cudaSuccess;
  if (op.mode != 0 && op.mode != 2) return cudaErrorInvalidValue;
  auto encode = encode_fn();
  if (!encode) return cudaErrorNotSupported;
  const size_t elt = T == F32 ? 4 : 2;
  const int terms = T == F32 ? 2 : 1;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)op.K, (cuuint64_t)op.M};
  cuuint64_t strides[1] = {(cuuint64_t)op.K * elt};
  cuuint32_t box[2] = {(cuuint32_t)(128 / elt), (cuuint32_t)tcp::kTileM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(&map, T == F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                      const_cast<void *>(op.src), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;

  tcp::Params p;
  p.wimg = wimg, p.bias = op.bias, p.res = op.res, p.coarse = op.coarse, p.dst = op.dst, p.err = err;
  p.M = op.M, p.N = op.N, p.K = op.K, p.act = op.act, p.OH = op.OH, p.OW = op.OW;
  p.n_tile = plan.n_tile, p.n_tiles = plan.n_tiles, p.slabs = plan.slabs;
  p.m_tiles = (int)((op.M + tcp::kTileM - 1) / tcp::kTileM);
  p.acc_stride = 32;
  while ((int)p.acc_stride < plan.n_tile) p.acc_stride <<= 1;
  p.tmem_cols = 2 * p.acc_stride;
  p.b_bytes = (uint32_t)(terms * plan.n_tile * 128);
  const size_t stage = terms * tcp::kAImage + p.b_bytes;
  const size_t fixed = 1024 + 8 * (3 * 8 + 4) + 16;
  int stages = (int)((kSmemBudget - fixed) / stage);
  if (stages > 6) stages = 6;
  if (stages < 2) return cudaErrorInvalidValue;
  p.stages = stages;
  const size_t smem = stages * stage + 1024 + 8 * (3 * stages + 4) + 16;
  if (T == F32) return op.mode == 0 ? launch<float, 0>(map, p, smem, st) : launch<float, 2>(map, p, smem, st);
  return op.mode == 0 ? launch<__nv_bfloat16, 0>(map, p, smem, st) : launch<__nv_bfloat16, 2>(map, p, smem, st);
}

}  // namespace gpu
}  // namespace illumina
