// Shared pieces of the persistent tcgen05 kernels (tc_pw.cu, tc_dw.cu):
// PTX wrappers for mbarriers, TMA, TMEM and UMMA, and the accumulator
// epilogue.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "arith.cuh"
#include "pdl.cuh"

namespace illumina {
namespace gpu {
namespace tcx {

constexpr int kTileM = 128;
constexpr uint32_t kAImage = kTileM * 128;  // one 128-row x 128-byte operand image
constexpr long long kWaitCycles = 1ll << 31;  // default wait limit: ~1.1 s at 1.965 GHz
// A waiting thread stays suspended in try_wait until the phase completes or
// this many nanoseconds pass, instead of re-polling at the hardware's default
// interval (polling warps take issue slots from the working ones).
constexpr uint32_t kSuspendNs = 20000;
constexpr int kEpiWarps = 8;                // 2 per TMEM lane quarter (column halves)
constexpr int kEpiCols = 16;                // accumulator columns per transpose block
constexpr int kEpiStride = 20;              // floats per row of a block (16 + 4 pad: conflict-free)
constexpr uint32_t kEpiSmem = kEpiWarps * 32 * kEpiStride * 4;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity, uint32_t suspend_ns = kSuspendNs) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of parity `parity`; false once `limit` cycles
// pass. The pipeline waits of a launch take the launch's limit (a kernel
// parameter, kWaitCycles unless the caller lowers it); the waits with which a
// role that gave up drains its own copies and MMAs before the CTA leaves keep
// kWaitCycles, so nothing is in flight when TMEM is released.
// A limit below the suspend interval also shortens each suspension (to about
// the limit at 2 cycles per ns), so a tiny limit gives up at the first probe
// that finds the phase incomplete.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, long long limit = kWaitCycles) {
  const uint32_t hint = limit >= 2ll * kSuspendNs ? kSuspendNs : (uint32_t)(limit / 2 + 1);
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity, hint))
    if (clock64() - t0 > limit) return false;
  return true;
}
// Records that a role gave up a wait: a plain store to the error word (host
// memory mapped into the device's address space, read by the host after the
// launch; nothing else writes it from the device).
__device__ __forceinline__ void report_gave_up(int *err) {
  if (err) *reinterpret_cast<volatile int *>(err) = 1;
}
// Per-warpgroup register budget changes (every warp of the warpgroup runs
// them): the block is launched with a uniform count and the roles trade
// registers; the shares must add up to at most the launch's total.
template <uint32_t N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
// Brings a kernel-parameter TMA descriptor into the descriptor cache ahead of
// its first copy.
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
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
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
// TMA tensor stores (shared -> global, bulk-group completion) and their waits.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(src)
               : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, uint32_t src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Every committed store group has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// At most the most recent committed store group may still be reading.
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// Every committed store group has completed (writes done).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
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
// 1024 bytes apart (SBO), LBO unused, descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: D fp32, A/B format (1 bf16, 2 tf32), K-major, M = 128.
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
// One 128-byte slab of K for a 128 x N tile: 4 MMAs of K = 32 bytes; fp32
// storage issues three TF32 cross products of the hi/lo split (3xTF32: the
// lo x lo term, ~2^-22 of the product, is dropped), small terms first.
template <bool F32>
// `nk`: the slab's 32-byte K chunks that hold channels (1..4); the chunks
// past them are zero padding of the last slab and are not multiplied.
__device__ __forceinline__ void mma_slab(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo,
                                         uint32_t idesc, bool first, int nk = 4) {
#pragma unroll
  for (int kk = 0; kk < 4; kk++) {
    if (kk >= nk) break;
    const uint32_t ko = kk * 32;
    const uint32_t acc = (first && kk == 0) ? 0u : 1u;
    if (F32) {
      mma_tf32(d, smem_desc(a_lo + ko), smem_desc(b_hi + ko), idesc, acc);
      mma_tf32(d, smem_desc(a_hi + ko), smem_desc(b_lo + ko), idesc, 1u);
      mma_tf32(d, smem_desc(a_hi + ko), smem_desc(b_hi + ko), idesc, 1u);
    } else {
      mma_f16(d, smem_desc(a_hi + ko), smem_desc(b_hi + ko), idesc, acc);
    }
  }
}
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, uint32_t r[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
// Round-to-nearest, ties away from zero, to TF32 (10 explicit mantissa bits)
// with two integer operations: adding half of the dropped range to the
// magnitude bits carries into the kept bits (and the exponent) exactly when
// the dropped part is at least one half ulp. illumina_selftest compares it
// with cvt.rna.tf32.f32 over every non-NaN binary32 input.
__device__ __forceinline__ uint32_t tf32_round(float x) { return (__float_as_uint(x) + 0x1000u) & 0xffffe000u; }
// x = hi + lo exactly: hi = x rounded to the nearest TF32 value, lo the
// binary32 remainder (at most 13 significant bits). The kind::tf32 MMA reads
// lo at TF32 precision (its low 13 bits dropped), so the operand it sees is
// within 2^-21 |x| of x (2^-22 if lo were rounded too, at two more
// instructions per element).
__device__ __forceinline__ void split(float x, uint32_t &hi, uint32_t &lo) {
  hi = tf32_round(x);
  lo = __float_as_uint(x - __uint_as_float(hi));
}
__device__ __forceinline__ float hardswish(float v) { return div6(v * fminf(fmaxf(v + 3.0f, 0.0f), 6.0f)); }
// hardswish with the division by 6 as one multiply by RN(1/6): within 1.5 ulp
// of the quotient (RN(1/6) is within half an ulp of 1/6, and the product is
// rounded once more) -- the accuracy class the reference shader's WGSL
// division is specified to (2.5 ulp) -- at one instruction instead of div6's
// four; the tensor-core kernels are issue bound. fp32 storage only: RN(1/6)
// is above 1/6, and where every layer's activations are re-rounded to bf16
// that bias shifts the bf16 roundings through the network, so the BF16
// instances keep div6.
__device__ __forceinline__ float hardswish_fast(float v) {
  return v * fminf(fmaxf(v + 3.0f, 0.0f), 6.0f) * (1.0f / 6.0f);
}
// Compile-time id of hardswish for storage type T (see hardswish_fast).
template <typename T>
constexpr int kHswish = sizeof(T) == 4 ? 4 : 3;
__device__ __forceinline__ float act_apply(int act, float v) {
  switch (act) {
    case 1: return fmaxf(v, 0.0f);
    case 2: return fminf(fmaxf(v, 0.0f), 6.0f);
    case 3: return hardswish(v);
    default: return v;
  }
}
// Compile-time activation (0 linear, 1 relu, 2 relu6, 3 hardswish, 4 the
// single-multiply hardswish) for loops that dispatch on the activation once,
// outside the loop.
template <int ACT>
__device__ __forceinline__ float act_c(float v) {
  if (ACT == 1) return fmaxf(v, 0.0f);
  if (ACT == 2) return fminf(fmaxf(v, 0.0f), 6.0f);
  if (ACT == 3) return hardswish(v);
  if (ACT == 4) return hardswish_fast(v);
  return v;
}
template <int ACT>
__device__ __forceinline__ float4 act_c4(float4 v) {
  return make_float4(act_c<ACT>(v.x), act_c<ACT>(v.y), act_c<ACT>(v.z), act_c<ACT>(v.w));
}
// ACT applied to NV float4 values in place.
template <int ACT, int NV>
__device__ __forceinline__ void act_n(float4 (&v)[NV]) {
#pragma unroll
  for (int i = 0; i < NV; i++) v[i] = act_c4<ACT>(v[i]);
}
__device__ __forceinline__ float4 act4(int act, float4 v) {
  return make_float4(act_apply(act, v.x), act_apply(act, v.y), act_apply(act, v.z), act_apply(act, v.w));
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
// Four fused multiply-adds as two packed f32x2 FMAs (sm_100): each lane is
// rounded once, exactly as fmaf, in half the instructions.
__device__ __forceinline__ float4 f4fma(float4 a, float4 b, float4 c) {
  const float2 lo = __ffma2_rn(make_float2(a.x, a.y), make_float2(b.x, b.y), make_float2(c.x, c.y));
  const float2 hi = __ffma2_rn(make_float2(a.z, a.w), make_float2(b.z, b.w), make_float2(c.z, c.w));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

struct EpiArgs {
  const float *bias;   // [N]; the kernels pass a shared-memory copy
  const void *res;     // [M][N] or null
  const void *coarse;  // lateral: (n, OH/2, OW/2, N) or null
  void *dst;           // [M][N]
  int N, act, OH, OW;
  int n_tile;
  // lateral: the tile's upsampled coarse term in shared memory, tile row r and
  // output column n at cs[r * cs_ld + n - cs_n0]; null: computed from `coarse`
  const float *cs;
  int cs_ld, cs_n0;
  // the depth head folded into the epilogue (TMA-store path, one n tile):
  // per pixel sigmoid(head_b + sum_n stored(n) * head_w[n]) into head_dst[m]
  const float *head_w = nullptr;
  float head_b = 0.0f;
  float *head_dst = nullptr;
};

// Accumulator-independent inputs of one 16-column block for the 4 rows a
// lane stores: per row, the residual (MODE 0) or the bilinear 2x upsample of
// the coarse map plus the residual (MODE 2).
struct EpiBlockIn {
  float4 x[4];
};

// Per-row pixel data of the rows a lane stores (fixed for a tile).
struct EpiRows {
  long m[4];  // output pixel, -1 for a padding row
  int r[4];   // tile row
};

template <typename T, int MODE>
__device__ __forceinline__ EpiBlockIn epi_block_in(const EpiArgs &a, const EpiRows &rows, int n, bool col_ok) {
  EpiBlockIn in;
  const float4 z = make_float4(0, 0, 0, 0);
  const T *res = reinterpret_cast<const T *>(a.res);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const long mm = rows.m[i];
    in.x[i] = (col_ok && mm >= 0 && res) ? ld4(res + mm * a.N + n) : z;
  }
  if (MODE == 2) {
    // the bilinear 2x upsample of the coarse map comes before the residual, as
    // in the reference: from shared memory when it was computed ahead (a.cs),
    // else from its four taps here
#pragma unroll
    for (int i = 0; i < 4; i++) {
      if (!col_ok || rows.m[i] < 0) continue;
      float4 c;
      if (a.cs) {
        c = *reinterpret_cast<const float4 *>(a.cs + rows.r[i] * a.cs_ld + (n - a.cs_n0));
      } else {
        const T *coarse = reinterpret_cast<const T *>(a.coarse);
        const long mm = rows.m[i];
        const uint32_t um = (uint32_t)mm, uow = (uint32_t)a.OW, uoh = (uint32_t)a.OH;
        const uint32_t t = um / uow;
        const int x = (int)(um - t * uow);
        const uint32_t bb = t / uoh;
        const int y = (int)(t - bb * uoh), b = (int)bb;
        const int CH = a.OH >> 1, CW = a.OW >> 1;
        const float sy = (y + 0.5f) * 0.5f - 0.5f, sx = (x + 0.5f) * 0.5f - 0.5f;
        const float fy0 = floorf(sy), fx0 = floorf(sx), fy = sy - fy0, fx = sx - fx0;
        const int y0 = min(max((int)fy0, 0), CH - 1), y1 = min(max((int)fy0 + 1, 0), CH - 1);
        const int x0 = min(max((int)fx0, 0), CW - 1), x1 = min(max((int)fx0 + 1, 0), CW - 1);
        const long rr0 = ((long)b * CH + y0) * CW, rr1 = ((long)b * CH + y1) * CW;
        const float w00 = (1 - fx) * (1 - fy), w01 = fx * (1 - fy), w10 = (1 - fx) * fy, w11 = fx * fy;
        const float4 c00 = ld4(coarse + (rr0 + x0) * a.N + n), c01 = ld4(coarse + (rr0 + x1) * a.N + n);
        const float4 c10 = ld4(coarse + (rr1 + x0) * a.N + n), c11 = ld4(coarse + (rr1 + x1) * a.N + n);
        c.x = c00.x * w00 + c01.x * w01 + c10.x * w10 + c11.x * w11;
        c.y = c00.y * w00 + c01.y * w01 + c10.y * w10 + c11.y * w11;
        c.z = c00.z * w00 + c01.z * w01 + c10.z * w10 + c11.z * w11;
        c.w = c00.w * w00 + c01.w * w01 + c10.w * w10 + c11.w * w11;
      }
      in.x[i] = res ? make_float4(c.x + in.x[i].x, c.y + in.x[i].y, c.z + in.x[i].z, c.w + in.x[i].w) : c;
    }
  }
  return in;
}

// Issues the tcgen05.ld of one block (8 or 16 columns) into v.
__device__ __forceinline__ void epi_block_ld(uint32_t taddr, int width, uint32_t (&v)[kEpiCols]) {
  tmem_ld8_nowait(taddr, v);
  if (width > 8) tmem_ld8_nowait(taddr + 8, v + 8);
}

// Moves one block's accumulator values (already waited for) into this warp's
// shared transpose block.
__device__ __forceinline__ void epi_block_stage(int width, const uint32_t (&v)[kEpiCols], float *blk) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < kEpiCols / 4; j++)
    if (j * 4 < width)
      *reinterpret_cast<float4 *>(blk + lane * kEpiStride + j * 4) =
          make_float4(__uint_as_float(v[j * 4]), __uint_as_float(v[j * 4 + 1]), __uint_as_float(v[j * 4 + 2]),
                      __uint_as_float(v[j * 4 + 3]));
  __syncwarp();
}

// Stores the staged block: row i*8 + lane/4, columns chunk lane%4. `a.bias`
// may point to shared memory (generic load).
template <typename T, int ACT>
__device__ __forceinline__ void epi_block_store(const EpiArgs &a, const EpiRows &rows, int n, bool col_ok,
                                                const EpiBlockIn &in, const float *blk) {
  const int lane = threadIdx.x & 31, chunk = lane & 3, rsub = lane >> 2;
  T *dst = reinterpret_cast<T *>(a.dst);
  if (col_ok) {
    const float4 bias = *reinterpret_cast<const float4 *>(a.bias + n);
    float4 o[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      o[i] = *reinterpret_cast<const float4 *>(blk + (i * 8 + rsub) * kEpiStride + chunk * 4);
      o[i].x += bias.x, o[i].y += bias.y, o[i].z += bias.z, o[i].w += bias.w;
      o[i].x += in.x[i].x, o[i].y += in.x[i].y, o[i].z += in.x[i].z, o[i].w += in.x[i].w;
    }
    act_n<ACT, 4>(o);
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (rows.m[i] >= 0) st4(dst + rows.m[i] * a.N + n, o[i]);
  }
  __syncwarp();
}

// Writes accumulator columns [col0, col0 + ncols) of the 32 TMEM lanes this
// warp owns. Lane l handles rows i*8 + l/4 (i < 4) of the warp's 32 and
// column chunk l%4 of every 16-column block. Each block is read with
// tcgen05.ld, transposed through this warp's shared block so that every store
// instruction writes eight 64-byte row segments (whole sectors), then
// biased, residual/coarse-added, activated and stored.
// Latency: everything that does not depend on the accumulator (residual,
// coarse taps) of the first block is loaded before `ready()` waits
// for the accumulator; once a block is staged in shared memory the next
// block's tcgen05.ld is issued so that it is in flight while the staged block
// is stored, and the next block's residual loads follow those stores (a
// second block of residuals in registers would spill). Returns false when
// `ready()` gave up. The tcgen05.ld issue count depends only on warp-uniform
// values.
template <typename T, int MODE, int ACT, typename ReadyFn>
__device__ __forceinline__ bool epilogue_body(const EpiArgs &a, uint32_t tacc_lane, int col0, int ncols, int n_base,
                                              float *blk, const EpiRows &rows, ReadyFn ready) {
  const int chunk = (threadIdx.x & 31) & 3;
  EpiBlockIn cur;
  {
    const int n = n_base + col0 + chunk * 4;
    cur = epi_block_in<T, MODE>(a, rows, n, chunk * 4 < min(kEpiCols, ncols) && n < a.N);
  }
  if (!ready()) return false;
  uint32_t v[kEpiCols];
  epi_block_ld(tacc_lane + (uint32_t)col0, min(kEpiCols, ncols), v);
  for (int cb = 0; cb < ncols; cb += kEpiCols) {
    const int width = min(kEpiCols, ncols - cb);
    const int n = n_base + col0 + cb + chunk * 4;
    const bool col_ok = chunk * 4 < width && n < a.N;
    const int cb1 = cb + kEpiCols;
    const int n1 = n + kEpiCols;
    const bool ok1 = cb1 < ncols && chunk * 4 < min(kEpiCols, ncols - cb1) && n1 < a.N;
    tmem_wait_ld();
    epi_block_stage(width, v, blk);
    if (cb1 < ncols) epi_block_ld(tacc_lane + (uint32_t)(col0 + cb1), min(kEpiCols, ncols - cb1), v);
    epi_block_store<T, ACT>(a, rows, n, col_ok, cur, blk);
    if (cb1 < ncols) cur = epi_block_in<T, MODE>(a, rows, n1, ok1);  // residual / coarse of the next block
  }
  return true;
}

// Split-K: writes the fp32 accumulator columns [0, ncols) of this warp's 32
// TMEM lanes as rows lane_base + lane of a [128][ld] partial tile (no bias,
// no activation); warps whose rows all lie past `rows_valid` write nothing.
// Bypasses L1: another SM reads the tile.
__device__ __forceinline__ void store_partial(uint32_t tacc_lane, int lane_base, int ncols, float *tile, int ld,
                                              int rows_valid) {
  if (lane_base >= rows_valid) return;  // warp-uniform: rows past the patch are padding
  const int lane = threadIdx.x & 31;
  float *row = tile + (size_t)(lane_base + lane) * ld;
  for (int cb = 0; cb < ncols; cb += kEpiCols) {
    const int width = min(kEpiCols, ncols - cb);
    uint32_t v[kEpiCols];
    epi_block_ld(tacc_lane + (uint32_t)cb, width, v);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < kEpiCols / 4; j++)
      if (j * 4 < width)
        __stcg(reinterpret_cast<float4 *>(row + cb + j * 4),
               make_float4(__uint_as_float(v[j * 4]), __uint_as_float(v[j * 4 + 1]), __uint_as_float(v[j * 4 + 2]),
                           __uint_as_float(v[j * 4 + 3])));
  }
}

// Split-K: output pixel of tile row r of an output patch (th x tw pixels at
// (x0, y0) of frame b), or -1 for a padding row.
struct PatchMap {
  int b, x0, y0, tw, th, OH, OW;
  __device__ __forceinline__ long operator()(int r) const {
    const int ly = r / tw, lx = r - ly * tw;
    const int y = y0 + ly, x = x0 + lx;
    if (ly >= th || y >= OH || x >= OW) return -1;
    return ((long)b * OH + y) * OW + x;
  }
};

// Split-K: sums the ksplit partial tiles of one item ([ksplit][128][ld] at
// `part`; split order fixed, so the result does not depend on the order in
// which the splits were computed), then bias, residual, activation and store.
// a.bias holds the tile's bias (column c of the tile at a.bias[c], 16-byte
// aligned). The nw calling warps (warp index wi) share (8-row group, 16-column
// block) units; groups beyond the patch's th*tw rows are skipped. Four
// splits' loads are in flight at once; partials are read past L1 (written by
// other SMs).
template <typename T, int ACT>
__device__ __forceinline__ void reduce_units(const EpiArgs &a, const float *part, int ksplit, size_t split_stride,
                                             int ld, int ncols, int n_base, const PatchMap &pm, int wi, int nw) {
  const int lane = threadIdx.x & 31, chunk = lane & 3, rsub = lane >> 2;
  const T *res = reinterpret_cast<const T *>(a.res);
  T *dst = reinterpret_cast<T *>(a.dst);
  const int nblocks = (ncols + kEpiCols - 1) / kEpiCols;
  const int ngroups = (pm.th * pm.tw + 7) / 8;
  for (int u = wi; u < ngroups * nblocks; u += nw) {
    const int rg = u / nblocks, blk = u - rg * nblocks;
    const int r = rg * 8 + rsub;
    const int c = blk * kEpiCols + chunk * 4;
    const int n = n_base + c;
    const long m = pm(r);
    if (m < 0 || c >= ncols || n >= a.N) continue;
    const float *pr = part + (size_t)r * ld + c;
    float4 o = make_float4(0, 0, 0, 0);
    for (int j = 0; j < ksplit; j += 4) {
      float4 q[4];
#pragma unroll
      for (int k = 0; k < 4; k++)
        q[k] = j + k < ksplit ? __ldcg(reinterpret_cast<const float4 *>(pr + (j + k) * split_stride))
                              : make_float4(0, 0, 0, 0);
#pragma unroll
      for (int k = 0; k < 4; k++)
        if (j + k < ksplit) o.x += q[k].x, o.y += q[k].y, o.z += q[k].z, o.w += q[k].w;
    }
    const float4 bias = *reinterpret_cast<const float4 *>(a.bias + c);
    o.x += bias.x, o.y += bias.y, o.z += bias.z, o.w += bias.w;
    if (res) {
      const float4 q = ld4(res + m * a.N + n);
      o.x += q.x, o.y += q.y, o.z += q.z, o.w += q.w;
    }
    st4(dst + m * a.N + n, act_c4<ACT>(o));
  }
}

// Out of line: the reduction's registers stay out of the persistent loop that
// calls it.
template <typename T>
__device__ __noinline__ void epilogue_reduce(const EpiArgs a, const float *part, int ksplit, size_t split_stride, int ld,
                                             int ncols, int n_base, const PatchMap pm, int wi, int nw) {
  switch (a.act) {
    case 1: reduce_units<T, 1>(a, part, ksplit, split_stride, ld, ncols, n_base, pm, wi, nw); break;
    case 2: reduce_units<T, 2>(a, part, ksplit, split_stride, ld, ncols, n_base, pm, wi, nw); break;
    case 3: reduce_units<T, kHswish<T>>(a, part, ksplit, split_stride, ld, ncols, n_base, pm, wi, nw); break;
    default: reduce_units<T, 0>(a, part, ksplit, split_stride, ld, ncols, n_base, pm, wi, nw); break;
  }
}

// Split-K reduction launched after a k_tc_dw or k_tc_pw launch that split K:
// item = blockIdx.x (frame, tiles_x x tiles_y patch grid of tw x th pixels,
// n tile; a pointwise item is a 128 x 1 patch of a 1 x M image), its (8-row,
// 16-column) units spread over every warp of gridDim.y CTAs. The partials are
// summed in split order (reduce_units), so the result does not depend on how
// the launches were scheduled; bias, residual, activation and the store
// follow as in the unsplit epilogue.
template <typename T>
__global__ void __launch_bounds__(256) k_splitk_reduce(const EpiArgs a, const float *__restrict__ ws, int ksplit,
                                                       int tiles_x, int tiles_y, int n_tiles, int tw, int th) {
  pdl_trigger();
  pdl_wait();  // the partials are the previous kernel's output
  const int t = blockIdx.x;
  const int nt = t % n_tiles;
  int q = t / n_tiles;
  const int tx = q % tiles_x;
  q /= tiles_x;
  const int ty = q % tiles_y;
  const int b = q / tiles_y;
  const PatchMap pm{b, tx * tw, ty * th, tw, th, a.OH, a.OW};
  const size_t tile_elems = (size_t)kTileM * a.n_tile;
  // the tile's bias, staged with scalar loads (the weight buffer's alignment is 4 bytes)
  __shared__ __align__(16) float sbias[256];
  for (int c = threadIdx.x; c < a.n_tile; c += blockDim.x) {
    const int n = nt * a.n_tile + c;
    sbias[c] = n < a.N ? a.bias[n] : 0.0f;
  }
  __syncthreads();
  EpiArgs ea = a;
  ea.bias = sbias;
  const int wi = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5), nw = gridDim.y * (blockDim.x >> 5);
  epilogue_reduce<T>(ea, ws + (size_t)t * ksplit * tile_elems, ksplit, tile_elems, a.n_tile, a.n_tile,
                     nt * a.n_tile, pm, wi, nw);
}

__device__ __forceinline__ void bar_named(int id, int n);

// TMA-store epilogue. The tile's output columns go out in 16-column slices:
// each lane owns accumulator row `row` (its TMEM lane), adds bias and
// residual, applies the activation and writes its 16 values into a slice
// buffer in the layout of the output tensor map's box (rows of 16 columns,
// SWIZZLE_64B for fp32, SWIZZLE_32B for bf16); once the four warps of the
// group have written a pair of slices, one elected thread issues
// `store(buffer, c0)` for each (a TMA store of columns [c0, c0 + 16) of the
// tile) and commits them; before the pair of buffers is rewritten those
// stores have finished reading it (`slice` counts pairs across tiles). Rows with
// m < 0 (padding) are not written (the box does not cover them, or TMA clips
// them at the tensor edge).
constexpr int kSliceCols = 16;
constexpr uint32_t kSliceBytes = kTileM * kSliceCols * 4;  // one fp32 slice buffer

template <typename T>
__device__ __forceinline__ void slice_put(uint8_t *buf, int row, const float (&o)[kSliceCols]);
template <>
__device__ __forceinline__ void slice_put<float>(uint8_t *buf, int row, const float (&o)[kSliceCols]) {
#pragma unroll
  for (int c = 0; c < 4; c++)
    *reinterpret_cast<float4 *>(buf + row * 64 + ((c ^ ((row >> 1) & 3)) << 4)) =
        make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
}
template <>
__device__ __forceinline__ void slice_put<__nv_bfloat16>(uint8_t *buf, int row, const float (&o)[kSliceCols]) {
#pragma unroll
  for (int c = 0; c < 2; c++) {
    uint4 u;
    uint32_t *pu = &u.x;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(o[8 * c + 2 * j], o[8 * c + 2 * j + 1]);
      pu[j] = *reinterpret_cast<uint32_t *>(&b2);
    }
    *reinterpret_cast<uint4 *>(buf + row * 32 + ((c ^ ((row >> 2) & 1)) << 4)) = u;
  }
}
// Residual of one row's 16 slice columns (zero where absent or past N).
// The value a store of v as T keeps.
template <typename T>
__device__ __forceinline__ float stored_value(float v) {
  return sizeof(T) == 4 ? v : __bfloat162float(__float2bfloat16_rn(v));
}

template <typename T>
__device__ __forceinline__ void slice_res(const EpiArgs &a, long m, int n, float (&r)[kSliceCols]) {
  const T *res = reinterpret_cast<const T *>(a.res);
#pragma unroll
  for (int c = 0; c < 4; c++) {
    float4 q = make_float4(0, 0, 0, 0);
    if (res && m >= 0 && n + 4 * c < a.N) q = ld4(res + m * a.N + n + 4 * c);
    r[4 * c] = q.x, r[4 * c + 1] = q.y, r[4 * c + 2] = q.z, r[4 * c + 3] = q.w;
  }
}

template <typename T, int ACT, typename ReadyFn, typename ReleaseFn, typename StoreFn>
__device__ __forceinline__ bool epilogue_tma_body(const EpiArgs &a, uint32_t tacc_lane, int row, int ncols, int n_base,
                                                  long m, uint8_t *bufs, uint32_t &slice, bool elected, int bar_id,
                                                  int bar_n, ReadyFn ready, ReleaseFn release, StoreFn store) {
  float rv[kSliceCols];
  slice_res<T>(a, m, n_base, rv);
  if (!ready()) return false;
  float hs = a.head_b;  // folded head: the stored values in column order, as k_head sums them
  // slices go out in pairs (32 columns): one barrier pair and two stores per
  // pair, into one pair of buffers
  for (int cb = 0; cb < ncols; cb += 2 * kSliceCols) {
    uint8_t *buf = bufs;
    if (elected) bulk_wait_read0();  // the previous pair's stores have finished reading the buffers
    bar_named(bar_id, bar_n);
    const int pair = min(2, (ncols - cb) / kSliceCols);
    for (int h = 0; h < pair; h++) {
      const int c = cb + h * kSliceCols;
      uint32_t v[kSliceCols];
      tmem_ld8_nowait(tacc_lane + (uint32_t)c, v);
      tmem_ld8_nowait(tacc_lane + (uint32_t)c + 8, v + 8);
      tmem_wait_ld();
      if (c + kSliceCols >= ncols) release();  // the accumulator is free once its last columns are read
      float o[kSliceCols];
      const int n = n_base + c;
#pragma unroll
      for (int j = 0; j < kSliceCols; j += 4) {
        float4 bias = make_float4(0, 0, 0, 0);
        if (n + j < a.N) bias = *reinterpret_cast<const float4 *>(a.bias + n + j);
        o[j] = __uint_as_float(v[j]) + bias.x + rv[j];
        o[j + 1] = __uint_as_float(v[j + 1]) + bias.y + rv[j + 1];
        o[j + 2] = __uint_as_float(v[j + 2]) + bias.z + rv[j + 2];
        o[j + 3] = __uint_as_float(v[j + 3]) + bias.w + rv[j + 3];
      }
      if (c + kSliceCols < ncols) slice_res<T>(a, m, n + kSliceCols, rv);  // next slice's residual in flight
#pragma unroll
      for (int j = 0; j < kSliceCols; j++) o[j] = act_c<ACT>(o[j]);
      if (a.head_dst) {
#pragma unroll
        for (int j = 0; j < kSliceCols; j++)
          if (n + j < a.N) hs = fmaf(stored_value<T>(o[j]), __ldg(a.head_w + n + j), hs);
      }
      if (m >= 0) slice_put<T>(buf + h * kSliceBytes, row, o);
    }
    fence_async_smem();
    bar_named(bar_id, bar_n);
    if (elected) {
      for (int h = 0; h < pair; h++) store(smem_u32(buf + h * kSliceBytes), cb + h * kSliceCols);
      bulk_commit();
    }
    slice++;
  }
  if (a.head_dst && m >= 0) a.head_dst[m] = 1.0f / (1.0f + expf(-hs));
  return true;
}

// `row`: the lane's accumulator row (its TMEM lane); `m`: that row's output
// pixel or -1.
template <typename T, typename ReadyFn, typename ReleaseFn, typename StoreFn>
__device__ __forceinline__ bool epilogue_tma(const EpiArgs &a, uint32_t tacc_lane, int row, int ncols, int n_base,
                                             long m, uint8_t *bufs, uint32_t &slice, bool elected, int bar_id,
                                             int bar_n, ReadyFn ready, ReleaseFn release, StoreFn store) {
  switch (a.act) {
    case 1:
      return epilogue_tma_body<T, 1>(a, tacc_lane, row, ncols, n_base, m, bufs, slice, elected, bar_id, bar_n, ready,
                                     release, store);
    case 2:
      return epilogue_tma_body<T, 2>(a, tacc_lane, row, ncols, n_base, m, bufs, slice, elected, bar_id, bar_n, ready,
                                     release, store);
    case 3:
      return epilogue_tma_body<T, kHswish<T>>(a, tacc_lane, row, ncols, n_base, m, bufs, slice, elected, bar_id, bar_n, ready,
                                     release, store);
    default:
      return epilogue_tma_body<T, 0>(a, tacc_lane, row, ncols, n_base, m, bufs, slice, elected, bar_id, bar_n, ready,
                                     release, store);
  }
}

// Per-warp TMA-store epilogue for tiles whose 32 rows per warp are 32
// consecutive output pixels (pointwise / lateral): lane = accumulator row,
// values go through a 32-row x 16-column swizzled slice (two per warp,
// alternating) and lane 0 stores each as a 2-D box; no other warp is waited
// for. `m`: the lane's output pixel or -1; `cs_row`: for laterals, the lane's
// row of the upsampled coarse term in shared memory (columns relative to the
// tile), else null.
constexpr uint32_t kWarpSliceBytes = 32 * kSliceCols * 4;

template <typename T, int ACT, typename ReadyFn, typename ReleaseFn, typename StoreFn>
__device__ __forceinline__ bool warp_tma_body(const EpiArgs &a, uint32_t tacc_lane, int col0, int ncols, int n_base,
                                              long m, const float *cs_row, uint8_t *wbuf, uint32_t &blocks,
                                              ReadyFn ready, ReleaseFn release, StoreFn store) {
  const int lane = threadIdx.x & 31;
  float rv[kSliceCols];
  slice_res<T>(a, m, n_base + col0, rv);
  if (!ready()) return false;
  for (int cb = 0; cb < ncols; cb += kSliceCols) {
    uint32_t v[kSliceCols];
    tmem_ld8_nowait(tacc_lane + (uint32_t)(col0 + cb), v);
    tmem_ld8_nowait(tacc_lane + (uint32_t)(col0 + cb) + 8, v + 8);
    tmem_wait_ld();
    if (cb + kSliceCols >= ncols) release();
    const int n = n_base + col0 + cb;
    float o[kSliceCols];
#pragma unroll
    for (int j = 0; j < kSliceCols; j += 4) {
      float4 bias = make_float4(0, 0, 0, 0), c = make_float4(0, 0, 0, 0);
      if (n + j < a.N) {
        bias = *reinterpret_cast<const float4 *>(a.bias + n + j);
        if (cs_row) c = *reinterpret_cast<const float4 *>(cs_row + col0 + cb + j);
      }
      // acc + bias, then the coarse term (laterals), then the residual
      o[j] = __uint_as_float(v[j]) + bias.x + c.x + rv[j];
      o[j + 1] = __uint_as_float(v[j + 1]) + bias.y + c.y + rv[j + 1];
      o[j + 2] = __uint_as_float(v[j + 2]) + bias.z + c.z + rv[j + 2];
      o[j + 3] = __uint_as_float(v[j + 3]) + bias.w + c.w + rv[j + 3];
    }
    if (cb + kSliceCols < ncols) slice_res<T>(a, m, n + kSliceCols, rv);
#pragma unroll
    for (int j = 0; j < kSliceCols; j++) o[j] = act_c<ACT>(o[j]);
    uint8_t *buf = wbuf + (blocks & 1) * kWarpSliceBytes;
    if (lane == 0) bulk_wait_read1();  // this buffer's previous store has finished reading it
    __syncwarp();
    if (m >= 0) slice_put<T>(buf, lane, o);
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      store(smem_u32(buf), col0 + cb);
      bulk_commit();
    }
    blocks++;
  }
  return true;
}

template <typename T, typename ReadyFn, typename ReleaseFn, typename StoreFn>
__device__ __forceinline__ bool warp_tma_epilogue(const EpiArgs &a, uint32_t tacc_lane, int col0, int ncols, int n_base,
                                                  long m, const float *cs_row, uint8_t *wbuf, uint32_t &blocks,
                                                  ReadyFn ready, ReleaseFn release, StoreFn store) {
  switch (a.act) {
    case 1: return warp_tma_body<T, 1>(a, tacc_lane, col0, ncols, n_base, m, cs_row, wbuf, blocks, ready, release, store);
    case 2: return warp_tma_body<T, 2>(a, tacc_lane, col0, ncols, n_base, m, cs_row, wbuf, blocks, ready, release, store);
    case 3:
      return warp_tma_body<T, kHswish<T>>(a, tacc_lane, col0, ncols, n_base, m, cs_row, wbuf, blocks, ready, release,
                                         store);
    default:
      return warp_tma_body<T, 0>(a, tacc_lane, col0, ncols, n_base, m, cs_row, wbuf, blocks, ready, release, store);
  }
}

// Named barrier `id` over `n` threads; returns the AND of `v` over them.
__device__ __forceinline__ bool bar_and(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void bar_named(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// `pix(r)` maps a tile row (0..127) to its output pixel, or -1 for a padding
// row; `lane_base` is the first of the warp's 32 TMEM lanes; `ready()` waits
// (bounded) for the accumulator and returns false when it gave up.
template <typename T, int MODE, typename PixFn, typename ReadyFn>
__device__ __forceinline__ bool epilogue_rows(const EpiArgs &a, uint32_t tacc_lane, int lane_base, int col0, int ncols,
                                              int n_base, float *blk, PixFn pix, ReadyFn ready) {
  const int rsub = (threadIdx.x & 31) >> 2;
  EpiRows rows;
#pragma unroll
  for (int i = 0; i < 4; i++) rows.r[i] = lane_base + i * 8 + rsub, rows.m[i] = pix(rows.r[i]);
  switch (a.act) {
    case 1: return epilogue_body<T, MODE, 1>(a, tacc_lane, col0, ncols, n_base, blk, rows, ready);
    case 2: return epilogue_body<T, MODE, 2>(a, tacc_lane, col0, ncols, n_base, blk, rows, ready);
    case 3: return epilogue_body<T, MODE, kHswish<T>>(a, tacc_lane, col0, ncols, n_base, blk, rows, ready);
    default: return epilogue_body<T, MODE, 0>(a, tacc_lane, col0, ncols, n_base, blk, rows, ready);
  }
}

}  // namespace tcx
}  // namespace gpu
}  // namespace illumina
