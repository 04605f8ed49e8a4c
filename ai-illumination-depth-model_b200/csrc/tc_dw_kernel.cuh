// Persistent, warp-specialised tcgen05 kernel for the fused depthwise ->
// pointwise op (reference: src/model/reference.ts refDepthwise + refPointwise,
// tools/train/illumina/model.py DwPw). The depthwise output never leaves the
// SM: it is computed from a shared-memory halo straight into the swizzled A
// operand of the pointwise GEMM.
//
// Work item = (frame, output patch of th x tw pixels, tile of n_tile output
// channels); the patch's th*tw <= 128 pixels are the 128 rows of one UMMA
// tile. Per item the kernel walks the input channels in 128-byte slabs.
//
// Roles inside one CTA (640 threads, one CTA per SM, items strided by grid):
//   warp 0        halo producer: per (item, slab) one 4-D TMA load of the
//                 input halo ((th-1)*S+KS rows x (tw-1)*S+KS columns x one
//                 slab, unswizzled; coordinates outside the frame read as
//                 zero, which is the depthwise zero padding) plus a bulk copy
//                 of the slab's depthwise taps and bias into the `H` ring.
//   warp 2        weight producer: bulk copies of the pre-swizzled pointwise
//                 weight images into the `G` ring, or once into a resident
//                 region when all of the op's images fit in shared memory.
//   warps 4-11    depthwise, in `ng` groups of four warps that take the
//                 (item, slab) steps in turn (group g takes steps g, g+ng, ..),
//                 so one group's shared-memory latency hides behind the
//                 other's arithmetic. Each thread owns 4 channels of a run of
//                 P adjacent output pixels, accumulates bias + sum over
//                 (ky, kx) of x * w from the halo (the reference's tap order),
//                 applies the mid activation and writes the A image (TF32
//                 hi/lo pair for fp32 storage, bf16 for bf16 storage).
//   warp 1        one thread issues tcgen05.mma into one of two TMEM
//                 accumulators and commits each G stage back to the ring.
//   warps 12-19   epilogue, two teams of four warps (one per TMEM
//                 accumulator), one warp per TMEM lane quarter: bias and
//                 residual loaded before the accumulator is waited for, then
//                 activation and store; then release the accumulator.
// A ring stage is always used by the same depthwise group (the ring depths
// are multiples of ng), so a group's own previous use of a stage orders its
// parity waits. Every mbarrier wait is bounded; a role that gives up records
// it in *err and leaves its loop; the producers wait (bounded) for their own
// copies and the MMA thread for its own MMAs before all roles meet and TMEM
// is released.
// This header holds the kernel; tc_dw_{f32,bf16}{,_split}.cu instantiate it
// (one storage type and split mode each, so the instances compile in
// parallel) and tc_dw.cu holds the host side.
#pragma once

#include <cudaTypedefs.h>

#include "kernels.h"
#include "pdl.cuh"
#include "tc_common.cuh"

namespace illumina {
namespace gpu {

int sm_count();

namespace tcd {

using namespace tcx;

// Warpgroups: 0 = producers and MMA (warps 0-3), 1-2 = depthwise groups,
// 3-4 = epilogue teams (one per TMEM accumulator). Registers are moved from
// the producer and epilogue warpgroups to the depthwise ones with setmaxnreg:
// 4 x 32 x 32 + 8 x 32 x 136 + 8 x 32 x 88 = 61440 = 640 threads x 96.
constexpr int kMmaWarp = 1, kBWarp = 2, kXfWarp0 = 4, kGroupWarps = 4, kMaxGroups = 2, kEpiWarp0 = 12, kEpiW = 4,
              kEpiTeams = 2;
constexpr int kThreads = 32 * (kEpiWarp0 + kEpiTeams * kEpiW);
constexpr int kLaunchRegs = 96, kProducerRegs = 32, kXfRegs = 136, kEpiRegs = 88;
static_assert(128 * kProducerRegs + 256 * kXfRegs + 256 * kEpiRegs <= kThreads * kLaunchRegs, "register split");
// per epilogue team: one pair of TMA-store slice buffers, or the
// transposed-store blocks of wide tiles
constexpr uint32_t kEpiBytes = 2 * kSliceBytes > kEpiW * 32 * kEpiStride * 4 ? 2 * kSliceBytes
                                                                             : kEpiW * 32 * kEpiStride * 4;


struct Params {
  const uint8_t *wimg;   // pointwise images [n tile][slab], b_bytes each
  const uint8_t *dwblk;  // [slab][KS*KS + 1][slab_c] f32: taps, then bias
  EpiArgs epi;           // OH, OW: output spatial size
  int *err;
  long long wait;  // cycles a pipeline wait may take before the role gives up
  float *ws;  // split-K partial tiles [item][split][128][n_tile] (ksplit > 1)
  int tiles_x, tiles_y, n_tiles, slabs, items, ksplit, spk, total;  // total = items * ksplit units
  int tw, th, iw, mid_act;
  // last K slab: 32-byte K chunks holding channels (MMAs issued) and the
  // 4-channel groups they span (depthwise computed); full slabs use 4 and 128 / 4 / sizeof(T)
  int nk_last, cg_last;
  int sh, sg, b_res, ng;
  int teams;  // epilogue teams: 2 = one per accumulator, 1 = team 0 takes every item
  uint32_t halo_bytes, dw_bytes, h_stage, g_stage, b_bytes, acc_stride, tmem_cols, bias_bytes;
};

struct Item {
  int b, x0, y0, nt;
  int id, split, s0, s1;  // item index, K split, slab range [s0, s1)
};
// Work unit u = item * ksplit + split; items enumerate (frame, patch, n tile)
// with the n tile fastest.
template <bool SPLIT>
__device__ __forceinline__ Item decode(const Params &p, int u) {
  Item it;
  if (SPLIT) {
    it.id = u / p.ksplit;
    it.split = u - it.id * p.ksplit;
    it.s0 = it.split * p.spk;
    it.s1 = min(it.s0 + p.spk, p.slabs);
  } else {
    it.id = u, it.split = 0, it.s0 = 0, it.s1 = p.slabs;
  }
  const int t = it.id;
  it.nt = t % p.n_tiles;
  int q = t / p.n_tiles;
  const int tx = q % p.tiles_x;
  q /= p.tiles_x;
  const int ty = q % p.tiles_y;
  it.b = q / p.tiles_y;
  it.x0 = tx * p.tw;
  it.y0 = ty * p.th;
  return it;
}

// Four channels (group `cg`) of halo pixel R: the TMA wrote one unswizzled
// 128-byte row per pixel. The eight (fp32) or sixteen (bf16) threads that
// read one pixel's row cover it once, so a warp's read takes the minimum
// number of shared-memory wavefronts, and every tap's address is the
// thread's base plus a constant.
__device__ __forceinline__ float4 halo_ld(const float *, const uint8_t *halo, int R, int cg) {
  return *reinterpret_cast<const float4 *>(halo + R * 128 + (cg << 4));
}
__device__ __forceinline__ float4 halo_ld(const __nv_bfloat16 *, const uint8_t *halo, int R, int cg) {
  const uint2 v = *reinterpret_cast<const uint2 *>(halo + R * 128 + (cg << 3));
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&v.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&v.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
// Row r, channel group cg of the K-major SWIZZLE_128B A image(s).
__device__ __forceinline__ void a_st(const float *, uint8_t *A, int r, int cg, float4 v) {
  uint4 hi, lo;
  split(v.x, hi.x, lo.x), split(v.y, hi.y, lo.y), split(v.z, hi.z, lo.z), split(v.w, hi.w, lo.w);
  const int off = r * 128 + ((cg ^ (r & 7)) << 4);
  *reinterpret_cast<uint4 *>(A + off) = hi;
  *reinterpret_cast<uint4 *>(A + kAImage + off) = lo;
}
__device__ __forceinline__ void a_st(const __nv_bfloat16 *, uint8_t *A, int r, int cg, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t *>(&a);
  u.y = *reinterpret_cast<uint32_t *>(&b);
  *reinterpret_cast<uint2 *>(A + r * 128 + (((cg >> 1) ^ (r & 7)) << 4) + ((cg & 1) << 3)) = u;
}

// Depthwise of one slab for one item: halo + weights -> A image. `ct` is the
// thread's index within its group of kGroupWarps warps.
template <typename T, int KS, int S, int P, int ACT>
__device__ __forceinline__ void depthwise_slab(const Params &p, const Item &it, const uint8_t *halo,
                                               const float *dww, uint8_t *A, int ct, int cgn) {
  constexpr int kSlabC = 128 / (int)sizeof(T);
  constexpr int kSpan = (P - 1) * S + KS;
  const int runs = p.tw / P;
  const int units = p.th * runs * cgn;
  const int OH = p.epi.OH, OW = p.epi.OW;
  // u / cgn as a multiply-high: with m = floor(2^32 / cgn) + 1 the quotient is
  // exact for u * cgn < 2^32 (units <= 128 x 16 here)
  const uint32_t cg_magic = 0xffffffffu / (uint32_t)cgn + 1u;
  for (int u = ct; u < units; u += kGroupWarps * 32) {
    const int q = (int)__umulhi((uint32_t)u, cg_magic);
    const int cg = u - q * cgn;
    const int run = q % runs, ly = q / runs;
    const int lx0 = run * P;
    if (it.y0 + ly >= OH || it.x0 + lx0 >= OW) continue;
    const float4 bias = *reinterpret_cast<const float4 *>(dww + KS * KS * kSlabC + cg * 4);
    float4 acc[P];
#pragma unroll
    for (int pp = 0; pp < P; pp++) acc[pp] = bias;
#pragma unroll
    for (int ky = 0; ky < KS; ky++) {
      float4 w[KS];
#pragma unroll
      for (int kx = 0; kx < KS; kx++)
        w[kx] = *reinterpret_cast<const float4 *>(dww + (ky * KS + kx) * kSlabC + cg * 4);
      const int R0 = (ly * S + ky) * p.iw + lx0 * S;
#pragma unroll
      for (int j = 0; j < kSpan; j++) {
        const float4 x = halo_ld(static_cast<const T *>(nullptr), halo, R0 + j, cg);
#pragma unroll
        for (int pp = 0; pp < P; pp++) {
          const int kx = j - pp * S;
          if (kx >= 0 && kx < KS) acc[pp] = f4fma(x, w[kx], acc[pp]);
        }
      }
    }
    const int nvalid = min(P, OW - (it.x0 + lx0));
#pragma unroll
    for (int pp = 0; pp < P; pp++)
      if (pp < nvalid) a_st(static_cast<const T *>(nullptr), A, ly * p.tw + lx0 + pp, cg, act_c4<ACT>(acc[pp]));
  }
}

template <typename T, int KS, int S, int P>
__device__ __forceinline__ void depthwise_dispatch(const Params &p, const Item &it, const uint8_t *halo,
                                                   const float *dww, uint8_t *A, int ct, int cgn) {
  switch (p.mid_act) {
    case 1: depthwise_slab<T, KS, S, P, 1>(p, it, halo, dww, A, ct, cgn); break;
    case 2: depthwise_slab<T, KS, S, P, 2>(p, it, halo, dww, A, ct, cgn); break;
    case 3: depthwise_slab<T, KS, S, P, kHswish<T>>(p, it, halo, dww, A, ct, cgn); break;
    default: depthwise_slab<T, KS, S, P, 0>(p, it, halo, dww, A, ct, cgn); break;
  }
}

// SPLIT: the launch splits K (p.ksplit > 1); a separate instantiation keeps
// the split-K epilogue out of the common kernel's code and registers.
template <typename T, int KS, int S, int P, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) k_tc_dw(const __grid_constant__ CUtensorMap tmap,
                                                       const __grid_constant__ CUtensorMap tmap_out, const Params p) {
  constexpr bool kF32 = sizeof(T) == 4;
  constexpr int kTerms = kF32 ? 2 : 1;
  constexpr int kSlabC = 128 / (int)sizeof(T);
  constexpr int kPad = (KS - 1) / 2;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t *hbase = base;
  uint8_t *gbase = hbase + p.sh * p.h_stage;
  uint8_t *bres = gbase + p.sg * p.g_stage;
  const uint32_t res_bytes = p.b_res ? (uint32_t)(p.n_tiles * p.slabs) * p.b_bytes : 0u;
  float *epi_smem = reinterpret_cast<float *>(bres + res_bytes);
  float *bias_smem = epi_smem + p.teams * kEpiBytes / 4;
  uint64_t *h_full = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(bias_smem) + p.bias_bytes);
  uint64_t *h_empty = h_full + p.sh;
  uint64_t *g_full = h_empty + p.sh;
  uint64_t *a_ready = g_full + p.sg;
  uint64_t *g_empty = a_ready + p.sg;
  uint64_t *acc_full = g_empty + p.sg;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *b_full = acc_empty + 2;
  uint64_t *drain = b_full + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tile = p.epi.n_tile;
  if (tid == 0) {
    for (int s = 0; s < p.sh; s++) {
      mbar_init(&h_full[s], 1);
      mbar_init(&h_empty[s], kGroupWarps);
    }
    for (int s = 0; s < p.sg; s++) {
      mbar_init(&g_full[s], 1);
      mbar_init(&a_ready[s], kGroupWarps);
      mbar_init(&g_empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiW);
    }
    mbar_init(b_full, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (tid == 0) pdl_trigger();
  if (tid == 32) prefetch_tmap(&tmap), prefetch_tmap(&tmap_out);
  if (warp == 0) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  const long long lim = p.wait;

  if (warp < kXfWarp0) {
    reg_dealloc<kProducerRegs>();
    if (warp == 0) {
      // ------------------------------------------------------- halo producer
      if (lane == 0) {
        pdl_wait();  // the input is the previous kernel's output
        int hs = 0;
        uint32_t hph = 0;
        long issued = 0;
        for (int t = blockIdx.x; t < p.total && ok; t += gridDim.x) {
          const Item it = decode<SPLIT>(p, t);
          for (int s = it.s0; s < it.s1; s++) {
            if (!mbar_wait(&h_empty[hs], hph ^ 1u, lim)) {
              ok = false;
              break;
            }
            uint8_t *hst = hbase + (size_t)hs * p.h_stage;
            mbar_expect_tx(&h_full[hs], p.halo_bytes + p.dw_bytes);
            tma_load_4d(smem_u32(hst), &tmap, s * kSlabC, it.x0 * S - kPad, it.y0 * S - kPad, it.b, &h_full[hs]);
            bulk_load(smem_u32(hst + p.halo_bytes), p.dwblk + (size_t)s * p.dw_bytes, p.dw_bytes, &h_full[hs]);
            issued++;
            if (++hs == p.sh) hs = 0, hph ^= 1u;
          }
        }
        // every copy issued above lands before the CTA may leave
        for (long i = issued > p.sh ? issued - p.sh : 0; i < issued; i++)
          ok = mbar_wait(&h_full[i % p.sh], (uint32_t)((i / p.sh) & 1)) && ok;
      }
    } else if (warp == kBWarp) {
      // ------------------------------------------------------- weight producer
      if (lane == 0) {
        if (p.b_res) {
          mbar_expect_tx(b_full, res_bytes);
          for (int i = 0; i < p.n_tiles * p.slabs; i++)
            bulk_load(smem_u32(bres + (size_t)i * p.b_bytes), p.wimg + (size_t)i * p.b_bytes, p.b_bytes, b_full);
          ok = mbar_wait(b_full, 0);
        } else {
          int gs = 0;
          uint32_t gph = 0;
          long issued = 0;
          for (int t = blockIdx.x; t < p.total && ok; t += gridDim.x) {
            const Item it = decode<SPLIT>(p, t);
            const int nt = it.nt;
            for (int s = it.s0; s < it.s1; s++) {
              if (!mbar_wait(&g_empty[gs], gph ^ 1u, lim)) {
                ok = false;
                break;
              }
              mbar_expect_tx(&g_full[gs], p.b_bytes);
              bulk_load(smem_u32(gbase + (size_t)gs * p.g_stage + kTerms * kAImage),
                        p.wimg + ((size_t)nt * p.slabs + s) * p.b_bytes, p.b_bytes, &g_full[gs]);
              issued++;
              if (++gs == p.sg) gs = 0, gph ^= 1u;
            }
          }
          for (long i = issued > p.sg ? issued - p.sg : 0; i < issued; i++)
            ok = mbar_wait(&g_full[i % p.sg], (uint32_t)((i / p.sg) & 1)) && ok;
        }
      }
    } else if (warp == kMmaWarp) {
      // ------------------------------------------------------- MMA issuer
      if (lane == 0) {
        if (p.b_res && !mbar_wait(b_full, 0, lim)) ok = false;
        int gs = 0, acc = 0;
        uint32_t gph = 0, acc_phase = 0;
        const uint32_t idesc = instr_desc(kF32 ? 2u : 1u, (uint32_t)n_tile);
        const uint32_t b_img = (uint32_t)n_tile * 128u;
        for (int t = blockIdx.x; t < p.total && ok; t += gridDim.x) {
          const Item it = decode<SPLIT>(p, t);
          const int nt = it.nt;
          if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, lim)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)acc * p.acc_stride;
          for (int s = it.s0; s < it.s1; s++) {
            if (!mbar_wait(&a_ready[gs], gph, lim) || (!p.b_res && !mbar_wait(&g_full[gs], gph, lim))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(gbase + (size_t)gs * p.g_stage);
            const uint32_t sb = p.b_res ? smem_u32(bres + ((size_t)nt * p.slabs + s) * p.b_bytes) : sa + kTerms * kAImage;
            mma_slab<kF32>(d, sa, sa + kAImage, sb, sb + b_img, idesc, s == it.s0, s == p.slabs - 1 ? p.nk_last : 4);
            mma_commit(&g_empty[gs]);
            if (++gs == p.sg) gs = 0, gph ^= 1u;
          }
          if (!ok) break;
          mma_commit(&acc_full[acc]);
          if (++acc == 2) acc = 0, acc_phase ^= 1u;
        }
        // no MMA of this thread is in flight once `drain` completes
        mma_commit(drain);
        if (!mbar_wait(drain, 0)) ok = false;
      }
  }
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------------- depthwise
    reg_alloc<kXfRegs>();
    const int grp = (warp - kXfWarp0) / kGroupWarps;
    const int ct = tid - (kXfWarp0 + grp * kGroupWarps) * 32;
    if (grp < p.ng) {
      long q = 0;  // (item, slab) step index of this CTA
      for (int t = blockIdx.x; t < p.total && ok; t += gridDim.x) {
        const Item it = decode<SPLIT>(p, t);
        for (int s = it.s0; s < it.s1; s++, q++) {
          if ((int)(q % p.ng) != grp) continue;
          const int hs = (int)(q % p.sh), gs = (int)(q % p.sg);
          const uint32_t hph = (uint32_t)((q / p.sh) & 1), gph = (uint32_t)((q / p.sg) & 1);
          if (!__all_sync(0xffffffffu, mbar_wait(&h_full[hs], hph, lim)) ||
              !__all_sync(0xffffffffu, mbar_wait(&g_empty[gs], gph ^ 1u, lim))) {
            ok = false;
            break;
          }
          const uint8_t *hst = hbase + (size_t)hs * p.h_stage;
          depthwise_dispatch<T, KS, S, P>(p, it, hst, reinterpret_cast<const float *>(hst + p.halo_bytes),
                                          gbase + (size_t)gs * p.g_stage, ct,
                                          s == p.slabs - 1 ? p.cg_last : 32 / (int)sizeof(T));
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&a_ready[gs]);
            mbar_arrive(&h_empty[hs]);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------- epilogue
    // With two teams, team k takes the items of TMEM accumulator k (every
    // other item of this CTA) so two items' epilogues run at once; with one,
    // team 0 takes every item and team 1 idles.
    reg_dealloc<kEpiRegs>();
    const int team = (warp - kEpiWarp0) / kEpiW;
    const int e = (warp - kEpiWarp0) % kEpiW;
    const int lane_base = (warp & 3) * 32;
    const int t_first = (int)blockIdx.x + team * (int)gridDim.x, t_step = p.teams * (int)gridDim.x;
    const int bar_id = 1 + team;
    int acc = team;
    uint32_t acc_phase = 0;
    // next accumulator (and parity) of this team
    auto next_acc = [&]() {
      if (p.teams == 2) acc_phase ^= 1u;
      else if (++acc == 2) acc = 0, acc_phase ^= 1u;
    };
    float *epi_team = epi_smem + team * (kEpiBytes / 4);
    const int tw = p.tw, th = p.th, OH = p.epi.OH, OW = p.epi.OW;
    EpiArgs ea = p.epi;
    ea.bias = bias_smem;
    // the bias is staged here by both teams, off the CTA's set-up path (only
    // the epilogue reads it)
    for (int i = tid - kEpiWarp0 * 32; i < p.epi.N; i += kEpiTeams * kEpiW * 32) bias_smem[i] = p.epi.bias[i];
    bar_named(3, kEpiTeams * kEpiW * 32);
    pdl_wait();  // residual reads, split-K workspace and stores follow the previous kernel
    auto pix_of = [=](const Item &it) {
      return [=](int r) -> long {
        const int ly = r / tw, lx = r - ly * tw;
        const int y = it.y0 + ly, x = it.x0 + lx;
        if (ly >= th || y >= OH || x >= OW) return -1;
        return ((long)it.b * OH + y) * OW + x;
      };
    };
    if (team >= p.teams) {
      // this team has no items
    } else if (!SPLIT && n_tile > 2 * kSliceCols) {
      // wide tiles: transposed stores straight from the epilogue warps
      float *blk = epi_team + e * 32 * kEpiStride;
      for (int t = t_first; t < p.total && ok; t += t_step) {
        const Item it = decode<SPLIT>(p, t);
        uint64_t *full = &acc_full[acc];
        const uint32_t ph = acc_phase;
        if (!epilogue_rows<T, 0>(ea, tmem + (uint32_t)acc * p.acc_stride + ((uint32_t)lane_base << 16), lane_base, 0,
                                 n_tile, it.nt * n_tile, blk, pix_of(it), [full, ph, lim]() {
                                   const bool w = __all_sync(0xffffffffu, mbar_wait(full, ph, lim));
                                   tc_fence_after();
                                   return w;
                                 })) {
          ok = false;
          break;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        next_acc();
      }
    } else if (!SPLIT) {
      // tiles of up to 32 columns: TMA-store epilogue, 16-column slices of the
      // patch go out as 4-D boxes (tensor edges clipped by TMA); the team's
      // four warps meet at named barrier 1 + team.
      uint8_t *bufs = reinterpret_cast<uint8_t *>(epi_team);
      const bool elected = e == 0 && lane == 0;
      uint32_t slice = 0;
      for (int t = t_first; t < p.total && ok; t += t_step) {
        const Item it = decode<SPLIT>(p, t);
        uint64_t *full = &acc_full[acc];
        const uint32_t ph = acc_phase;
        uint64_t *empty_bar = &acc_empty[acc];
        const int row = lane_base + lane;
        const long m = pix_of(it)(row);
        const int n0 = it.nt * n_tile;
        if (!epilogue_tma<T>(
                ea, tmem + (uint32_t)acc * p.acc_stride + ((uint32_t)lane_base << 16), row, n_tile, n0, m, bufs, slice,
                elected, bar_id, kEpiW * 32,
                [full, ph, bar_id, lim]() {
                  const bool w = bar_and(bar_id, kEpiW * 32, mbar_wait(full, ph, lim));
                  tc_fence_after();
                  return w;
                },
                [empty_bar, lane]() {
                  tc_fence_before();
                  __syncwarp();
                  if (lane == 0) mbar_arrive(empty_bar);
                },
                [&tmap_out, it, n0](uint32_t src, int cb) { tma_store_4d(&tmap_out, src, n0 + cb, it.x0, it.y0, it.b); })) {
          ok = false;
          break;
        }
        next_acc();
      }
      if (elected) bulk_wait_all();  // the output is written before the CTA leaves
    } else {
      // split-K: write this split's partial tile and release the accumulator;
      // k_splitk_reduce, launched after this kernel, sums the item's partials
      // in split order and stores the item. The four epilogue warps agree on
      // every wait's outcome through named barrier 1.
      const size_t tile_elems = (size_t)kTileM * n_tile;
      for (int t = t_first; t < p.total && ok; t += t_step) {
        const Item it = decode<SPLIT>(p, t);
        const bool w = bar_and(1, kEpiW * 32, mbar_wait(&acc_full[acc], acc_phase, lim));
        tc_fence_after();
        if (!w) {
          ok = false;
          break;
        }
        float *part = p.ws + (size_t)it.id * p.ksplit * tile_elems;
        store_partial(tmem + (uint32_t)acc * p.acc_stride + ((uint32_t)lane_base << 16), lane_base, n_tile,
                      part + it.split * tile_elems, n_tile, th * tw);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        next_acc();
      }
    }
  }

  if (!ok) report_gave_up(p.err);
  __syncwarp();  // lanes that idled while lane 0 worked rejoin before the block barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, p.tmem_cols);
}


constexpr size_t kSmemBudget = 227 * 1024;

template <typename T, int KS, int S, int P, bool SPLIT>
cudaError_t launch_dw(const CUtensorMap &map, const CUtensorMap &map_out, const tcd::Params &p, size_t smem,
                      cudaStream_t st) {
  auto kern = tcd::k_tc_dw<T, KS, S, P, SPLIT>;
  static unsigned long long granted = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !(granted & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget);
    if (e != cudaSuccess) return e;
    granted |= 1ull << dev;
  }
  const unsigned grid = (unsigned)(p.total < sm_count() ? p.total : sm_count());
  cudaError_t e = launch_pdl(kern, dim3(grid), dim3(tcd::kThreads), smem, st, map, map_out, p);
  if (e != cudaSuccess || !SPLIT) return e;
  // one warp per (8-row, 16-column) unit of an item
  const int units = ((p.th * p.tw + 7) / 8) * ((p.epi.n_tile + kEpiCols - 1) / kEpiCols);
  EpiArgs ea = p.epi;
  return launch_pdl(k_splitk_reduce<T>, dim3((unsigned)p.items, (unsigned)((units + 7) / 8)), dim3(256), 0, st, ea,
                    (const float *)p.ws, p.ksplit, p.tiles_x, p.tiles_y, p.n_tiles, p.tw, p.th);
}

template <typename T, int KS, int S, bool SPLIT>
cudaError_t launch_p(int P, const CUtensorMap &map, const CUtensorMap &map_out, const tcd::Params &p, size_t smem,
                     cudaStream_t st) {
  switch (P) {
    case 8: return launch_dw<T, KS, S, 8, SPLIT>(map, map_out, p, smem, st);
    case 7: return launch_dw<T, KS, S, 7, SPLIT>(map, map_out, p, smem, st);
    case 4: return launch_dw<T, KS, S, 4, SPLIT>(map, map_out, p, smem, st);
    case 2: return launch_dw<T, KS, S, 2, SPLIT>(map, map_out, p, smem, st);
    default: return cudaErrorInvalidValue;
  }
}
// Launch of the instance for (KS, S, P); SPLIT must match p.ksplit > 1.
template <typename T, bool SPLIT>
cudaError_t launch_all(int KS, int S, int P, const CUtensorMap &map, const CUtensorMap &map_out, const tcd::Params &p,
                       size_t smem, cudaStream_t st) {
  if (KS == 3 && S == 1) return launch_p<T, 3, 1, SPLIT>(P, map, map_out, p, smem, st);
  if (KS == 3 && S == 2) return launch_p<T, 3, 2, SPLIT>(P, map, map_out, p, smem, st);
  if (KS == 5 && S == 1) return launch_p<T, 5, 1, SPLIT>(P, map, map_out, p, smem, st);
  if (KS == 5 && S == 2) return launch_p<T, 5, 2, SPLIT>(P, map, map_out, p, smem, st);
  return cudaErrorInvalidValue;
}


}  // namespace tcd
}  // namespace gpu
}  // namespace illumina
