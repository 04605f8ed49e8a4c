// Persistent, warp-specialised tcgen05 kernel for the pointwise and lateral
// ops (the ops whose A operand is an activation tensor read as-is).
//
// Roles inside one CTA (448 threads, one CTA per SM, tiles strided by grid):
//   warp 0        TMA producer: per (tile, K slab) waits for a free ring
//                 stage, then cp.async.bulk.tensor loads the 128-pixel x 128-byte
//                 A tile (SWIZZLE_128B, zero fill past M and K) and
//                 cp.async.bulk copies the pre-swizzled weight image, both
//                 completing on the stage's `full` mbarrier (expect_tx).
//   warps 2-5     fp32 only: split A in shared memory into exact TF32 parts,
//                 hi = rna_tf32(x) rewritten in place and lo = rna_tf32(x - hi)
//                 in a second image, then arrive on `lo_ready`.
//   warp 1        one thread issues tcgen05.mma into one of two TMEM
//                 accumulators (4 TF32 cross products per K step for fp32, one
//                 kind::f16 MMA for bf16), commits each stage back to `empty`
//                 and each finished tile to `acc_full`.
//   warps 6-13    epilogue (tcx::epilogue_rows): two warps per TMEM lane
//                 quarter, one per column half; loads what does not depend on
//                 the accumulator (bias, residual, coarse taps) before waiting
//                 for it, then releases it (`acc_empty`) so the next tile's
//                 MMAs overlap these stores.
// Every mbarrier wait is bounded; a role that gives up records it in *err and
// leaves its loop; all roles meet before TMEM is released.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

#include "kernels.h"
#include "pdl.cuh"
#include "tc_common.cuh"

namespace illumina {
namespace gpu {
namespace tcp {

using namespace tcx;

constexpr int kMmaWarp = 1, kConvWarp0 = 2, kNumConv = 4, kEpiWarp0 = 6;
constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
// epilogue shared memory: two TMA-store slices per warp, or (laterals without
// the coarse ring) the transposed-store blocks
constexpr uint32_t kEpiPw = 2 * kEpiWarps * kWarpSliceBytes > kEpiSmem ? 2 * kEpiWarps * kWarpSliceBytes : kEpiSmem;

struct Params {
  const uint8_t *wimg;  // [n tile][slab] images of b_bytes
  EpiArgs epi;
  int *err;
  long long wait;  // cycles a pipeline wait may take before the role gives up
  long M;
  int n_tiles, m_tiles, slabs, stages;
  uint32_t acc_stride, tmem_cols, b_bytes, bias_bytes;
  int cs_ld;           // lateral: row stride (floats) of the coarse ring's tiles
  int cs_stages;       // lateral: coarse ring depth (0: the epilogue gathers the taps itself)
  uint32_t cs_bytes;   // cs_stages * 128 * cs_ld * 4
  // split-K (pointwise only): unit u = tile * ksplit + split covers slabs
  // [split * spk, min((split + 1) * spk, slabs)) and stores its fp32 partial
  // tile at ws[(tile * ksplit + split) * 128 * n_tile]
  int ksplit, spk;
  float *ws;
};

// Tile (m tile, n tile) and slab range of work unit t.
template <bool SPLIT>
__device__ __forceinline__ void unit_of(const Params &p, int t, int &mt, int &nt, int &s0, int &s1) {
  int tile = t;
  s0 = 0, s1 = p.slabs;
  if (SPLIT) {
    tile = t / p.ksplit;
    s0 = (t - tile * p.ksplit) * p.spk;
    s1 = min(s0 + p.spk, p.slabs);
  }
  mt = tile / p.n_tiles, nt = tile - mt * p.n_tiles;
}

// Lateral: the bilinear 2x upsample (refUpsample2, reference.ts:161-193:
// source coordinate (i + 0.5) / 2 - 0.5, both taps from the unclamped floor,
// clamped independently) of the coarse map for the tile's 128 rows (pixels
// m0 ..) and columns [n0, n0 + n_tile) of N, into `cs` (row stride cs_ld).
// Work item = (run of 8 consecutive tile rows, 4-column group); threads take
// items with the column group fastest, so a warp's loads of one coarse pixel
// are contiguous. A run inside one output row starting at an even x needs
// coarse columns x/2 - 1 .. x/2 + 4 (clamped) of two coarse rows: its 12
// loads are issued together and each pixel combines its four taps with the
// reference's weights and expression. Other runs (row ends, odd widths) take
// the taps per pixel.
template <typename T>
__device__ __forceinline__ void coarse_tile(const EpiArgs &a, long M, long m0, int n0, int n_tile, float *cs,
                                            int cs_ld, int ct, int nthreads) {
  const T *coarse = reinterpret_cast<const T *>(a.coarse);
  const int ncol = min(n_tile, a.N - n0);
  const int nchunks = ncol / 4;
  const int CH = a.OH >> 1, CW = a.OW >> 1;
  const uint32_t uow = (uint32_t)a.OW, uoh = (uint32_t)a.OH;
  for (int item = ct; item < 16 * nchunks; item += nthreads) {
    const int run = item / nchunks, c4 = item - run * nchunks;
    const int r0 = run * 8;
    const long mA = m0 + r0;
    if (mA >= M) continue;
    const int n = n0 + c4 * 4;
    const uint32_t um = (uint32_t)mA;
    const uint32_t t = um / uow;
    const int x = (int)(um - t * uow);
    const uint32_t bb = t / uoh;
    const int y = (int)(t - bb * uoh), b = (int)bb;
    const float sy = (y + 0.5f) * 0.5f - 0.5f;
    const float fy0 = floorf(sy), fy = sy - fy0;
    const int y0 = min(max((int)fy0, 0), CH - 1), y1 = min(max((int)fy0 + 1, 0), CH - 1);
    const long rr0 = ((long)b * CH + y0) * CW, rr1 = ((long)b * CH + y1) * CW;
    if ((x & 1) == 0 && x + 7 < a.OW && mA + 7 < M) {
      const int base = x / 2 - 1;
      float4 t0[6], t1[6];
#pragma unroll
      for (int j = 0; j < 6; j++) {
        const int cx = min(max(base + j, 0), CW - 1);
        t0[j] = ld4(coarse + (rr0 + cx) * a.N + n);
        t1[j] = ld4(coarse + (rr1 + cx) * a.N + n);
      }
#pragma unroll
      for (int pp = 0; pp < 8; pp++) {
        const int xp = x + pp;
        const float sx = (xp + 0.5f) * 0.5f - 0.5f;
        const float fx0 = floorf(sx), fx = sx - fx0;
        // for even x the unclamped taps are base + (pp + 1) / 2 and the next
        // one; the loaded column base + j already holds clamp(base + j)
        const int l0 = (pp + 1) / 2;
        const float w00 = (1 - fx) * (1 - fy), w01 = fx * (1 - fy), w10 = (1 - fx) * fy, w11 = fx * fy;
        const float4 c00 = t0[l0], c01 = t0[l0 + 1], c10 = t1[l0], c11 = t1[l0 + 1];
        float4 o;
        o.x = c00.x * w00 + c01.x * w01 + c10.x * w10 + c11.x * w11;
        o.y = c00.y * w00 + c01.y * w01 + c10.y * w10 + c11.y * w11;
        o.z = c00.z * w00 + c01.z * w01 + c10.z * w10 + c11.z * w11;
        o.w = c00.w * w00 + c01.w * w01 + c10.w * w10 + c11.w * w11;
        *reinterpret_cast<float4 *>(cs + (size_t)(r0 + pp) * cs_ld + c4 * 4) = o;
      }
    } else {
      for (int pp = 0; pp < 8 && mA + pp < M; pp++) {
        const uint32_t ump = (uint32_t)(mA + pp);
        const uint32_t tp = ump / uow;
        const int xp = (int)(ump - tp * uow);
        const uint32_t bp = tp / uoh;
        const int yp = (int)(tp - bp * uoh);
        const float syp = (yp + 0.5f) * 0.5f - 0.5f, sx = (xp + 0.5f) * 0.5f - 0.5f;
        const float fyp0 = floorf(syp), fx0 = floorf(sx), fyp = syp - fyp0, fx = sx - fx0;
        const int ya = min(max((int)fyp0, 0), CH - 1), yb = min(max((int)fyp0 + 1, 0), CH - 1);
        const int xa = min(max((int)fx0, 0), CW - 1), xb = min(max((int)fx0 + 1, 0), CW - 1);
        const long q0 = ((long)bp * CH + ya) * CW, q1 = ((long)bp * CH + yb) * CW;
        const float w00 = (1 - fx) * (1 - fyp), w01 = fx * (1 - fyp), w10 = (1 - fx) * fyp, w11 = fx * fyp;
        const float4 c00 = ld4(coarse + (q0 + xa) * a.N + n), c01 = ld4(coarse + (q0 + xb) * a.N + n);
        const float4 c10 = ld4(coarse + (q1 + xa) * a.N + n), c11 = ld4(coarse + (q1 + xb) * a.N + n);
        float4 o;
        o.x = c00.x * w00 + c01.x * w01 + c10.x * w10 + c11.x * w11;
        o.y = c00.y * w00 + c01.y * w01 + c10.y * w10 + c11.y * w11;
        o.z = c00.z * w00 + c01.z * w01 + c10.z * w10 + c11.z * w11;
        o.w = c00.w * w00 + c01.w * w01 + c10.w * w10 + c11.w * w11;
        *reinterpret_cast<float4 *>(cs + (size_t)(r0 + pp) * cs_ld + c4 * 4) = o;
      }
    }
  }
}

// MODE 0 pointwise, 2 lateral; SPLIT: the launch splits K (pointwise only)
// and the epilogue stores fp32 partial tiles for k_splitk_reduce.
template <typename T, int MODE, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) k_tc_pw(const __grid_constant__ CUtensorMap tmap_a,
                                                       const __grid_constant__ CUtensorMap tmap_out, const Params p) {
  constexpr bool kF32 = sizeof(T) == 4;
  constexpr int kTerms = kF32 ? 2 : 1;
  constexpr int kSlabC = 128 / (int)sizeof(T);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const uint32_t stage_bytes = kTerms * kAImage + p.b_bytes;
  const int S = p.stages;
  float *epi_smem = reinterpret_cast<float *>(base + S * stage_bytes);
  float *bias_smem = epi_smem + kEpiPw / 4;
  float *cs_smem = bias_smem + p.bias_bytes / 4;  // lateral coarse ring: 2 x [128][cs_ld]
  uint64_t *full = reinterpret_cast<uint64_t *>(base + S * stage_bytes + kEpiPw + p.bias_bytes + p.cs_bytes);
  uint64_t *lo_rdy = full + S;
  uint64_t *empty = lo_rdy + S;
  uint64_t *acc_full = empty + S;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *c_full = acc_empty + 2;
  uint64_t *c_empty = c_full + 2;
  uint64_t *drain = c_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tile = p.epi.n_tile;
  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&lo_rdy[s], kNumConv);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiWarps);
      mbar_init(&c_full[a], kNumConv);
      mbar_init(&c_empty[a], kEpiWarps);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (tid == 0) pdl_trigger();
  if (tid == 32) prefetch_tmap(&tmap_a), prefetch_tmap(&tmap_out);
  if (warp == 0) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = p.m_tiles * p.n_tiles * (SPLIT ? p.ksplit : 1);
  bool ok = true;
  const long long lim = p.wait;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      pdl_wait();  // the A tiles are the previous kernel's output
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int mt, nt, s0, s1;
        unit_of<SPLIT>(p, t, mt, nt, s0, s1);
        for (int s = s0; s < s1; s++) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, lim)) {
            ok = false;
            break;
          }
          uint8_t *st = base + stage * stage_bytes;
          mbar_expect_tx(&full[stage], kAImage + p.b_bytes);
          tma_load_2d(smem_u32(st), &tmap_a, s * kSlabC, mt * kTileM, &full[stage]);
          bulk_load(smem_u32(st + kTerms * kAImage), p.wimg + ((size_t)nt * p.slabs + s) * p.b_bytes, p.b_bytes,
                    &full[stage]);
          issued++;
          if (++stage == S) stage = 0, phase ^= 1u;
        }
      }
      // every copy issued above lands before the CTA may leave (a consumer
      // that gave up leaves its stages unread)
      for (long i = issued > S ? issued - S : 0; i < issued; i++)
        ok = mbar_wait(&full[i % S], (uint32_t)((i / S) & 1)) && ok;
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      const uint32_t idesc = instr_desc(kF32 ? 2u : 1u, (uint32_t)n_tile);
      const uint32_t b_img = (uint32_t)n_tile * 128u;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, lim)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)acc * p.acc_stride;
        int mt_, nt_, s0, s1;
        unit_of<SPLIT>(p, t, mt_, nt_, s0, s1);
        (void)mt_, (void)nt_;
        for (int s = s0; s < s1; s++) {
          if (!mbar_wait(&full[stage], phase, lim) || (kF32 && !mbar_wait(&lo_rdy[stage], phase, lim))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(base + stage * stage_bytes);
          const uint32_t sb = sa + kTerms * kAImage;
          mma_slab<kF32>(d, sa, sa + kAImage, sb, sb + b_img, idesc, s == s0);
          mma_commit(&empty[stage]);
          if (++stage == S) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        mma_commit(&acc_full[acc]);
        if (++acc == 2) acc = 0, acc_phase ^= 1u;
      }
      // no MMA of this thread is in flight once `drain` completes
      mma_commit(drain);
      if (!mbar_wait(drain, 0)) ok = false;
    }
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------ TF32 split, lateral coarse term
    const int ct = tid - kConvWarp0 * 32;
    int stage = 0, cst = 0;
    uint32_t phase = 0, cph = 0;
    const bool ring = MODE == 2 && p.cs_stages > 0;
    if (ring) pdl_wait();  // the coarse map is an earlier kernel's output
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      if (kF32) {
        int mt_, nt_, s0, s1;
        unit_of<SPLIT>(p, t, mt_, nt_, s0, s1);
        (void)mt_, (void)nt_;
        for (int s = s0; s < s1; s++) {
          if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, lim))) {
            ok = false;
            break;
          }
          uint8_t *st = base + stage * stage_bytes;
#pragma unroll 4
          for (int q = ct; q < (int)(kAImage / 16); q += kNumConv * 32) {
            const float4 v = *reinterpret_cast<const float4 *>(st + q * 16);
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
        if (!ok) break;
      }
      if (ring) {
        // (8-row run, 4-column group) items, ahead of the epilogue
        if (!__all_sync(0xffffffffu, mbar_wait(&c_empty[cst], cph ^ 1u, lim))) {
          ok = false;
          break;
        }
        const int mt = t / p.n_tiles, nt = t % p.n_tiles;
        coarse_tile<T>(p.epi, p.M, (long)mt * kTileM, nt * n_tile, n_tile, cs_smem + cst * kTileM * p.cs_ld, p.cs_ld,
                       ct, kNumConv * 32);
        __syncwarp();
        if (lane == 0) mbar_arrive(&c_full[cst]);
        if (++cst == p.cs_stages) cst = 0, cph ^= 1u;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - kEpiWarp0;
    const int lane_base = (warp & 3) * 32;
    const int half = n_tile / 2;
    int acc = 0, cst = 0;
    uint32_t acc_phase = 0, cph = 0;
    EpiArgs ea = p.epi;
    ea.bias = bias_smem;
    ea.cs = nullptr;
    ea.cs_ld = p.cs_ld;
    // the bias is staged here, off the CTA's set-up path (only the epilogue reads it)
    for (int i = tid - kEpiWarp0 * 32; i < p.epi.N; i += kEpiWarps * 32) bias_smem[i] = p.epi.bias[i];
    bar_named(1, kEpiWarps * 32);
    pdl_wait();  // residual / coarse reads and the stores follow the previous kernel
    // per-warp TMA stores of whole 16-column slices, unless a warp's column
    // half is not a multiple of 16 (a slice would spill into the other half)
    // or a lateral gathers its coarse taps itself
    const bool tma_out = (MODE == 0 || p.cs_stages > 0) && half % kSliceCols == 0;
    uint8_t *wbuf = reinterpret_cast<uint8_t *>(epi_smem) + e * 2 * kWarpSliceBytes;
    float *blk = epi_smem + e * 32 * kEpiStride;
    uint32_t blocks = 0;
    if (SPLIT) {
      // each warp stores its lane quarter x column half of the partial tile
      const size_t tile_elems = (size_t)kTileM * n_tile;
      const int col0 = (e >> 2) * half;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int mt, nt, s0, s1;
        unit_of<SPLIT>(p, t, mt, nt, s0, s1);
        if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase, lim))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const long rows = p.M - (long)mt * kTileM;
        store_partial(tmem + (uint32_t)acc * p.acc_stride + ((uint32_t)lane_base << 16) + (uint32_t)col0, lane_base,
                      half, p.ws + (size_t)t * tile_elems + col0, n_tile, rows < kTileM ? (int)rows : kTileM);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        if (++acc == 2) acc = 0, acc_phase ^= 1u;
      }
    }
    for (int t = blockIdx.x; t < total && ok && !SPLIT; t += gridDim.x) {
      const int mt = t / p.n_tiles, nt = t % p.n_tiles;
      const long m0 = (long)mt * kTileM;
      const long M = p.M;
      uint64_t *full = &acc_full[acc];
      uint64_t *empty_bar = &acc_empty[acc];
      const uint32_t ph = acc_phase;
      const uint32_t tacc = tmem + (uint32_t)acc * p.acc_stride + ((uint32_t)lane_base << 16);
      const float *cs_row = nullptr;
      if (MODE == 2 && p.cs_stages > 0) {
        if (!__all_sync(0xffffffffu, mbar_wait(&c_full[cst], cph, lim))) {
          ok = false;
          break;
        }
        ea.cs = cs_smem + cst * kTileM * p.cs_ld;
        ea.cs_n0 = nt * n_tile;
        cs_row = ea.cs + (lane_base + lane) * p.cs_ld;
      }
      auto ready = [full, ph, lim]() {
        const bool w = __all_sync(0xffffffffu, mbar_wait(full, ph, lim));
        tc_fence_after();
        return w;
      };
      if (tma_out) {
        const long mrow = m0 + lane_base + lane < M ? m0 + lane_base + lane : -1;
        const int n_base = nt * n_tile;
        if (!warp_tma_epilogue<T>(
                ea, tacc, (e >> 2) * half, half, n_base, mrow, cs_row, wbuf, blocks, ready,
                [empty_bar, lane]() {
                  tc_fence_before();
                  __syncwarp();
                  if (lane == 0) mbar_arrive(empty_bar);
                },
                [&tmap_out, n_base, m0, lane_base](uint32_t src, int c) {
                  tma_store_2d(&tmap_out, src, n_base + c, (int)(m0 + lane_base));
                })) {
          ok = false;
          break;
        }
      } else {
        if (!epilogue_rows<T, MODE>(ea, tacc, lane_base, (e >> 2) * half, half, nt * n_tile, blk,
                                    [m0, M](int r) -> long { return m0 + r < M ? m0 + r : -1; }, ready)) {
          ok = false;
          break;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar);
      }
      if (++acc == 2) acc = 0, acc_phase ^= 1u;
      if (MODE == 2 && p.cs_stages > 0) {
        if (lane == 0) mbar_arrive(&c_empty[cst]);
        if (++cst == p.cs_stages) cst = 0, cph ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_all();  // this warp's stores are written before the CTA leaves
  }

  if (!ok) report_gave_up(p.err);
  __syncwarp();  // lanes that idled while lane 0 worked rejoin before the block barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, p.tmem_cols);
}

}  // namespace tcp

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

namespace {

constexpr size_t kSmemBudget = 227 * 1024;
constexpr int kSplitMinSlabs = 10;  // shortest K walk (in 128-byte slabs) that split-K shortens enough

template <typename T, int MODE, bool SPLIT>
cudaError_t launch(const CUtensorMap &map, const CUtensorMap &map_out, const tcp::Params &p, size_t smem,
                   cudaStream_t st) {
  auto kern = tcp::k_tc_pw<T, MODE, SPLIT>;
  static unsigned long long granted = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !(granted & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget);
    if (e != cudaSuccess) return e;
    granted |= 1ull << dev;
  }
  const long tiles = (long)p.m_tiles * p.n_tiles;
  const long units = tiles * (SPLIT ? p.ksplit : 1);
  const unsigned grid = (unsigned)(units < sm_count() ? units : sm_count());
  cudaError_t e = launch_pdl(kern, dim3(grid), dim3(tcp::kThreads), smem, st, map, map_out, p);
  if (e != cudaSuccess || !SPLIT) return e;
  // the partials of each (m tile, n tile) item, summed in split order: an item
  // is a run of 128 pixels, one 128 x 1 "patch" of a 1 x M image
  tcx::EpiArgs ea = p.epi;
  ea.OH = 1, ea.OW = (int)p.M;
  const int red_units = (tcx::kTileM / 8) * ((p.epi.n_tile + tcx::kEpiCols - 1) / tcx::kEpiCols);
  return launch_pdl(tcx::k_splitk_reduce<T>, dim3((unsigned)tiles, (unsigned)((red_units + 7) / 8)), dim3(256), 0,
                    st, ea, (const float *)p.ws, p.ksplit, p.m_tiles, 1, p.n_tiles, tcx::kTileM, 1);
}

}  // namespace

cudaError_t tc_pw(int T, const GemmOp &op, const TcWeights &plan, const uint8_t *wimg, int *err, cudaStream_t st) {
  if (op.M <= 0) return cudaSuccess;
  if (op.mode != 0 && op.mode != 2) return cudaErrorInvalidValue;
  if (op.M > 0x7fffffffL) return cudaErrorInvalidValue;  // the epilogue decomposes pixels in 32 bits
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  const size_t elt = T == F32 ? 4 : 2;
  const int terms = T == F32 ? 2 : 1;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)op.K, (cuuint64_t)op.M};
  cuuint64_t strides[1] = {(cuuint64_t)op.K * elt};
  cuuint32_t box[2] = {(cuuint32_t)(128 / elt), (cuuint32_t)tcx::kTileM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(&map, T == F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                      const_cast<void *>(op.src), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  // output: per-warp 32-row x 16-column boxes (rows of 64 B fp32 / 32 B bf16)
  CUtensorMap map_out;
  cuuint64_t odims[2] = {(cuuint64_t)op.N, (cuuint64_t)op.M};
  cuuint64_t ostrides[1] = {(cuuint64_t)op.N * elt};
  cuuint32_t obox[2] = {(cuuint32_t)tcx::kSliceCols, 32};
  r = encode(&map_out, T == F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, op.dst, odims,
             ostrides, obox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             T == F32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;

  tcp::Params p;
  p.wimg = wimg, p.err = err, p.M = op.M;
  p.wait = op.wait_cycles > 0 ? op.wait_cycles : tcx::kWaitCycles;
  p.epi.bias = op.bias, p.epi.res = op.res, p.epi.coarse = op.coarse, p.epi.dst = op.dst;
  p.epi.N = op.N, p.epi.act = op.act, p.epi.OH = op.OH, p.epi.OW = op.OW, p.epi.n_tile = plan.n_tile;
  p.n_tiles = plan.n_tiles, p.slabs = plan.slabs;
  p.m_tiles = (int)((op.M + tcx::kTileM - 1) / tcx::kTileM);
  p.acc_stride = 32;
  while ((int)p.acc_stride < plan.n_tile) p.acc_stride <<= 1;
  p.tmem_cols = 2 * p.acc_stride;
  p.b_bytes = (uint32_t)(terms * plan.n_tile * 128);
  const size_t stage = terms * tcx::kAImage + p.b_bytes;
  p.bias_bytes = (uint32_t)(((size_t)op.N * 4 + 15) / 16 * 16);
  // lateral coarse ring: row stride = 16 mod 32 floats, so the two rows a
  // quarter-warp reads fall in different bank halves
  p.cs_ld = plan.n_tile + (plan.n_tile % 32 == 0 ? 16 : 0);
  // deepest coarse ring (2, 1 or none) that leaves at least 3 (else 2) A/B stages
  const size_t cs_stage = (size_t)tcx::kTileM * p.cs_ld * 4;
  const size_t fixed0 = 1024 + tcp::kEpiPw + p.bias_bytes + 8 * (3 * 8 + 9) + 16;
  p.cs_stages = 0;
  if (op.mode == 2)
    for (int want_ab = 3; want_ab >= 2 && !p.cs_stages; want_ab--)
      for (int cs = 2; cs >= 1; cs--)
        if (fixed0 + cs * cs_stage + want_ab * stage <= kSmemBudget) {
          p.cs_stages = cs;
          break;
        }
  p.cs_bytes = (uint32_t)(p.cs_stages * cs_stage);
  const size_t fixed = fixed0 + p.cs_bytes;
  int stages = (int)((kSmemBudget - fixed) / stage);
  if (stages > 6) stages = 6;
  if (stages < 2) return cudaErrorInvalidValue;
  p.stages = stages;
  // split-K when the launch has too few tiles to occupy the SMs and the tile's
  // K walk is long (pointwise only): each split takes spk slabs of the tile and
  // the partials fit the workspace. The reduction is a second launch, which at
  // small batches costs about as much as 6-8 slabs of one tile's serial walk
  // (measured), so shorter K walks are not split.
  p.ksplit = 1, p.spk = plan.slabs, p.ws = nullptr;
  {
    const long tiles = (long)p.m_tiles * p.n_tiles;
    const double tile_bytes = (double)tcx::kTileM * plan.n_tile * 4;
    if (op.mode == 0 && op.ws && plan.slabs >= kSplitMinSlabs && tiles * 2 <= sm_count()) {
      int want = (int)std::min<long>(plan.slabs, std::max<long>(1, sm_count() / tiles));
      for (; want > 1; want--) {
        const int spk = (plan.slabs + want - 1) / want, ks = (plan.slabs + spk - 1) / spk;
        if (tiles * ks * tile_bytes <= (double)op.ws_bytes) {
          p.spk = spk, p.ksplit = ks;
          break;
        }
      }
    }
    if (p.ksplit > 1) p.ws = op.ws;
  }
  const size_t smem = stages * stage + 1024 + tcp::kEpiPw + p.bias_bytes + p.cs_bytes + 8 * (3 * stages + 9) + 16;
  const bool split = p.ksplit > 1;
  if (T == F32) {
    if (op.mode == 2) return launch<float, 2, false>(map, map_out, p, smem, st);
    return split ? launch<float, 0, true>(map, map_out, p, smem, st) : launch<float, 0, false>(map, map_out, p, smem, st);
  }
  if (op.mode == 2) return launch<__nv_bfloat16, 2, false>(map, map_out, p, smem, st);
  return split ? launch<__nv_bfloat16, 0, true>(map, map_out, p, smem, st)
               : launch<__nv_bfloat16, 0, false>(map, map_out, p, smem, st);
}

}  // namespace gpu
}  // namespace illumina
