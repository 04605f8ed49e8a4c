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
// Roles inside one CTA (480 threads, one CTA per SM, items strided by grid):
//   warp 0        halo producer: per (item, slab) one 4-D TMA load of the
//                 input halo ((th-1)*S+KS rows x (tw-1)*S+KS columns x one
//                 slab, unswizzled; coordinates outside the frame read as
//                 zero, which is the depthwise zero padding) plus a bulk copy
//                 of the slab's depthwise taps and bias into the `H` ring.
//   warp 14       weight producer: bulk copies of the pre-swizzled pointwise
//                 weight images into the `G` ring, or once into a resident
//                 region when all of the op's images fit in shared memory.
//   warps 2-9     depthwise, in `ng` groups of four warps that take the
//                 (item, slab) steps in turn (group g takes steps g, g+ng, ..),
//                 so one group's shared-memory latency hides behind the
//                 other's arithmetic. Each thread owns 4 channels of a run of
//                 P adjacent output pixels, accumulates bias + sum over
//                 (ky, kx) of x * w from the halo (the reference's tap order),
//                 applies the mid activation and writes the A image (TF32
//                 hi/lo pair for fp32 storage, bf16 for bf16 storage).
//   warp 1        one thread issues tcgen05.mma into one of two TMEM
//                 accumulators and commits each G stage back to the ring.
//   warps 10-13   epilogue (tcx::epilogue_rows), one warp per TMEM lane
//                 quarter: bias and residual loaded before the accumulator
//                 is waited for, then activation and store; then release
//                 the accumulator.
// A ring stage is always used by the same depthwise group (the ring depths
// are multiples of ng), so a group's own previous use of a stage orders its
// parity waits. Every mbarrier wait is bounded; a role that gives up records
// it in *err and leaves its loop; the producers wait (bounded) for their own
// copies and the MMA thread for its own MMAs before all roles meet and TMEM
// is released.
#include <cudaTypedefs.h>

#include <array>
#include <cmath>
#include <map>
#include <mutex>

#include "kernels.h"
#include "tc_common.cuh"
#include "tc_dw_kernel.cuh"

namespace illumina {
namespace gpu {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

namespace tcd {

// [K*K][C] packed depthwise taps + [C] bias -> per slab blocks of
// (K*K + 1) rows x slab_c floats, zero past C.
__global__ void k_pack_dw_slabs(const float *dw_w, const float *dw_b, int C, int kk, int slab_c, int slabs,
                                float *out) {
  const long total = (long)slabs * (kk + 1) * slab_c;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int c = (int)(i % slab_c);
  const long q = i / slab_c;
  const int t = (int)(q % (kk + 1)), s = (int)(q / (kk + 1));
  const int ch = s * slab_c + c;
  out[i] = ch < C ? (t < kk ? dw_w[(long)t * C + ch] : dw_b[ch]) : 0.0f;
}


// Instantiated in tc_dw_{f32,bf16}{,_split}.cu.
extern template cudaError_t launch_all<float, false>(int, int, int, const CUtensorMap &, const CUtensorMap &,
                                               const Params &, size_t, cudaStream_t);
extern template cudaError_t launch_all<float, true>(int, int, int, const CUtensorMap &, const CUtensorMap &,
                                               const Params &, size_t, cudaStream_t);
extern template cudaError_t launch_all<__nv_bfloat16, false>(int, int, int, const CUtensorMap &, const CUtensorMap &,
                                               const Params &, size_t, cudaStream_t);
extern template cudaError_t launch_all<__nv_bfloat16, true>(int, int, int, const CUtensorMap &, const CUtensorMap &,
                                               const Params &, size_t, cudaStream_t);

}  // namespace tcd

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

namespace {

using tcd::kSmemBudget;

size_t align_to(size_t v, size_t a) { return (v + a - 1) / a * a; }
// Bytes of one fp32 split-K partial tile of n_tile columns.
double kTileMBytes(int n_tile) { return (double)tcx::kTileM * n_tile * 4; }

struct DwTiling {
  int tw = 0, th = 0, P = 0, iw = 0, ih = 0, sh = 0, sg = 0, b_res = 0, ng = 0, ksplit = 1, spk = 0;
  size_t smem = 0;
  double cost = 0;
};

// Patch shape, run length P, depthwise groups, ring depths, weight residency
// and K split for one launch, by a per-SM cycle estimate of the launch's wall
// time: units (item x K split) spread over the SMs in waves; per (unit, slab)
// a depthwise group needs the halo copy (~1500 cycles of latency plus 64 B per
// cycle) and its arithmetic (~6 cycles per instruction of one warp: the groups
// are latency bound), overlapped when the group owns two H stages and
// serialised otherwise; `ng` groups interleave; the MMAs, the halo bandwidth
// and the shared-memory wavefronts (depthwise loads and stores, UMMA operand
// reads, TMA writes) bound the step from below. A split item adds the partial
// tile store, and the launch a reduction kernel whose (8-row, 16-column)
// units spread over every SM.
DwTiling plan_tiling(int T, long n_frames, int OH, int OW, int KS, int S, const TcWeights &w, bool has_res,
                     size_t ws_bytes) {
  const bool f32 = T == F32;
  const size_t bias_bytes = align_to((size_t)w.N * 4, 16);
  const int terms = f32 ? 2 : 1, slab_c = f32 ? 32 : 64, cgs = slab_c / 4;
  const size_t dw_bytes = (size_t)(KS * KS + 1) * slab_c * 4;
  const size_t a_bytes = (size_t)terms * tcx::kAImage, b_bytes = (size_t)terms * w.n_tile * 128;
  const size_t res_total = (size_t)w.n_tiles * w.slabs * b_bytes;
  // the last slab computes and multiplies only its 32-byte K chunks that hold
  // channels; a one-slab op is costed at that width
  const int nk = w.slabs == 1 ? (int)((w.K * (f32 ? 4 : 2) + 31) / 32) : 4;
  int cgs_eff = cgs;
  if (w.slabs == 1)
    for (cgs_eff = 1; cgs_eff < nk * (f32 ? 2 : 4);) cgs_eff <<= 1;
  const double mma = (f32 ? 1000.0 + 8.0 * w.n_tile : 300.0 + 2.0 * w.n_tile) * nk / 4.0;
  const double mma_rd = (f32 ? 512.0 + 4.0 * w.n_tile : 128.0 + 1.0 * w.n_tile) * nk / 4.0;
  const double epi = (w.n_tile / 16.0) * (has_res ? 1400.0 : 700.0);
  const double G = sm_count();
  DwTiling best;
  const int Ps[4] = {8, 7, 4, 2};
  for (int P : Ps) {
    for (int tw = P; tw <= 128 && tw < OW + P; tw += P) {
      const int iw = (tw - 1) * S + KS;
      if (iw > 256) break;
      for (int th_div = 1; th_div <= 4; th_div *= 2) {
        const int th_max = std::max(1, 128 / tw / th_div);
        if (th_div > 1 && th_max == std::max(1, 128 / tw / (th_div / 2))) continue;
        const int tiles_y = (OH + th_max - 1) / th_max;
        const int th = (OH + tiles_y - 1) / tiles_y;
        const int ih = (th - 1) * S + KS;
        if (ih > 256) continue;
        const double items = (double)n_frames * ((OW + tw - 1) / tw) * tiles_y * w.n_tiles;
        const size_t halo = (size_t)iw * ih * 128;
        const size_t h_stage = align_to(halo + dw_bytes, 1024);
        const int units = th * (tw / P) * cgs_eff;
        const int rounds = (units + tcd::kGroupWarps * 32 - 1) / (tcd::kGroupWarps * 32);
        const int span = (P - 1) * S + KS;
        const double xf = 6.0 * rounds * (KS * (4.0 * P * KS + span + KS) + 40.0 * P);
        const double lat = 1500.0 + halo / 64.0, bw = halo / 64.0;
        const double smem_rd = units / 8.0 * KS * (span + KS) + units * P * terms / 8.0 + mma_rd + iw * ih;
        for (int b_res = 1; b_res >= 0; b_res--) {
          const size_t g_stage = a_bytes + (b_res ? 0 : b_bytes);
          for (int ng = tcd::kMaxGroups; ng >= 1; ng--) {
            for (int sh = ng; sh <= 4; sh += ng) {
              for (int sg = ng; sg <= 4; sg += ng) {
                const size_t smem = 1024 + sh * h_stage + sg * g_stage + (b_res ? res_total : 0) + tcd::kEpiBytes +
                                    bias_bytes + 8 * (2 * sh + 3 * sg + 6) + 16;
                if (smem > kSmemBudget) continue;
                double group = sh / ng >= 2 ? std::fmax(lat, xf) : lat + xf;
                if (sg / ng < 2) group += mma;
                const double per_slab = std::fmax(std::fmax(group / ng, mma), std::fmax(bw, smem_rd));
                int last_ks = 0;
                for (int want = 1; want <= std::min(w.slabs, 32); want++) {
                  const int spk = (w.slabs + want - 1) / want;
                  const int ks = (w.slabs + spk - 1) / spk;
                  if (ks == last_ks) continue;
                  last_ks = ks;
                  if (ks > 1 && items * ks * kTileMBytes(w.n_tile) > (double)ws_bytes) break;
                  const double nunits = items * ks;
                  const double waves = std::ceil(nunits / G);
                  // split: partial store per unit, then the reduction launch
                  // (~4000 cycles to start behind this kernel) whose latency-bound
                  // (8-row, 16-column) units (four splits' loads in flight per
                  // unit) run one per warp, 32 warps per SM
                  const double red_units = std::ceil(th * tw / 8.0) * std::ceil(w.n_tile / 16.0);
                  const double per_unit = std::fmax(spk * per_slab, epi) + (ks > 1 ? 300.0 * w.n_tile / 16 : 0.0);
                  const double red = ks > 1 ? 4000.0 + std::ceil(items * red_units / (G * 32.0)) *
                                                           (std::ceil(ks / 4.0) * 700.0 + 150.0)
                                            : 0.0;
                  // patches of <= 64 pixels (at most half an MMA tile) run slower than the
                  // model predicts when there are waves of items: per-item costs it does not
                  // count (measured at batch 256: bf16 e5a.dw_project 8x8 patches 0.653 ms,
                  // 14x8 0.529 ms; fp32 d2.refine 8x8 0.230 ms, the next plan 0.148 ms); with
                  // fewer items than two waves the small patches' parallelism wins
                  const double small_patch = tw * th <= 64 && items >= 2 * G ? 1.2 : 1.0;
                  const double cost =
                      (waves * per_unit + red) * (b_res ? 0.99 : 1.0) * (1.0 - 0.001 * (sh + sg)) * small_patch;
                  if (best.tw == 0 || cost < best.cost) {
                    best.tw = tw, best.th = th, best.P = P, best.iw = iw, best.ih = ih, best.ng = ng;
                    best.sh = sh, best.sg = sg, best.b_res = b_res, best.smem = smem, best.cost = cost;
                    best.ksplit = ks, best.spk = spk;
                  }
                }
              }
            }
          }
        }
      }
    }
  }
  return best;
}

// Shared memory of tiling `t` for storage type T (the layout plan_tiling costs).
size_t dw_smem(int T, const DwTiling &t, int KS, const TcWeights &w) {
  const bool f32 = T == F32;
  const int terms = f32 ? 2 : 1, slab_c = f32 ? 32 : 64;
  const size_t dw_bytes = (size_t)(KS * KS + 1) * slab_c * 4;
  const size_t a_bytes = (size_t)terms * tcx::kAImage, b_bytes = (size_t)terms * w.n_tile * 128;
  const size_t h_stage = align_to((size_t)t.iw * t.ih * 128 + dw_bytes, 1024);
  const size_t g_stage = a_bytes + (t.b_res ? 0 : b_bytes);
  return 1024 + t.sh * h_stage + t.sg * g_stage + (t.b_res ? (size_t)w.n_tiles * w.slabs * b_bytes : 0) +
         tcd::kEpiBytes + align_to((size_t)w.N * 4, 16) + 8 * (2 * t.sh + 3 * t.sg + 6) + 16;
}

// plan_tiling is a few-thousand-candidate search; launches of one shape reuse it.
DwTiling cached_tiling(int T, long n_frames, int OH, int OW, int KS, int S, const TcWeights &w, bool has_res,
                       size_t ws_bytes) {
  using Key = std::array<long, 12>;
  static std::mutex mu;
  static std::map<Key, DwTiling> cache;
  const Key key{T, n_frames, OH, OW, KS, S, w.N, w.K, has_res ? 1 : 0, (long)ws_bytes, 0, sm_count()};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  const DwTiling t = plan_tiling(T, n_frames, OH, OW, KS, S, w, has_res, ws_bytes);
  cache.emplace(key, t);
  return t;
}

}  // namespace

TcWeights tc_plan_dw(int T, int N, int K, int ks) {
  TcWeights w = tc_plan(T, N, K);
  const int slab_c = T == F32 ? 32 : 64;
  w.ks = ks;
  w.dw_off = align_to(w.bytes, 1024);
  w.dw_bytes = (size_t)w.slabs * (ks * ks + 1) * slab_c * 4;
  w.bytes = w.dw_off + w.dw_bytes;
  return w;
}

cudaError_t tc_pack_dw(int T, const float *dw_w, const float *dw_b, const TcWeights &plan, uint8_t *out,
                       cudaStream_t st) {
  const int slab_c = T == F32 ? 32 : 64;
  const long total = (long)plan.slabs * (plan.ks * plan.ks + 1) * slab_c;
  if (total <= 0 || plan.dw_bytes == 0) return cudaErrorInvalidValue;
  tcd::k_pack_dw_slabs<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
      dw_w, dw_b, plan.K, plan.ks * plan.ks, slab_c, plan.slabs, reinterpret_cast<float *>(out + plan.dw_off));
  return cudaGetLastError();
}

cudaError_t tc_dw(int T, const GemmOp &op, const TcWeights &plan, const uint8_t *wimg, int *err, cudaStream_t st) {
  if (op.M <= 0) return cudaSuccess;
  if (op.mode != 1 || plan.dw_bytes == 0 || plan.ks != op.ks) return cudaErrorInvalidValue;
  if ((op.ks != 3 && op.ks != 5) || (op.stride != 1 && op.stride != 2)) return cudaErrorInvalidValue;
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  DwTiling tl = cached_tiling(T, op.n, op.OH, op.OW, op.ks, op.stride, plan, op.res != nullptr,
                              op.ws ? op.ws_bytes : 0);
  if (T == BF16 && op.stride == 2) {
    // stride-2 (expand) ops in bf16 take the patch, groups and rings the fp32
    // model picks for the same op, which measured 10-35 % faster than the bf16
    // model's choice (batch 256: e2 0.693 -> 0.482 ms, e4 0.315 -> 0.206,
    // e6 0.141 -> 0.101, e8 0.102 -> 0.092); the cycle model has no per-item
    // or shared-memory footprint costs, which decide between these plans
    const TcWeights w32 = tc_plan_dw(F32, plan.N, plan.K, op.ks);
    DwTiling t = cached_tiling(F32, op.n, op.OH, op.OW, op.ks, op.stride, w32, op.res != nullptr,
                               op.ws ? op.ws_bytes : 0);
    if (t.tw != 0 && t.ksplit == 1) {
      t.spk = plan.slabs;
      t.smem = dw_smem(T, t, op.ks, plan);
      if (t.smem <= kSmemBudget) tl = t;
    }
  }
  if (tl.tw == 0) return cudaErrorInvalidValue;

  const size_t elt = T == F32 ? 4 : 2;
  const int slab_c = T == F32 ? 32 : 64;
  CUtensorMap map;
  cuuint64_t dims[4] = {(cuuint64_t)op.K, (cuuint64_t)op.W, (cuuint64_t)op.H, (cuuint64_t)op.n};
  cuuint64_t strides[3] = {(cuuint64_t)op.K * elt, (cuuint64_t)op.W * op.K * elt,
                           (cuuint64_t)op.H * op.W * op.K * elt};
  cuuint32_t box[4] = {(cuuint32_t)slab_c, (cuuint32_t)tl.iw, (cuuint32_t)tl.ih, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode(&map, T == F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                      const_cast<void *>(op.src), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  // output: 16-column slices of a th x tw patch, rows of 64 B (fp32) or 32 B
  // (bf16) in the epilogue's swizzled slice buffers
  CUtensorMap map_out;
  cuuint64_t odims[4] = {(cuuint64_t)op.N, (cuuint64_t)op.OW, (cuuint64_t)op.OH, (cuuint64_t)op.n};
  cuuint64_t ostrides[3] = {(cuuint64_t)op.N * elt, (cuuint64_t)op.OW * op.N * elt,
                            (cuuint64_t)op.OH * op.OW * op.N * elt};
  cuuint32_t obox[4] = {(cuuint32_t)tcx::kSliceCols, (cuuint32_t)tl.tw, (cuuint32_t)tl.th, 1};
  r = encode(&map_out, T == F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, op.dst, odims,
             ostrides, obox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             T == F32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;

  const int terms = T == F32 ? 2 : 1;
  tcd::Params p;
  p.wimg = wimg, p.dwblk = wimg + plan.dw_off, p.err = err;
  p.wait = op.wait_cycles > 0 ? op.wait_cycles : tcx::kWaitCycles;
  p.epi.bias = op.bias, p.epi.res = op.res, p.epi.coarse = nullptr, p.epi.dst = op.dst;
  p.epi.N = op.N, p.epi.act = op.act, p.epi.OH = op.OH, p.epi.OW = op.OW, p.epi.n_tile = plan.n_tile;
  p.tiles_x = (op.OW + tl.tw - 1) / tl.tw;
  p.tiles_y = (op.OH + tl.th - 1) / tl.th;
  p.n_tiles = plan.n_tiles, p.slabs = plan.slabs;
  const long items = (long)op.n * p.tiles_x * p.tiles_y * plan.n_tiles;
  const long total = items * tl.ksplit;
  if (total > 0x7fffffffL) return cudaErrorInvalidValue;
  p.items = (int)items, p.ksplit = tl.ksplit, p.spk = tl.spk, p.total = (int)total;
  p.ws = op.ws;
  p.tw = tl.tw, p.th = tl.th, p.iw = tl.iw, p.mid_act = op.mid_act;
  {
    const int k_last = op.K - (plan.slabs - 1) * slab_c;  // channels in the last slab
    p.nk_last = (int)((k_last * elt + 31) / 32);
    // depthwise width of the last slab: its chunks' channel groups, rounded up
    // to a power of two so a warp's halo reads still cover every bank
    p.cg_last = 1;
    while (p.cg_last < p.nk_last * 8 / (int)elt) p.cg_last <<= 1;
    if (k_last <= 0 || p.nk_last > 4) return cudaErrorInvalidValue;
  }
  p.sh = tl.sh, p.sg = tl.sg, p.b_res = tl.b_res, p.ng = tl.ng;
  // a second epilogue team (one per TMEM accumulator, so two items'
  // epilogues run at once) when its buffers fit beside the planned rings
  p.teams = tl.ksplit == 1 && tl.smem + tcd::kEpiBytes <= kSmemBudget ? 2 : 1;
  const size_t smem = tl.smem + (p.teams - 1) * tcd::kEpiBytes;
  // the head folds into the TMA-store epilogue when one tile holds every column
  const bool fold_head = op.head_dst && tl.ksplit == 1 && plan.n_tiles == 1 && plan.n_tile <= 2 * tcx::kSliceCols;
  if (fold_head) p.epi.head_w = op.head_w, p.epi.head_b = op.head_b, p.epi.head_dst = op.head_dst;
  p.halo_bytes = (uint32_t)(tl.iw * tl.ih * 128);
  p.dw_bytes = (uint32_t)((op.ks * op.ks + 1) * slab_c * 4);
  p.h_stage = (uint32_t)align_to(p.halo_bytes + p.dw_bytes, 1024);
  p.b_bytes = (uint32_t)(terms * plan.n_tile * 128);
  p.g_stage = (uint32_t)(terms * tcx::kAImage + (tl.b_res ? 0 : p.b_bytes));
  p.acc_stride = 32;
  while ((int)p.acc_stride < plan.n_tile) p.acc_stride <<= 1;
  p.tmem_cols = 2 * p.acc_stride;
  p.bias_bytes = (uint32_t)align_to((size_t)op.N * 4, 16);
  const bool split = tl.ksplit > 1;
  cudaError_t e;
  if (T == F32)
    e = split ? tcd::launch_all<float, true>(op.ks, op.stride, tl.P, map, map_out, p, smem, st)
              : tcd::launch_all<float, false>(op.ks, op.stride, tl.P, map, map_out, p, smem, st);
  else
    e = split ? tcd::launch_all<__nv_bfloat16, true>(op.ks, op.stride, tl.P, map, map_out, p, smem, st)
              : tcd::launch_all<__nv_bfloat16, false>(op.ks, op.stride, tl.P, map, map_out, p, smem, st);
  if (e == cudaSuccess && op.head_dst && !fold_head)
    e = head(T, op.dst, op.M, op.N, op.head_w, op.head_b, op.head_dst, nullptr, st);
  return e;
}

}  // namespace gpu
}  // namespace illumina
