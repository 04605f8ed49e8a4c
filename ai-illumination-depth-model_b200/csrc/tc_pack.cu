// Weight images of the tensor-core kernels (tc_pw.cu, tc_dw.cu): the plan of
// a pointwise weight matrix's (n tile, 128-byte K slab) images and the device
// packing of the logical [N][K] fp32 weights into them, in the UMMA K-major
// SWIZZLE_128B layout (rows of 128 bytes, 8-row groups of 1024 bytes, 16-byte
// chunk c of row r stored at chunk c ^ (r & 7)): a TF32 hi/lo pair for fp32
// storage (w = hi + lo to ~2^-22 relative) or bf16.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "tc_common.cuh"

namespace illumina {
namespace gpu {

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
    const uint32_t hi = tcx::tf32_rna(v);
    const uint32_t lo = tcx::tf32_rna(v - __uint_as_float(hi));
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

}  // namespace gpu
}  // namespace illumina
