// Launch wrappers of the network kernels (implemented in net_kernels.cu and
// shade.cu). All pointers are device pointers; every wrapper returns the
// launch's cudaError_t.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace illumina {
namespace gpu {

enum StorageType { F32 = 0, BF16 = 1 };

struct PreprocessParams {
  float mean[3], inv_std[3], std[3];
  float exposure;
  int decode_srgb;
};

// Argument positions of the kernels whose pointer arguments a replayed CUDA
// graph re-targets (cudaGraphExecKernelNodeSetParams); they must match the
// parameter lists of k_preprocess and k_bilateral in net_kernels.cu.
constexpr int kPreprocessArgCount = 8, kPreprocessFramesArg = 0;
constexpr int kBilateralArgCount = 12, kBilateralDstArg = 9;

// frames (layout 0 planar / 1 rgba) -> input (n*S*S*4, storage T), luma (n*S*S
// f32), scene (n*S*S*4 f32, nullable).
cudaError_t preprocess(int T, const float *frames, int layout, int n, int S, const PreprocessParams &p,
                       void *input, float *luma, float *scene, cudaStream_t st);

// Preprocess fused into the stem conv (3x3, stride 2, 4 -> 16 channels, zero
// padding): frames -> stem output dst (n, S/2, S/2, 16) and luma, plus scene
// and the normalised input when those are non-null. Packed weights
// [3][3][4][16], bias [16].
struct StemParams {
  int layout, S, OH, OW, tiles_x, tiles_y, act;
  PreprocessParams pre;
  const float *w, *bias;
  void *dst;
  float *luma, *scene;
  void *input;
};
constexpr int kStemArgCount = 2, kStemFramesArg = 0;  // k_stem_fused(frames, StemParams)
cudaError_t stem_fused(int T, const float *frames, int layout, int n, int S, const PreprocessParams &pre,
                       const float *wpk, const float *bias, int act, void *dst, float *luma, float *scene, void *input,
                       cudaStream_t st);

// Dense conv: src (n,H,W,Cin) -> dst (n,OH,OW,Cout); packed weights [k][k][Cin][Cout].
cudaError_t conv(int T, const void *src, int n, int H, int W, int Cin, const float *wpk, const float *bias,
                 int Cout, int k, int stride, int act, void *dst, cudaStream_t st);

struct GemmOp {
  int mode = 0;                  // 0 pointwise, 1 depthwise->pointwise, 2 lateral
  const void *src = nullptr;     // pw: [M][K]; dw: (n,H,W,K); lateral: skip [M][K]
  const float *w = nullptr;      // [N][K] f32
  const float *bias = nullptr;   // [N]
  const void *res = nullptr;     // [M][N] or null
  void *dst = nullptr;           // [M][N]
  int n = 1;         // frames
  int H = 0, W = 0;  // dw: input spatial; lateral: output spatial
  int OH = 0, OW = 0;// output spatial (dw) ; pw: OH*OW*n = M
  long M = 0;
  int N = 0, K = 0;
  int act = 0, mid_act = 0;
  int ks = 0, stride = 1;        // dw
  const float *dw_w = nullptr;   // packed [ks*ks][K]
  const float *dw_b = nullptr;   // [K]
  const void *coarse = nullptr;  // lateral: (n, H/2, W/2, N)
  // Optional split-K workspace of the tensor-core kernels: fp32 partial tiles
  // of the K splits, summed by a reduction launch that follows the op's
  // kernel. Without it the kernels do not split K.
  float *ws = nullptr;
  size_t ws_bytes = 0;
  // Optional depth head on the op's output (dw->pw on the tensor engine):
  // head_dst[m] = sigmoid(head_b + sum_n dst[m][n] * head_w[n]), folded into
  // the epilogue when the launch allows it, else a separate head launch.
  const float *head_w = nullptr;
  float head_b = 0.0f;
  float *head_dst = nullptr;
  // Tensor engine: cycles a pipeline wait may take before the kernel gives up
  // and sets *err (0 = the default, ~1 s).
  long long wait_cycles = 0;
};

cudaError_t gemm(int T, const GemmOp &op, cudaStream_t st);

// Tensor-core (tcgen05) engine for the same ops. The weights of each op are
// pre-packed (tc_pack.cu) into swizzled per-(n tile, K slab) shared-memory
// images: tf32 hi/lo pairs for fp32 storage, bf16 for bf16 storage.
struct TcWeights {
  int N = 0, K = 0;
  int n_tile = 0, n_tiles = 0, slabs = 0;  // accumulator columns per CTA, tiles along N, K slabs
  uint32_t tmem_cols = 0;
  size_t bytes = 0;                         // size of the packed images
  int ks = 0;                               // depthwise kernel size (dw->pw ops)
  size_t dw_off = 0, dw_bytes = 0;          // depthwise slab blocks after the images
};
TcWeights tc_plan(int T, int N, int K);
cudaError_t tc_pack(int T, const float *w, int N, int K, const TcWeights &plan, uint8_t *out, cudaStream_t st);
// Persistent warp-specialised variant for pointwise (mode 0) and lateral
// (mode 2): TMA A tiles, bulk-copied weight images, double-buffered TMEM
// accumulators (tc_pw.cu).
cudaError_t tc_pw(int T, const GemmOp &op, const TcWeights &plan, const uint8_t *wimg, int *err, cudaStream_t st);

// Depthwise->pointwise (mode 1) on the persistent kernel of tc_dw.cu: the
// plan adds per-slab depthwise weight blocks ([slab][ks*ks + 1][slab_c] f32,
// taps then bias) after the pointwise images; tc_pack_dw fills them from the
// packed [ks*ks][K] taps and the [K] bias.
TcWeights tc_plan_dw(int T, int N, int K, int ks);
cudaError_t tc_pack_dw(int T, const float *dw_w, const float *dw_b, const TcWeights &plan, uint8_t *out,
                       cudaStream_t st);
cudaError_t tc_dw(int T, const GemmOp &op, const TcWeights &plan, const uint8_t *wimg, int *err, cudaStream_t st);

// Tensor-core dispatch: pointwise / lateral on tc_pw, depthwise->pointwise on tc_dw.
inline cudaError_t tc_op(int T, const GemmOp &op, const TcWeights &plan, const uint8_t *wimg, int *err,
                         cudaStream_t st) {
  return op.mode == 1 ? tc_dw(T, op, plan, wimg, err, st) : tc_pw(T, op, plan, wimg, err, st);
}

// Head: src (M,C) storage T -> dst1 (M) f32 disparity (1 channel) and/or
// dst4 (M*4) f32 broadcast.
cudaError_t head(int T, const void *src, long M, int C, const float *w, float bias, float *dst1, float *dst4,
                 cudaStream_t st);

struct BilateralParams {
  float range_sigma, base_alpha, sensitivity;
};
// low1: (n, lh, lw) f32; luma: (n, 2lh, 2lw) f32. dst: (n, 2lh, 2lw) f32.
// history/out_tex (S*S*4 f32, n must be 1) enable the temporal blend.
cudaError_t bilateral(const float *low1, int n, int lh, int lw, const float *luma, const BilateralParams &p,
                      float *dst, const float *history, float *out_tex, cudaStream_t st);

// Op-API adaptors: low with channel stride `low_c`, guide with `guide_c`
// channels of linear colour.
cudaError_t bilateral_strided(const float *low, int lh, int lw, int low_c, const float *guide, int guide_c,
                              float range_sigma, float *dst, cudaStream_t st);

// Weight packing (logical .idm layouts -> kernel layouts), optional bf16 rounding.
cudaError_t pack_dw(const float *w, int C, int k, float *out, int round_bf16, cudaStream_t st);
cudaError_t pack_conv(const float *w, int O, int I, int k, float *out, int round_bf16, cudaStream_t st);
cudaError_t copy_round(const float *w, long n, float *out, int round_bf16, cudaStream_t st);

// Expand a 1-channel map to 4 channels (debugTensor of depth_low).
cudaError_t expand4(const float *src, long n, float *dst4, cudaStream_t st);
// Bilateral guide of a given fp32 network input (n*S*S x 4): its channel 3.
cudaError_t input_luma(const float *input, long px, float *luma, cudaStream_t st);
// Convert storage T -> f32.
cudaError_t to_f32(int T, const void *src, long n, float *dst, cudaStream_t st);

cudaError_t generate_frames(int kind, uint32_t seed0, int n, int S, float *out, cudaStream_t st);
cudaError_t checksums(const float *maps, int n, long count, uint64_t *sum64, double *fsum, cudaStream_t st);

// Shading (shade.cu)
struct ShadeParams {
  float camera[4], toggles[4], ambient[4], misc[4], fog[4], size[4], debug[4], grade[4];
};
struct ShadeLight {
  float position[4], color[4], direction[4], params[4];
};
struct ShadeSteps {
  int contact, ao_dirs, ao_steps, volumetric;
};
cudaError_t shade(const float *depth, int dw, int dh, int dch, const float *albedo, int aw, int ah,
                  const ShadeLight *lights, const ShadeParams &P, const ShadeSteps &steps, int out_w, int out_h,
                  float *hdr, uint8_t *rgba8, cudaStream_t st);
cudaError_t resize_bilinear(const float *src, int sw, int sh, float *dst, int dw, int dh, cudaStream_t st);

// 8-bit RGBA source (n x sh x sw x 4) sampled at the network's resolution with
// the uv transform of makePreprocess -> planar float frames (n x 3 x size x size).
cudaError_t sample_source(const uint8_t *rgba8, int n, int sw, int sh, const float uv_scale[2],
                          const float uv_offset[2], int mirror, int size, float *frames, cudaStream_t st);

// Procedural scene and depth metrics (scene.cu). SceneParams is the scene's
// uniform block (camera.xyz + time, look-at.xyz + tan(fovY/2), aspect, far,
// key-light azimuth, variant); one launch renders up to kSceneBatch frames
// whose uniforms travel in the kernel's parameter block.
struct SceneParams {
  float camera[4], focus[4], options[4];
};
constexpr int kSceneBatch = 64;
struct SceneBatch {
  int first;
  SceneParams frames[kSceneBatch];
};
struct DepthMetrics {
  long long samples;
  double abs_rel, rmse, delta1, delta2, delta3, scale, shift;
};
// n frames of w x h: rgb (n x 3 x h x w, nullable), rgba8 (n x h x w x 4,
// nullable), truth (n x h x w x 2 float: depth, hit; nullable). params: host array of n.
cudaError_t scene_render(const SceneParams *params, int n, int w, int h, float *rgb, uint8_t *rgba8, float *truth,
                         cudaStream_t st);
// pred: n maps of `plane` texels of pred_ch floats (channel 0 read); truth: n x plane x 2; out: n (device).
cudaError_t evaluate_depth(const float *pred, int pred_ch, const float *truth, int n, long plane, DepthMetrics *out,
                           cudaStream_t st);

}  // namespace gpu
}  // namespace illumina
