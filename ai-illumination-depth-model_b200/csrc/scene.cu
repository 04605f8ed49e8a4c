// Procedural SDF scene and depth metrics on the GPU.
//
// k_scene is the ray-marched signed-distance scene of src/scene/procedural.ts
// (sdSphere/sdBox/smoothUnion :36-62, the scene map :70-125, calcNormal
// :128-137, softShadow :140-158, materialColor :160-175, sceneFragment
// :191-273), one thread per pixel, with the reference's constants (96 march
// steps, 28 shadow steps). Instead of an rgba8unorm render target and an
// rgba16float truth texture it writes, per frame, any of: the 8-bit colour as
// the network's planar float input (value / 255, what sampling the rgba8unorm
// source texture returns), the 8-bit RGBA image itself, and the exact (depth,
// hit) pair in float32. A launch renders a batch of frames, each with its own
// uniforms, so ground-truth RGB/depth pairs come out at batch rate.
//
// k_metrics is evaluateDepth (src/scene/metrics.ts:66-161) on device maps: the
// least-squares (scale, shift) in disparity space over valid pixels (hit,
// 0.05 < depth <= 25), then AbsRel, RMSE and delta1..3 of the aligned depth,
// all in double. A cluster of 8 CTAs per frame reads the frame twice (the
// second pass from L2) and reduces in a fixed order through distributed shared
// memory, so results are deterministic; they differ from the reference's
// sequential sums only in double rounding.
#include <cooperative_groups.h>
#include <cstdint>

#include "kernels.h"

namespace illumina {
namespace gpu {

namespace {

struct f3 {
  float x, y, z;
};
__device__ __forceinline__ f3 mk(float x, float y, float z) { return {x, y, z}; }
__device__ __forceinline__ f3 operator+(f3 a, f3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
__device__ __forceinline__ f3 operator-(f3 a, f3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
__device__ __forceinline__ f3 operator*(float s, f3 a) { return {s * a.x, s * a.y, s * a.z}; }
__device__ __forceinline__ float dot3(f3 a, f3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ float len3(f3 a) { return sqrtf(dot3(a, a)); }
__device__ __forceinline__ f3 norm3(f3 a) {
  float l = len3(a);
  return {a.x / l, a.y / l, a.z / l};
}
__device__ __forceinline__ f3 cross3(f3 a, f3 b) {
  return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
__device__ __forceinline__ float clampf(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }
__device__ __forceinline__ float mixf(float a, float b, float t) { return a * (1.0f - t) + b * t; }

__device__ __forceinline__ float sd_sphere(f3 p, float r) { return len3(p) - r; }

__device__ __forceinline__ float sd_box(f3 p, f3 b) {
  f3 q = mk(fabsf(p.x), fabsf(p.y), fabsf(p.z)) - b;
  return len3(mk(fmaxf(q.x, 0.0f), fmaxf(q.y, 0.0f), fmaxf(q.z, 0.0f))) + fminf(fmaxf(q.x, fmaxf(q.y, q.z)), 0.0f);
}

__device__ __forceinline__ float smooth_union(float a, float b, float k) {
  float h = clampf(0.5f + (0.5f * (b - a)) / k, 0.0f, 1.0f);
  return mixf(b, a, h) - k * h * (1.0f - h);
}

// Time-dependent parts of the scene map, computed once per pixel.
struct Anim {
  float bob, near_x;
};

template <bool MATERIAL>
__device__ __forceinline__ float scene_map(f3 p, const Anim &an, float *mat) {
  float dist = p.y + 1.0f + 0.06f * sinf(p.x * 0.7f) * cosf(p.z * 0.6f);
  float material = 1.0f;
  float a = sd_sphere(p - mk(-0.35f, -0.25f + an.bob, -2.1f), 0.62f);
  float b = sd_sphere(p - mk(0.4f, -0.45f + an.bob * 0.6f, -1.75f), 0.42f);
  float blob = smooth_union(a, b, 0.35f);
  if (blob < dist) {
    dist = blob;
    material = 2.0f;
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float x = -2.4f + (float)i * 1.55f;
    const float z = -4.6f - (float)((i * 7) % 5) * 0.55f;
    const float h = 0.9f + 0.35f * (float)((i * 3) % 4);
    float box = sd_box(p - mk(x, -1.0f + h, z), mk(0.22f, h, 0.22f));
    if (box < dist) {
      dist = box;
      material = 3.0f;
    }
  }
  float arch = fmaxf(sd_box(p - mk(0.2f, 0.6f, -8.5f), mk(2.6f, 1.9f, 0.3f)),
                     -sd_sphere(p - mk(0.2f, -0.4f, -8.5f), 1.7f));
  if (arch < dist) {
    dist = arch;
    material = 4.0f;
  }
  float nr = sd_sphere(p - mk(an.near_x, 0.15f, -1.15f), 0.28f);
  if (nr < dist) {
    dist = nr;
    material = 5.0f;
  }
  if (MATERIAL) *mat = material;
  return dist;
}

__device__ f3 calc_normal(f3 p, const Anim &an) {
  const float e = 0.0015f;
  float dx = scene_map<false>(p + mk(e, 0, 0), an, nullptr) - scene_map<false>(p - mk(e, 0, 0), an, nullptr);
  float dy = scene_map<false>(p + mk(0, e, 0), an, nullptr) - scene_map<false>(p - mk(0, e, 0), an, nullptr);
  float dz = scene_map<false>(p + mk(0, 0, e), an, nullptr) - scene_map<false>(p - mk(0, 0, e), an, nullptr);
  return norm3(mk(dx, dy, dz));
}

__device__ float soft_shadow(f3 origin, f3 dir, const Anim &an) {
  float res = 1.0f, t = 0.04f;
  for (int i = 0; i < 28; i++) {
    float h = scene_map<false>(origin + t * dir, an, nullptr);
    res = fminf(res, (12.0f * h) / t);
    t += clampf(h, 0.02f, 0.4f);
    if (res < 0.002f || t > 12.0f) break;
  }
  return clampf(res, 0.0f, 1.0f);
}

__device__ __forceinline__ f3 material_color(float material, f3 p) {
  if (material < 1.5f) {
    float c = floorf(p.x * 0.8f) + floorf(p.z * 0.8f);
    float hc = c * 0.5f;
    float checker = (hc - floorf(hc)) < 0.25f ? 0.34f : 0.18f;
    return mk(checker * 1.05f, checker, checker * 0.92f);
  }
  if (material < 2.5f) return mk(0.82f, 0.28f, 0.22f);
  if (material < 3.5f) return mk(0.28f, 0.42f, 0.6f);
  if (material < 4.5f) return mk(0.55f, 0.5f, 0.44f);
  return mk(0.9f, 0.76f, 0.32f);
}

__global__ void __launch_bounds__(128) k_scene(SceneBatch batch, int w, int h, float *__restrict__ rgb,
                                               uint8_t *__restrict__ rgba8, float *__restrict__ truth) {
  const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
  if (x >= w || y >= h) return;
  const int f = blockIdx.z;
  const SceneParams &P = batch.frames[f];
  const long frame = (long)batch.first + f;
  const float time = P.camera[3];
  const Anim an = {0.12f * sinf(time * 0.9f), 1.25f + 0.25f * sinf(time * 0.5f)};

  const f3 origin = mk(P.camera[0], P.camera[1], P.camera[2]);
  const f3 forward = norm3(mk(P.focus[0], P.focus[1], P.focus[2]) - origin);
  const f3 right = norm3(cross3(forward, mk(0, 1, 0)));
  const f3 up = cross3(right, forward);
  const float u = ((float)x + 0.5f) / (float)w, v = ((float)y + 0.5f) / (float)h;
  const float ndc_x = u * 2.0f - 1.0f, ndc_y = 1.0f - v * 2.0f;
  const f3 dir = norm3(((ndc_x * P.options[0] * P.focus[3]) * right + (ndc_y * P.focus[3]) * up) + forward);

  float t = 0.02f, material = 0.0f;
  bool hit = false;
  for (int i = 0; i < 96; i++) {
    float m;
    float s = scene_map<true>(origin + t * dir, an, &m);
    if (s < 0.0015f * t) {
      hit = true;
      material = m;
      break;
    }
    t += s * 0.85f;
    if (t > P.options[1]) {
      t = P.options[1];
      break;
    }
  }

  const float horizon = clampf(dir.y * 0.5f + 0.5f, 0.0f, 1.0f);
  f3 color = mk(mixf(0.42f, 0.12f, horizon), mixf(0.47f, 0.18f, horizon), mixf(0.55f, 0.32f, horizon));
  if (hit) {
    const f3 pos = origin + t * dir;
    const f3 n = calc_normal(pos, an);
    const f3 albedo = material_color(material, pos);
    const float sa = P.options[2];
    const f3 sun = norm3(mk(cosf(sa), 0.72f, sinf(sa)));
    const float shadow = soft_shadow(pos + 0.02f * n, sun, an);
    const float diffuse = fmaxf(dot3(n, sun), 0.0f) * shadow;
    const float sky = 0.5f + 0.5f * n.y;
    const float bounce = fmaxf(-n.y, 0.0f) * 0.2f;
    const f3 light = ((diffuse * 1.5f) * mk(1.0f, 0.94f, 0.82f) + (sky * 0.35f) * mk(0.35f, 0.45f, 0.65f)) +
                     mk(bounce * 0.25f, bounce * 0.25f, bounce * 0.25f);
    const f3 half = norm3(sun - dir);
    const float spec = powf(fmaxf(dot3(n, half), 0.0f), 48.0f) * shadow * 0.35f;
    color = mk(albedo.x * light.x + spec, albedo.y * light.y + spec, albedo.z * light.z + spec);
    const float fog = clampf(1.0f - expf(-t * 0.055f), 0.0f, 1.0f);
    color = mk(mixf(color.x, 0.3f, fog), mixf(color.y, 0.36f, fog), mixf(color.z, 0.46f, fog));
  }

  const long plane = (long)w * h, i = (long)y * w + x;
  const float c3[3] = {color.x, color.y, color.z};
  uint32_t packed = 0xFF000000u;
#pragma unroll
  for (int k = 0; k < 3; k++) {
    const float mapped = c3[k] / (c3[k] + 0.6f);
    const float s = powf(clampf(mapped, 0.0f, 1.0f), 1.0f / 2.2f);
    const uint32_t q = (uint32_t)__float2int_rn(clampf(s, 0.0f, 1.0f) * 255.0f);
    packed |= q << (8 * k);
    if (rgb) rgb[(frame * 3 + k) * plane + i] = (float)q / 255.0f;
  }
  if (rgba8) reinterpret_cast<uint32_t *>(rgba8)[frame * plane + i] = packed;
  if (truth) reinterpret_cast<float2 *>(truth)[frame * plane + i] = make_float2(t * dot3(dir, forward), hit ? 1.0f : 0.0f);
}

// ---- metrics -----------------------------------------------------------------------

constexpr int kMetricThreads = 512;
constexpr int kMetricCluster = 8;

// Block-wide sum in a fixed order: warp butterflies, then warp 0 over the warp sums.
template <typename T>
__device__ __forceinline__ T block_sum(T v, T *smem) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? smem[lane] : T(0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) smem[0] = v;
  }
  __syncthreads();
  v = smem[0];
  return v;
}

__device__ __forceinline__ bool valid_truth(float2 tr) { return !(tr.y < 0.5f) && tr.x > 0.05f && !(tr.x > 25.0f); }

// Per-CTA partial sums, read by the cluster's rank-0 CTA through distributed
// shared memory.
struct FitPart {
  double sxx, sx, sxy, sy;
  long long n;
};
struct ErrPart {
  double abs_rel, sq;
  long long d1, d2, d3, counted;
};

// One frame per cluster of kMetricCluster CTAs: CTA r reduces the r-th chunk of
// the frame's pixels, rank 0 combines the chunks' partials in rank order (so
// the result is independent of scheduling), solves the fit and publishes it to
// the cluster for the second pass. Every CTA stays resident until the last
// remote read of its shared memory (the trailing cluster barriers).
__global__ void __cluster_dims__(kMetricCluster, 1, 1) __launch_bounds__(kMetricThreads)
    k_metrics(const float *__restrict__ pred, int pred_ch, const float2 *__restrict__ truth, long plane,
              DepthMetrics *__restrict__ out) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ double sd[32];
  __shared__ long long sl[32];
  __shared__ FitPart fit_part;
  __shared__ ErrPart err_part;
  __shared__ double fit[2];
  __shared__ long long fit_n;
  const unsigned rank = cluster.block_rank();
  const long f = blockIdx.x / kMetricCluster;
  const float *pf = pred + f * plane * pred_ch;
  const float2 *tf = truth + f * plane;
  const long chunk = (plane + kMetricCluster - 1) / kMetricCluster;
  const long begin = (long)rank * chunk, end = begin + chunk < plane ? begin + chunk : plane;

  long long n = 0;
  double sxx = 0, sx = 0, sxy = 0, sy = 0;
#pragma unroll 4
  for (long i = begin + threadIdx.x; i < end; i += kMetricThreads) {
    const float2 tr = tf[i];
    const float pv = pf[i * pred_ch];
    if (valid_truth(tr)) {
      const double xv = (double)pv, yv = 1.0 / (double)tr.x;
      sxx += xv * xv;
      sx += xv;
      sxy += xv * yv;
      sy += yv;
      n++;
    }
  }
  n = block_sum<long long>(n, sl);
  sxx = block_sum<double>(sxx, sd);
  sx = block_sum<double>(sx, sd);
  sxy = block_sum<double>(sxy, sd);
  sy = block_sum<double>(sy, sd);
  if (threadIdx.x == 0) fit_part = {sxx, sx, sxy, sy, n};
  cluster.sync();
  if (rank == 0 && threadIdx.x == 0) {
    FitPart a = {0, 0, 0, 0, 0};
    for (unsigned r = 0; r < kMetricCluster; r++) {
      const FitPart *p = cluster.map_shared_rank(&fit_part, r);
      a.sxx += p->sxx;
      a.sx += p->sx;
      a.sxy += p->sxy;
      a.sy += p->sy;
      a.n += p->n;
    }
    const double dn = (double)a.n;
    const double det = a.sxx * dn - a.sx * a.sx;
    fit[0] = fabs(det) > 1e-12 ? (dn * a.sxy - a.sx * a.sy) / det : 1.0;
    fit[1] = fabs(det) > 1e-12 ? (a.sxx * a.sy - a.sx * a.sxy) / det : 0.0;
    fit_n = a.n;
  }
  cluster.sync();
  const double *fit0 = cluster.map_shared_rank(&fit[0], 0);
  const double scale = fit0[0], shift = fit0[1];
  const long long total = *cluster.map_shared_rank(&fit_n, 0);
  cluster.sync();  // rank 0's fit stays readable until every CTA has it
  if (total < 64) {
    if (rank == 0 && threadIdx.x == 0) {
      DepthMetrics r;
      r.samples = total;
      r.abs_rel = r.rmse = r.scale = r.shift = __longlong_as_double(0x7ff8000000000000ll);
      r.delta1 = r.delta2 = r.delta3 = 0.0;
      out[f] = r;
    }
    return;
  }

  double abs_rel = 0, sq = 0;
  long long d1 = 0, d2 = 0, d3 = 0, counted = 0;
#pragma unroll 4
  for (long i = begin + threadIdx.x; i < end; i += kMetricThreads) {
    const float2 tr = tf[i];
    const float pv = pf[i * pred_ch];
    if (!valid_truth(tr)) continue;
    const double disparity = scale * (double)pv + shift;
    if (!(disparity > 1e-4)) continue;
    const double zhat = 1.0 / disparity, z = (double)tr.x;
    abs_rel += fabs(zhat - z) / z;
    sq += (zhat - z) * (zhat - z);
    const double ratio = fmax(zhat / z, z / zhat);
    d1 += ratio < 1.25;
    d2 += ratio < 1.5625;
    d3 += ratio < 1.953125;
    counted++;
  }
  abs_rel = block_sum<double>(abs_rel, sd);
  sq = block_sum<double>(sq, sd);
  d1 = block_sum<long long>(d1, sl);
  d2 = block_sum<long long>(d2, sl);
  d3 = block_sum<long long>(d3, sl);
  counted = block_sum<long long>(counted, sl);
  if (threadIdx.x == 0) err_part = {abs_rel, sq, d1, d2, d3, counted};
  cluster.sync();
  if (rank == 0 && threadIdx.x == 0) {
    ErrPart a = {0, 0, 0, 0, 0, 0};
    for (unsigned r = 0; r < kMetricCluster; r++) {
      const ErrPart *p = cluster.map_shared_rank(&err_part, r);
      a.abs_rel += p->abs_rel;
      a.sq += p->sq;
      a.d1 += p->d1;
      a.d2 += p->d2;
      a.d3 += p->d3;
      a.counted += p->counted;
    }
    const double denom = a.counted > 1 ? (double)a.counted : 1.0;
    DepthMetrics r;
    r.samples = a.counted;
    r.abs_rel = a.abs_rel / denom;
    r.rmse = sqrt(a.sq / denom);
    r.delta1 = (double)a.d1 / denom;
    r.delta2 = (double)a.d2 / denom;
    r.delta3 = (double)a.d3 / denom;
    r.scale = scale;
    r.shift = shift;
    out[f] = r;
  }
  cluster.sync();  // partials stay readable until rank 0 has combined them
}

}  // namespace

cudaError_t scene_render(const SceneParams *params, int n, int w, int h, float *rgb, uint8_t *rgba8, float *truth,
                         cudaStream_t st) {
  if (n <= 0 || w <= 0 || h <= 0) return cudaSuccess;
  const dim3 block(16, 8);
  for (int first = 0; first < n; first += kSceneBatch) {
    SceneBatch b;
    b.first = first;
    const int cnt = n - first < kSceneBatch ? n - first : kSceneBatch;
    for (int i = 0; i < cnt; i++) b.frames[i] = params[first + i];
    const dim3 grid((w + 15) / 16, (h + 7) / 8, cnt);
    k_scene<<<grid, block, 0, st>>>(b, w, h, rgb, rgba8, truth);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t evaluate_depth(const float *pred, int pred_ch, const float *truth, int n, long plane, DepthMetrics *out,
                           cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_metrics<<<n * kMetricCluster, kMetricThreads, 0, st>>>(pred, pred_ch, reinterpret_cast<const float2 *>(truth), plane, out);
  return cudaGetLastError();
}

}  // namespace gpu
}  // namespace illumina
