// Depth-aware shading + tone-map in one sm_100a kernel.
//
// Per render pixel (src/lighting/shade.ts:312-528): nearest disparity fetch,
// reciprocal depth map (:81-89), unprojection (:103-111), "accurate" normal
// reconstruction from a 5-tap cross (:135-169), bilinear sRGB albedo
// (renderer.ts:127-132), horizon AO (:242-274), up to 8 lights with windowed
// inverse-square / spot cones (:392-420), screen-space contact shadows
// (:202-230), GGX D x Smith-Schlick G specular (:287-308), volumetric
// in-scattering along the view ray (:452-488), depth fog (:496-501), exposure
// and the debug views (:506-517). The composite pass (composite.ts:87-113:
// ACES / Reinhard, saturation, contrast, vignette, exact linear->sRGB) is
// fused as the epilogue, writing 8-bit RGBA directly: the HDR target is
// optional.
//
// Depth neighbourhoods: each 16 x 8 block first stages the depth texels its
// pixels can reach through the normal stencil (+-2) and the AO horizon
// marches (+- the AO radius, up to kTileR) in a shared-memory tile, with the
// reference's clamp-to-edge already applied, so those fetches are one shared
// load with no clamping; the contact-shadow marches (screen projections of
// view-space points) read the tile when they land in it and the read-only
// cache otherwise.
//
// Arithmetic follows the accuracy WGSL specifies for the shader's built-ins
// (division 2.5 ulp, inverseSqrt 2 ulp, sqrt as 1/inverseSqrt, exp 3 + 2|x|
// ulp, pow via exp2(y log2 x), sin/cos 2^-11 absolute on [-pi, pi]): divisions
// by the hardware reciprocal-based division, square roots and normalisations
// by sqrt.approx / rsqrt.approx, exp / pow / sincos by the hardware
// approximations. Loop invariants (reciprocals of the step counts, of the
// projection scales and of the render size) are hoisted out of the marches.
// The AO horizon march and the volumetric march take two steps per iteration
// as packed f32x2 pairs (the kernel is issue bound: 8 % fewer cycles).
// Step counts are runtime parameters so the reference constants and longer
// marches share one kernel.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace illumina {
namespace gpu {

namespace {

constexpr int kShadeBX = 16, kShadeBY = 8;
constexpr int kTileR = 24;       // tile halo bound: larger AO radii read beyond it from the cache
constexpr int kTileMax = 3072;   // floats of the shared tile (12 KB)

__device__ __forceinline__ float fdiv(float a, float b) { return __fdividef(a, b); }
__device__ __forceinline__ float frcp(float a) { return __fdividef(1.0f, a); }
__device__ __forceinline__ float sqrt_a(float x) {
  float r;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float rsqrt_a(float x) {
  float r;
  asm("rsqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

struct v3 {
  float x, y, z;
};
__device__ __forceinline__ v3 mk(float x, float y, float z) { return v3{x, y, z}; }
__device__ __forceinline__ v3 operator+(v3 a, v3 b) { return mk(a.x + b.x, a.y + b.y, a.z + b.z); }
__device__ __forceinline__ v3 operator-(v3 a, v3 b) { return mk(a.x - b.x, a.y - b.y, a.z - b.z); }
__device__ __forceinline__ v3 operator*(float s, v3 a) { return mk(s * a.x, s * a.y, s * a.z); }
__device__ __forceinline__ v3 mulv(v3 a, v3 b) { return mk(a.x * b.x, a.y * b.y, a.z * b.z); }
__device__ __forceinline__ float dot3(v3 a, v3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ float len3(v3 a) { return sqrt_a(dot3(a, a)); }
__device__ __forceinline__ v3 norm3(v3 a) { return rsqrt_a(dot3(a, a)) * a; }
__device__ __forceinline__ v3 cross3(v3 a, v3 b) {
  return mk(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}
__device__ __forceinline__ float clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }
__device__ __forceinline__ float mixf(float a, float b, float t) { return a * (1.0f - t) + b * t; }
__device__ __forceinline__ v3 mixv(v3 a, v3 b, float t) {
  return mk(mixf(a.x, b.x, t), mixf(a.y, b.y, t), mixf(a.z, b.z, t));
}
__device__ __forceinline__ float fractf(float x) { return x - floorf(x); }
__device__ __forceinline__ float smoothstepf(float e0, float e1, float x) {
  float t = clampf(fdiv(x - e0, e1 - e0), 0.0f, 1.0f);
  return t * t * (3.0f - 2.0f * t);
}
// Packed pairs (sm_100 f32x2 ALU ops, each lane rounded as its scalar
// counterpart): two march steps per instruction.
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 f2s(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float pow4(float x) {
  float q = x * x;
  return q * q;
}

struct Ctx {
  const float *depth;
  int dw, dch;
  int maxX, maxY;
  float szw, szh;          // size.z, size.w
  float inv_szw, inv_szh;
  float tanh_, atanh_;     // tan(fov/2), aspect * tan(fov/2)
  float inv_near_minus_far, inv_far;
  // the block's shared tile: texels [tx0, tx0 + tw) x [ty0, ty0 + th), clamped
  const float *tile;
  int tx0, ty0, tw, th;
};

__device__ __forceinline__ float linear_depth(const Ctx &c, float d) {
  return frcp(fmaxf(d * c.inv_near_minus_far + c.inv_far, 1e-6f));
}
__device__ __forceinline__ float fetch(const Ctx &c, int x, int y) {
  const unsigned lx = (unsigned)(x - c.tx0), ly = (unsigned)(y - c.ty0);
  if (lx < (unsigned)c.tw && ly < (unsigned)c.th) return c.tile[ly * c.tw + lx];
  x = min(max(x, 0), c.maxX);
  y = min(max(y, 0), c.maxY);
  return __ldg(c.depth + ((long)y * c.dw + x) * c.dch);
}
__device__ __forceinline__ v3 view_position(const Ctx &c, float u, float v, float z) {
  float ndcX = u * 2.0f - 1.0f, ndcY = 1.0f - v * 2.0f;
  return mk(ndcX * c.atanh_ * z, ndcY * c.tanh_ * z, -z);
}
__device__ __forceinline__ v3 view_position_px(const Ctx &c, int x, int y, float d) {
  return view_position(c, ((float)x + 0.5f) * c.inv_szw, ((float)y + 0.5f) * c.inv_szh, linear_depth(c, d));
}

__device__ v3 reconstruct_normal(const Ctx &c, int x, int y) {
  float cc = fetch(c, x, y);
  float l1 = fetch(c, x - 1, y), l2 = fetch(c, x - 2, y);
  float r1 = fetch(c, x + 1, y), r2 = fetch(c, x + 2, y);
  float u1 = fetch(c, x, y - 1), u2 = fetch(c, x, y - 2);
  float b1 = fetch(c, x, y + 1), b2 = fetch(c, x, y + 2);
  float errL = fabsf(2.0f * l1 - l2 - cc), errR = fabsf(2.0f * r1 - r2 - cc);
  float errU = fabsf(2.0f * u1 - u2 - cc), errB = fabsf(2.0f * b1 - b2 - cc);
  // the positions use the clamped texel's disparity at the unclamped pixel
  // centre, as viewPositionAt does; only the chosen side of each axis is built
  v3 pc = view_position_px(c, x, y, cc);
  v3 dx = errL < errR ? pc - view_position_px(c, x - 1, y, l1) : view_position_px(c, x + 1, y, r1) - pc;
  v3 dy = errU < errB ? pc - view_position_px(c, x, y - 1, u1) : view_position_px(c, x, y + 1, b1) - pc;
  v3 n = cross3(dy, dx);
  float l2n = dot3(n, n);
  return l2n > 1e-24f ? rsqrt_a(l2n) * n : mk(0, 0, 1);
}

__device__ float contact_shadow(const Ctx &c, v3 origin, v3 to_light, float max_len, float jitter, int steps,
                                float inv_steps) {
  v3 step = (max_len * inv_steps) * to_light;
  float occlusion = 0.0f;
  v3 p = origin + jitter * step;
  const float kx = frcp(c.atanh_), ky = frcp(c.tanh_);
  for (int i = 0; i < steps; i++) {
    p = p + step;
    float inv_z = frcp(fmaxf(-p.z, 1e-4f));
    float u = (p.x * kx * inv_z) * 0.5f + 0.5f, v = 0.5f - (p.y * ky * inv_z) * 0.5f;
    if (u > 0.0f && u < 1.0f && v > 0.0f && v < 1.0f) {
      int cx = (int)(u * c.szw), cy = (int)(v * c.szh);
      float sceneZ = linear_depth(c, fetch(c, cx, cy));
      float delta = -p.z - sceneZ;
      float thickness = fmaxf(0.35f, sceneZ * 0.08f);
      if (delta > 0.012f && delta < thickness) occlusion = fmaxf(occlusion, 1.0f - (float)i * inv_steps);
    }
  }
  return 1.0f - clampf(occlusion, 0.0f, 1.0f);
}

__device__ float horizon_occlusion(const Ctx &c, int x, int y, v3 position, v3 normal, float radius_px,
                                   float jitter, int dirs, int steps) {
  float total = 0.0f;
  const float inv_dirs = frcp((float)dirs), inv_steps = frcp((float)steps);
  for (int i = 0; i < dirs; i++) {
    float angle = (((float)i + jitter) * inv_dirs) * 6.2831853f;
    if (angle > 3.14159265f) angle -= 6.2831853f;  // sin/cos of the same angle, on [-pi, pi]
    float s_, c_;
    __sincosf(angle, &s_, &c_);
    float horizon = -1.0f;
    // two steps per iteration as packed pairs (lane 0: step s, lane 1: s + 1);
    // an odd last step is taken by lane 0 only
    for (int s = 0; s < steps; s += 2) {
      const float2 dist = mul2(f2s(radius_px), mul2(f2((float)s + 1.0f, (float)s + 2.0f), f2s(inv_steps)));
      const float2 ox = mul2(f2s(c_), dist), oy = mul2(f2s(s_), dist);
      const int sx0 = x + (int)ox.x, sy0 = y + (int)oy.x, sx1 = x + (int)ox.y, sy1 = y + (int)oy.y;
      // view positions of the two samples (viewPositionAt at the sample pixels)
      const float2 d = f2(fetch(c, sx0, sy0), fetch(c, sx1, sy1));
      const float2 lin = fma2(d, f2s(c.inv_near_minus_far), f2s(c.inv_far));
      const float2 z = f2(frcp(fmaxf(lin.x, 1e-6f)), frcp(fmaxf(lin.y, 1e-6f)));
      const float2 u = mul2(add2(f2((float)sx0, (float)sx1), f2s(0.5f)), f2s(c.inv_szw));
      const float2 v = mul2(add2(f2((float)sy0, (float)sy1), f2s(0.5f)), f2s(c.inv_szh));
      const float2 ndcX = fma2(u, f2s(2.0f), f2s(-1.0f)), ndcY = fma2(v, f2s(-2.0f), f2s(1.0f));
      const float2 dx = add2(mul2(mul2(ndcX, f2s(c.atanh_)), z), f2s(-position.x));
      const float2 dy = add2(mul2(mul2(ndcY, f2s(c.tanh_)), z), f2s(-position.y));
      const float2 dz = add2(f2(-z.x, -z.y), f2s(-position.z));
      const float2 l2 = fma2(dz, dz, fma2(dy, dy, mul2(dx, dx)));
      const float2 inv_l = f2(rsqrt_a(l2.x), rsqrt_a(l2.y));
      const float2 len = mul2(l2, inv_l);
      const float2 cosH = mul2(fma2(f2s(normal.z), dz, fma2(f2s(normal.y), dy, mul2(f2s(normal.x), dx))), inv_l);
      const float2 fall = fma2(l2, f2s(-1.0f / 9.0f), f2s(1.0f));
      const float2 h = mul2(cosH, f2(clampf(fall.x, 0.0f, 1.0f), clampf(fall.y, 0.0f, 1.0f)));
      if (len.x > 1e-5f) horizon = fmaxf(horizon, h.x);
      if (s + 1 < steps && len.y > 1e-5f) horizon = fmaxf(horizon, h.y);
    }
    total += fmaxf(horizon, 0.0f);
  }
  return clampf(1.0f - total * inv_dirs, 0.0f, 1.0f);
}

__device__ __forceinline__ float ggx_d(float nDotH, float roughness) {
  float r = fmaxf(roughness, 1e-3f);
  float a = r * r;
  float a2 = a * a;
  float denom = fmaf(nDotH * nDotH, a2 - 1.0f, 1.0f);
  return fdiv(a2, 3.14159265f * denom * denom + 1e-20f);
}
__device__ __forceinline__ float smith_g(float nDotV, float nDotL, float roughness) {
  float k = (roughness + 1.0f) * (roughness + 1.0f) * 0.125f;
  return fdiv(nDotV, nDotV * (1.0f - k) + k) * fdiv(nDotL, nDotL * (1.0f - k) + k);
}
__device__ __forceinline__ float srgb_to_linear(float v) {
  return v <= 0.04045f ? v * (1.0f / 12.92f) : __powf((v + 0.055f) * (1.0f / 1.055f), 2.4f);
}
__device__ __forceinline__ float linear_to_srgb(float v) {
  return v <= 0.0031308f ? 12.92f * v : 1.055f * __powf(v, 1.0f / 2.4f) - 0.055f;
}
__device__ __forceinline__ float aces1(float x) {
  return clampf(fdiv(x * (2.51f * x + 0.03f), x * (2.43f * x + 0.59f) + 0.14f), 0.0f, 1.0f);
}
__device__ __forceinline__ float reinhard1(float x) {
  return clampf(fdiv(x * (1.0f + x * (1.0f / 16.0f)), 1.0f + x), 0.0f, 1.0f);
}
__device__ __forceinline__ uint32_t unorm8(float v) {
  if (!(v > 0.0f)) return 0u;
  if (v >= 1.0f) return 255u;
  return (uint32_t)floorf(v * 255.0f + 0.5f);
}

struct LightSet {
  ShadeLight l[8];
};

}  // namespace

__global__ void __launch_bounds__(kShadeBX * kShadeBY) k_shade(const float *__restrict__ depth, int dw, int dh,
                                                               int dch, const float *__restrict__ albedo, int aw,
                                                               int ah, LightSet L, ShadeParams P, ShadeSteps st,
                                                               int out_w, int out_h, float *hdr, uint8_t *rgba8) {
  __shared__ float tile[kTileMax];
  const int px = blockIdx.x * kShadeBX + threadIdx.x;
  const int py = blockIdx.y * kShadeBY + threadIdx.y;
  Ctx c;
  c.depth = depth, c.dw = dw, c.dch = dch;
  c.maxX = (int)P.size[2] - 1, c.maxY = (int)P.size[3] - 1;
  c.szw = P.size[2], c.szh = P.size[3];
  c.inv_szw = 1.0f / P.size[2], c.inv_szh = 1.0f / P.size[3];
  c.tanh_ = P.camera[0], c.atanh_ = P.camera[1] * P.camera[0];
  float near = fmaxf(P.camera[2], 1e-3f), far = fmaxf(P.camera[3], near + 1e-3f);
  c.inv_near_minus_far = 1.0f / near - 1.0f / far;
  c.inv_far = 1.0f / far;
  const float inv_w = 1.0f / P.size[0], inv_h = 1.0f / P.size[1];

  // ---- stage the block's depth neighbourhood (clamp-to-edge applied) ----
  {
    const int bx0 = blockIdx.x * kShadeBX, by0 = blockIdx.y * kShadeBY;
    const int bx1 = min(bx0 + kShadeBX, out_w) - 1, by1 = min(by0 + kShadeBY, out_h) - 1;
    const int dx0 = (int)(((float)bx0 + 0.5f) * inv_w * P.size[2]), dx1 = (int)(((float)bx1 + 0.5f) * inv_w * P.size[2]);
    const int dy0 = (int)(((float)by0 + 0.5f) * inv_h * P.size[3]), dy1 = (int)(((float)by1 + 0.5f) * inv_h * P.size[3]);
    const float ao_r = P.toggles[0] > 0.001f ? P.debug[3] : 0.0f;
    const int R = max(2, min(kTileR, (int)fminf(fmaxf(ao_r, 0.0f), (float)kTileR)));
    c.tx0 = dx0 - R, c.ty0 = dy0 - R;
    c.tw = dx1 - dx0 + 1 + 2 * R, c.th = dy1 - dy0 + 1 + 2 * R;
    if (c.tw * c.th > kTileMax) c.tw = c.th = 0;  // every fetch goes through the cache
    const int n = c.tw * c.th;
    const int tid = threadIdx.y * kShadeBX + threadIdx.x;
    for (int i = tid; i < n; i += kShadeBX * kShadeBY) {
      const int ly = i / c.tw, lx = i - ly * c.tw;
      const int x = min(max(c.tx0 + lx, 0), c.maxX), y = min(max(c.ty0 + ly, 0), c.maxY);
      tile[i] = __ldg(depth + ((long)y * dw + x) * dch);
    }
    c.tile = tile;
    __syncthreads();
  }
  if (px >= out_w || py >= out_h) return;

  float u = ((float)px + 0.5f) * inv_w, v = ((float)py + 0.5f) * inv_h;
  int dcx = (int)(u * P.size[2]), dcy = (int)(v * P.size[3]);
  float disparity = fetch(c, dcx, dcy);
  float z = linear_depth(c, disparity);
  v3 position = view_position(c, u, v, z);
  v3 rn = reconstruct_normal(c, dcx, dcy);
  v3 normal = norm3(mk(rn.x * P.misc[3], rn.y * P.misc[3], rn.z));

  // bilinear, clamp-to-edge albedo sample of the planar sRGB image
  v3 alb_lin;
  {
    float tx = u * (float)aw - 0.5f, ty = v * (float)ah - 0.5f;
    float fx0 = floorf(tx), fy0 = floorf(ty);
    float fx = tx - fx0, fy = ty - fy0;
    int x0 = min(max((int)fx0, 0), aw - 1), x1 = min(max((int)fx0 + 1, 0), aw - 1);
    int y0 = min(max((int)fy0, 0), ah - 1), y1 = min(max((int)fy0 + 1, 0), ah - 1);
    long plane = (long)aw * ah;
    float ch[3];
#pragma unroll
    for (int k = 0; k < 3; k++) {
      const float *p = albedo + k * plane;
      float a = __ldg(p + (long)y0 * aw + x0), b = __ldg(p + (long)y0 * aw + x1);
      float cc = __ldg(p + (long)y1 * aw + x0), d = __ldg(p + (long)y1 * aw + x1);
      float top = a + (b - a) * fx, bot = cc + (d - cc) * fx;
      ch[k] = srgb_to_linear(top + (bot - top) * fy);
    }
    alb_lin = mk(ch[0], ch[1], ch[2]);
  }
  v3 albedo_c = mixv(mk(0.6f, 0.6f, 0.6f), alb_lin, P.debug[1]);
  float fr = P.misc[0] * 5.588238f;
  float jitter = fractf(52.9829189f * fractf((px + fr) * 0.06711056f + (py + fr) * 0.00583715f));
  v3 view_dir = norm3(-1.0f * position);
  float nDotV = fmaxf(dot3(normal, view_dir), 1e-4f);
  float rough = clampf(P.misc[1], 0.04f, 1.0f);
  float ao = 1.0f;
  if (P.toggles[0] > 0.001f)
    ao = mixf(1.0f, horizon_occlusion(c, dcx, dcy, position, normal, P.debug[3], jitter, st.ao_dirs, st.ao_steps),
              P.toggles[0]);
  v3 radiance = mulv((P.ambient[3] * ao) * albedo_c, mk(P.ambient[0], P.ambient[1], P.ambient[2]));
  v3 scattering = mk(0, 0, 0);
  float ray_len = len3(position);
  v3 ray_dir = frcp(fmaxf(ray_len, 1e-5f)) * position;
  const float inv_contact = frcp((float)st.contact), inv_vol = frcp((float)st.volumetric);

  for (int li = 0; li < 8; li++) {
    const ShadeLight &Lt = L.l[li];
    float intensity = Lt.color[3];
    if (!(intensity > 0.0f)) continue;
    float kind = Lt.params[0];
    v3 lcol = mk(Lt.color[0], Lt.color[1], Lt.color[2]);
    v3 lpos = mk(Lt.position[0], Lt.position[1], Lt.position[2]);
    v3 to_light = mk(0, 0, 1);
    float atten = 1.0f, distance = 1e6f;
    const float inv_range = frcp(fmaxf(Lt.params[2], 1e-3f));
    if (kind > 1.5f) {
      to_light = norm3(-1.0f * lpos);
    } else {
      v3 delta = lpos - position;
      distance = fmaxf(len3(delta), 1e-4f);
      to_light = frcp(distance) * delta;
      float win = clampf(1.0f - pow4(distance * inv_range), 0.0f, 1.0f);
      atten = fdiv(win * win, distance * distance + 1e-4f);
    }
    v3 axis = mk(Lt.direction[0], Lt.direction[1], Lt.direction[2]);
    const float cone_hi = fmaxf(Lt.params[1], Lt.direction[3] + 1e-3f);
    if (kind > 0.5f && kind < 1.5f) {
      float cosA = -dot3(to_light, axis);
      atten *= smoothstepf(Lt.direction[3], cone_hi, cosA);
    }
    float nDotL = dot3(normal, to_light);
    if (nDotL > 0.0f && atten > 0.0f) {
      float shadow = 1.0f;
      float amount = Lt.params[3] * P.toggles[1];
      if (amount > 0.0f) {
        float march = fminf(P.debug[2], distance);
        shadow = mixf(1.0f, contact_shadow(c, position, to_light, march, jitter, st.contact, inv_contact), amount);
      }
      v3 half = norm3(to_light + view_dir);
      float nDotH = fmaxf(dot3(normal, half), 0.0f);
      float spec = ggx_d(nDotH, rough) * smith_g(nDotV, nDotL, rough) * P.fog[3];
      float energy = atten * intensity * nDotL * shadow;
      radiance = radiance + energy * mulv(lcol, albedo_c + mk(spec, spec, spec));
    }
    if (P.toggles[2] > 0.0f && kind < 1.5f) {
      const float step_len = ray_len * inv_vol;
      const float k = intensity * step_len * P.misc[2];
      const float inv_range2 = inv_range * inv_range;
      // two steps per iteration as packed pairs (lane 0: step s, lane 1: s + 1),
      // summed in two partial sums; an odd last step counts in lane 0 only
      const float2 lx = f2s(lpos.x), ly = f2s(lpos.y), lz = f2s(lpos.z);
      const float2 rx = f2s(ray_dir.x), ry = f2s(ray_dir.y), rz = f2s(ray_dir.z);
      const float2 nstep = f2s(-step_len), jit = f2s(jitter), ir2 = f2s(inv_range2);
      float2 acc2 = f2s(0.0f);
      for (int s = 0; s < st.volumetric; s += 2) {
        const float2 nt = mul2(add2(f2((float)s, (float)(s + 1)), jit), nstep);  // -t
        // toL = lpos - t * ray_dir; dist = max(|toL|, 1e-3) enters only squared
        const float2 tx = fma2(nt, rx, lx), ty = fma2(nt, ry, ly), tz = fma2(nt, rz, lz);
        float2 dd = fma2(tz, tz, fma2(ty, ty, mul2(tx, tx)));
        dd = f2(fmaxf(dd.x, 1e-6f), fmaxf(dd.y, 1e-6f));
        const float2 q = mul2(dd, ir2);  // (dist / range)^2
        float2 win = fma2(f2(-q.x, -q.y), q, f2s(1.0f));
        win = f2(clampf(win.x, 0.0f, 1.0f), clampf(win.y, 0.0f, 1.0f));
        const float2 den = add2(dd, f2s(1e-4f));
        float2 att = mul2(mul2(win, win), f2(frcp(den.x), frcp(den.y)));
        if (kind > 0.5f) {
          const float2 d = fma2(tz, f2s(axis.z), fma2(ty, f2s(axis.y), mul2(tx, f2s(axis.x))));
          const float2 cosA = mul2(d, f2(-rsqrt_a(dd.x), -rsqrt_a(dd.y)));
          att = mul2(att, f2(smoothstepf(Lt.direction[3], cone_hi, cosA.x),
                             smoothstepf(Lt.direction[3], cone_hi, cosA.y)));
        }
        if (s + 1 >= st.volumetric) att.y = 0.0f;
        acc2 = add2(acc2, att);
      }
      scattering = scattering + ((acc2.x + acc2.y) * k) * lcol;
    }
  }
  radiance = radiance + P.toggles[2] * scattering;
  float fog_amount = 1.0f - __expf(-z * P.misc[2]);
  radiance = mixv(radiance, mk(P.fog[0], P.fog[1], P.fog[2]), clampf(fog_amount, 0.0f, 1.0f));
  radiance = P.toggles[3] * radiance;
  float mode = P.debug[0];
  v3 oc = radiance;
  if (mode > 0.5f && mode < 1.5f) oc = mk(disparity, disparity, disparity);
  else if (mode > 1.5f && mode < 2.5f) oc = 0.5f * (normal + mk(1, 1, 1));
  else if (mode > 2.5f && mode < 3.5f) oc = mk(ao, ao, ao);
  else if (mode > 3.5f) oc = alb_lin;

  long o = (long)py * out_w + px;
  if (hdr) reinterpret_cast<float4 *>(hdr)[o] = make_float4(oc.x, oc.y, oc.z, 1.0f);
  if (rgba8) {
    v3 mapped = P.grade[0] < 0.5f ? mk(aces1(oc.x), aces1(oc.y), aces1(oc.z))
                                  : mk(reinhard1(oc.x), reinhard1(oc.y), reinhard1(oc.z));
    float luma = dot3(mapped, mk(0.2126f, 0.7152f, 0.0722f));
    v3 col = mixv(mk(luma, luma, luma), mapped, P.grade[2]);
    col = mk(clampf(0.5f + P.grade[1] * (col.x - 0.5f), 0.0f, 1.0f),
             clampf(0.5f + P.grade[1] * (col.y - 0.5f), 0.0f, 1.0f),
             clampf(0.5f + P.grade[1] * (col.z - 0.5f), 0.0f, 1.0f));
    float cu = u - 0.5f, cv = v - 0.5f;
    float vig = 1.0f - P.grade[3] * (cu * cu + cv * cv) * 2.0f;
    col = clampf(vig, 0.0f, 1.0f) * col;
    uint32_t r = unorm8(linear_to_srgb(col.x)), g = unorm8(linear_to_srgb(col.y)), b = unorm8(linear_to_srgb(col.z));
    reinterpret_cast<uint32_t *>(rgba8)[o] = r | (g << 8) | (b << 16) | (255u << 24);
  }
}

cudaError_t shade(const float *depth, int dw, int dh, int dch, const float *albedo, int aw, int ah, const ShadeLight *lights,
                  const ShadeParams &P, const ShadeSteps &steps, int out_w, int out_h, float *hdr, uint8_t *rgba8,
                  cudaStream_t st) {
  if (out_w <= 0 || out_h <= 0) return cudaSuccess;
  LightSet L;
  for (int i = 0; i < 8; i++) L.l[i] = lights[i];
  dim3 block(kShadeBX, kShadeBY);
  dim3 grid((out_w + kShadeBX - 1) / kShadeBX, (out_h + kShadeBY - 1) / kShadeBY);
  k_shade<<<grid, block, 0, st>>>(depth, dw, dh, dch, albedo, aw, ah, L, P, steps, out_w, out_h, hdr, rgba8);
  return cudaGetLastError();
}

__global__ void k_resize(const float *src, int sw, int sh, float *dst, int dw, int dh) {
  int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
  if (x >= dw || y >= dh) return;
  // every operation rounded on its own (no contraction), so the result is
  // the same float as a host evaluation in this order
  float u = __fdiv_rn((float)x + 0.5f, (float)dw), v = __fdiv_rn((float)y + 0.5f, (float)dh);
  float tx = __fsub_rn(__fmul_rn(u, (float)sw), 0.5f), ty = __fsub_rn(__fmul_rn(v, (float)sh), 0.5f);
  float fx0 = floorf(tx), fy0 = floorf(ty);
  float fx = __fsub_rn(tx, fx0), fy = __fsub_rn(ty, fy0);
  int x0 = min(max((int)fx0, 0), sw - 1), x1 = min(max((int)fx0 + 1, 0), sw - 1);
  int y0 = min(max((int)fy0, 0), sh - 1), y1 = min(max((int)fy0 + 1, 0), sh - 1);
  float a = __ldg(src + (long)y0 * sw + x0), b = __ldg(src + (long)y0 * sw + x1);
  float c = __ldg(src + (long)y1 * sw + x0), d = __ldg(src + (long)y1 * sw + x1);
  float top = __fadd_rn(a, __fmul_rn(__fsub_rn(b, a), fx)), bot = __fadd_rn(c, __fmul_rn(__fsub_rn(d, c), fx));
  dst[(long)y * dw + x] = __fadd_rn(top, __fmul_rn(__fsub_rn(bot, top), fy));
}

cudaError_t resize_bilinear(const float *src, int sw, int sh, float *dst, int dw, int dh, cudaStream_t st) {
  if (dw <= 0 || dh <= 0) return cudaSuccess;
  dim3 block(32, 8), grid((dw + 31) / 32, (dh + 7) / 8);
  k_resize<<<grid, block, 0, st>>>(src, sw, sh, dst, dw, dh);
  return cudaGetLastError();
}

}  // namespace gpu
}  // namespace illumina
