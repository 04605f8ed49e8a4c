/*
 * CPU oracle for the depth-aware shading pass and its tone-map: a scalar
 * float32 restatement of src/lighting/shade.ts:81-528 and
 * src/lighting/composite.ts:35-113. The reference has no CPU version of this
 * math (it is GPU-tested only), so this transcription is the checker.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by the test-suite, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg, never by the product.
 *
 * Conventions:
 *   - all arithmetic is float32, as WGSL f32 (built with -ffp-contract=off);
 *   - `x ** n` in the shader is evaluated as repeated multiplication;
 *   - the depth map is sampled by nearest fetch with clamp (fetchDisparity);
 *   - the albedo texture is sampled bilinearly with clamp-to-edge at the
 *     render uv (renderer.ts:127-132), then decoded from sRGB;
 *   - step counts are parameters: the reference compiles CONTACT_STEPS 12
 *     (shade.ts:192), AO 6 directions x 4 steps (:232-233) and 10 volumetric
 *     steps per light (:310).
 */
#include <math.h>
#include <stdint.h>

typedef struct { float x, y, z; } v3;

typedef struct {
  float position[4], color[4], direction[4], params[4];
} or_light;

/* ShadeParams, shade.ts:40-55, plus the composite grade (composite.ts:13-16). */
typedef struct {
  float camera[4], toggles[4], ambient[4], misc[4], fog[4], size[4], debug[4];
  float grade[4];
} or_shade_params;

typedef struct {
  int contact_steps, ao_dirs, ao_steps, vol_steps;
} or_steps;

static v3 mk(float x, float y, float z) { v3 r = {x, y, z}; return r; }
static v3 add(v3 a, v3 b) { return mk(a.x + b.x, a.y + b.y, a.z + b.z); }
static v3 sub(v3 a, v3 b) { return mk(a.x - b.x, a.y - b.y, a.z - b.z); }
static v3 scl(float s, v3 a) { return mk(s * a.x, s * a.y, s * a.z); }
static v3 mulv(v3 a, v3 b) { return mk(a.x * b.x, a.y * b.y, a.z * b.z); }
static v3 divs(v3 a, float s) { return mk(a.x / s, a.y / s, a.z / s); }
static float dot3(v3 a, v3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
static float len3(v3 a) { return sqrtf(dot3(a, a)); }
static v3 norm3(v3 a) { return divs(a, len3(a)); }
static v3 cross3(v3 a, v3 b) {
  return mk(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}
static float fmaxw(float a, float b) { return a > b ? a : b; }
static float fminw(float a, float b) { return a < b ? a : b; }
static float clampf(float v, float lo, float hi) { return fminw(fmaxw(v, lo), hi); }
static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
static float mixf(float a, float b, float t) { return a * (1 - t) + b * t; }
static v3 mixv(v3 a, v3 b, float t) {
  return mk(mixf(a.x, b.x, t), mixf(a.y, b.y, t), mixf(a.z, b.z, t));
}
static float fractf(float x) { return x - floorf(x); }
static float smoothstepf(float e0, float e1, float x) {
  float t = clampf((x - e0) / (e1 - e0), 0.0f, 1.0f);
  return t * t * (3.0f - 2.0f * t);
}
static float pow4(float x) { float q = x * x; return q * q; }

typedef struct {
  const or_shade_params *P;
  const float *depth; /* dh x dw, one float per texel (disparity) */
  int dw, dh;
} ctx_t;

/* linearDepth, shade.ts:81-89 */
static float linear_depth(const ctx_t *c, float disparity) {
  float near = fmaxw(c->P->camera[2], 1e-3f);
  float far = fmaxw(c->P->camera[3], near + 1e-3f);
  float invZ = disparity * (1.0f / near - 1.0f / far) + 1.0f / far;
  return 1.0f / fmaxw(invZ, 1e-6f);
}

/* fetchDisparity, shade.ts:92-100 */
static float fetch(const ctx_t *c, int x, int y) {
  int maxX = (int)c->P->size[2] - 1, maxY = (int)c->P->size[3] - 1;
  x = clampi(x, 0, maxX);
  y = clampi(y, 0, maxY);
  return c->depth[(long)y * c->dw + x];
}

/* viewPosition, shade.ts:103-111 */
static v3 view_position(const ctx_t *c, float u, float v, float z) {
  float ndcX = u * 2.0f - 1.0f, ndcY = 1.0f - v * 2.0f;
  float t = c->P->camera[0];
  return mk(ndcX * c->P->camera[1] * t * z, ndcY * t * z, -z);
}

/* viewPositionAt, shade.ts:114-123 */
static v3 view_position_at(const ctx_t *c, int x, int y) {
  float u = ((float)x + 0.5f) / c->P->size[2];
  float v = ((float)y + 0.5f) / c->P->size[3];
  return view_position(c, u, v, linear_depth(c, fetch(c, x, y)));
}

/* reconstructNormal, shade.ts:135-169 */
static v3 reconstruct_normal(const ctx_t *c, int x, int y) {
  float cc = fetch(c, x, y);
  float l1 = fetch(c, x - 1, y), l2 = fetch(c, x - 2, y);
  float r1 = fetch(c, x + 1, y), r2 = fetch(c, x + 2, y);
  float u1 = fetch(c, x, y - 1), u2 = fetch(c, x, y - 2);
  float b1 = fetch(c, x, y + 1), b2 = fetch(c, x, y + 2);
  float errL = fabsf(2.0f * l1 - l2 - cc), errR = fabsf(2.0f * r1 - r2 - cc);
  float errU = fabsf(2.0f * u1 - u2 - cc), errB = fabsf(2.0f * b1 - b2 - cc);
  v3 pc = view_position_at(c, x, y);
  v3 dxL = sub(pc, view_position_at(c, x - 1, y));
  v3 dxR = sub(view_position_at(c, x + 1, y), pc);
  v3 dyU = sub(pc, view_position_at(c, x, y - 1));
  v3 dyD = sub(view_position_at(c, x, y + 1), pc);
  v3 dx = errL < errR ? dxL : dxR;
  v3 dy = errU < errB ? dyU : dyD;
  v3 n = cross3(dy, dx);
  float l = len3(n);
  return l > 1e-12f ? divs(n, l) : mk(0, 0, 1);
}

/* dither, shade.ts:172-178 */
static float dither(float px, float py, float frame) {
  float ax = px + frame * 5.588238f, ay = py + frame * 5.588238f;
  return fractf(52.9829189f * fractf(ax * 0.06711056f + ay * 0.00583715f));
}

/* projectToDepthUv, shade.ts:181-190 */
static void project_uv(const ctx_t *c, v3 p, float *u, float *v) {
  float z = fmaxw(-p.z, 1e-4f);
  float t = c->P->camera[0];
  float ndcX = p.x / (c->P->camera[1] * t * z);
  float ndcY = p.y / (t * z);
  *u = ndcX * 0.5f + 0.5f;
  *v = 0.5f - ndcY * 0.5f;
}

/* contactShadow, shade.ts:202-230 */
static float contact_shadow(const ctx_t *c, v3 origin, v3 to_light, float max_len,
                            float jitter, int steps) {
  v3 step = scl(max_len / (float)steps, to_light);
  float occlusion = 0.0f;
  v3 p = add(origin, scl(jitter, step));
  for (int i = 0; i < steps; i++) {
    p = add(p, step);
    float u, v;
    project_uv(c, p, &u, &v);
    if (u > 0 && u < 1 && v > 0 && v < 1) {
      int cx = (int)(u * c->P->size[2]), cy = (int)(v * c->P->size[3]);
      float sceneZ = linear_depth(c, fetch(c, cx, cy));
      float rayZ = -p.z;
      float delta = rayZ - sceneZ;
      float thickness = fmaxw(0.35f, sceneZ * 0.08f);
      if (delta > 0.012f && delta < thickness)
        occlusion = fmaxw(occlusion, 1.0f - (float)i / (float)steps);
    }
  }
  return 1.0f - clampf(occlusion, 0.0f, 1.0f);
}

/* horizonOcclusion, shade.ts:242-274 */
static float horizon_occlusion(const ctx_t *c, int x, int y, v3 position, v3 normal,
                               float radius_px, float jitter, int dirs, int steps) {
  float total = 0.0f;
  for (int i = 0; i < dirs; i++) {
    float angle = (((float)i + jitter) / (float)dirs) * 6.2831853f;
    float dxv = cosf(angle), dyv = sinf(angle);
    float horizon = -1.0f;
    for (int s = 0; s < steps; s++) {
      float dist = radius_px * (((float)s + 1.0f) / (float)steps);
      int sx = x + (int)(dxv * dist), sy = y + (int)(dyv * dist);
      v3 diff = sub(view_position_at(c, sx, sy), position);
      float l = len3(diff);
      if (l > 1e-5f) {
        float cosH = dot3(normal, divs(diff, l));
        float falloff = clampf(1.0f - (l * l) / 9.0f, 0.0f, 1.0f);
        horizon = fmaxw(horizon, cosH * falloff);
      }
    }
    total += fmaxw(horizon, 0.0f);
  }
  return clampf(1.0f - total / (float)dirs, 0.0f, 1.0f);
}

/* distributionGGX, shade.ts:287-297 */
float or_ggx_d(float nDotH, float roughness) {
  float r = fmaxw(roughness, 1e-3f);
  float a = r * r;
  float a2 = a * a;
  /* One fused multiply-add, as the CUDA kernel (and GPU shader compilers)
   * evaluate it, so both sides round identically. */
  float denom = fmaf(nDotH * nDotH, a2 - 1.0f, 1.0f);
  return a2 / (3.14159265f * denom * denom + 1e-20f);
}

/* visibilitySmith, shade.ts:300-308 */
float or_smith_g(float nDotV, float nDotL, float roughness) {
  float k = (roughness + 1.0f) * (roughness + 1.0f) / 8.0f;
  float gv = nDotV / (nDotV * (1.0f - k) + k);
  float gl = nDotL / (nDotL * (1.0f - k) + k);
  return gv * gl;
}

/* srgbToLinear, src/model/kernels/io.ts:12-19 */
static float srgb_to_linear(float c) {
  return c <= 0.04045f ? c / 12.92f : powf((c + 0.055f) / 1.055f, 2.4f);
}

/* Bilinear, clamp-to-edge sample of a planar [3][ah][aw] image at uv. */
static v3 sample_albedo(const float *img, int aw, int ah, float u, float v) {
  float tx = u * (float)aw - 0.5f, ty = v * (float)ah - 0.5f;
  float fx0 = floorf(tx), fy0 = floorf(ty);
  float fx = tx - fx0, fy = ty - fy0;
  int x0 = clampi((int)fx0, 0, aw - 1), x1 = clampi((int)fx0 + 1, 0, aw - 1);
  int y0 = clampi((int)fy0, 0, ah - 1), y1 = clampi((int)fy0 + 1, 0, ah - 1);
  float out[3];
  long plane = (long)aw * ah;
  for (int ch = 0; ch < 3; ch++) {
    const float *p = img + ch * plane;
    float a = p[(long)y0 * aw + x0], b = p[(long)y0 * aw + x1];
    float cc = p[(long)y1 * aw + x0], d = p[(long)y1 * aw + x1];
    float top = a + (b - a) * fx, bot = cc + (d - cc) * fx;
    out[ch] = top + (bot - top) * fy;
  }
  return mk(out[0], out[1], out[2]);
}

/* acesFitted, composite.ts:35-47 */
static float aces1(float x) {
  float num = x * (2.51f * x + 0.03f);
  float den = x * (2.43f * x + 0.59f) + 0.14f;
  return clampf(num / den, 0.0f, 1.0f);
}
/* reinhard, composite.ts:50-57 */
static float reinhard1(float x) {
  float num = x * (1.0f + x / 16.0f);
  return clampf(num / (1.0f + x), 0.0f, 1.0f);
}
/* linearToSrgb, composite.ts:60-67 */
static float linear_to_srgb(float c) {
  return c <= 0.0031308f ? 12.92f * c : 1.055f * powf(c, 1.0f / 2.4f) - 0.055f;
}

/* compositeFragment, composite.ts:87-113, producing 8-bit sRGB by
 * round-to-nearest of clamp(v)*255. */
void or_composite_px(const float *grade, const float *hdr3, float u, float v,
                     float *srgb_out) {
  v3 col = mk(hdr3[0], hdr3[1], hdr3[2]);
  v3 mapped = grade[0] < 0.5f ? mk(aces1(col.x), aces1(col.y), aces1(col.z))
                              : mk(reinhard1(col.x), reinhard1(col.y), reinhard1(col.z));
  float luma = dot3(mapped, mk(0.2126f, 0.7152f, 0.0722f));
  col = mixv(mk(luma, luma, luma), mapped, grade[2]);
  col = mk(clampf(0.5f + grade[1] * (col.x - 0.5f), 0, 1),
           clampf(0.5f + grade[1] * (col.y - 0.5f), 0, 1),
           clampf(0.5f + grade[1] * (col.z - 0.5f), 0, 1));
  float cx = u - 0.5f, cy = v - 0.5f;
  float vig = 1.0f - grade[3] * (cx * cx + cy * cy) * 2.0f;
  col = scl(clampf(vig, 0, 1), col);
  srgb_out[0] = linear_to_srgb(col.x);
  srgb_out[1] = linear_to_srgb(col.y);
  srgb_out[2] = linear_to_srgb(col.z);
}

static uint8_t to_unorm8(float v) {
  if (!(v > 0.0f)) return 0;
  if (v >= 1.0f) return 255;
  return (uint8_t)floorf(v * 255.0f + 0.5f);
}

/* makeShade's per-pixel body, shade.ts:318-523. Writes hdr (rgba f32) and,
 * when rgba8 is non-null, the composited 8-bit sRGB pixel. */
void or_shade(const float *depth, int dw, int dh, const float *albedo, int aw, int ah,
              const or_light *lights, int n_lights, const or_shade_params *P,
              const or_steps *st, int out_w, int out_h, int row0, int row1,
              float *hdr, uint8_t *rgba8) {
  ctx_t cx = {P, depth, dw, dh};
  const ctx_t *c = &cx;
  for (int py = row0; py < row1; py++)
    for (int px = 0; px < out_w; px++) {
      float u = ((float)px + 0.5f) / P->size[0];
      float v = ((float)py + 0.5f) / P->size[1];
      int dcx = (int)(u * P->size[2]), dcy = (int)(v * P->size[3]);
      float disparity = fetch(c, dcx, dcy);
      float z = linear_depth(c, disparity);
      v3 position = view_position(c, u, v, z);
      v3 rn = reconstruct_normal(c, dcx, dcy);
      v3 normal = norm3(mk(rn.x * P->misc[3], rn.y * P->misc[3], rn.z));
      v3 srgb = sample_albedo(albedo, aw, ah, u, v);
      v3 alb_lin = mk(srgb_to_linear(srgb.x), srgb_to_linear(srgb.y), srgb_to_linear(srgb.z));
      v3 albedo_c = mixv(mk(0.6f, 0.6f, 0.6f), alb_lin, P->debug[1]);
      float jitter = dither((float)px, (float)py, P->misc[0]);
      v3 view_dir = norm3(scl(-1.0f, position));
      float nDotV = fmaxw(dot3(normal, view_dir), 1e-4f);
      float rough = clampf(P->misc[1], 0.04f, 1.0f);
      float ao = 1.0f;
      if (P->toggles[0] > 0.001f)
        ao = mixf(1.0f, horizon_occlusion(c, dcx, dcy, position, normal, P->debug[3], jitter,
                                          st->ao_dirs, st->ao_steps),
                  P->toggles[0]);
      v3 radiance = mulv(scl(P->ambient[3] * ao, albedo_c),
                         mk(P->ambient[0], P->ambient[1], P->ambient[2]));
      v3 scattering = mk(0, 0, 0);
      for (int li = 0; li < n_lights; li++) {
        const or_light *L = &lights[li];
        float intensity = L->color[3];
        if (!(intensity > 0)) continue;
        float kind = L->params[0];
        v3 lcol = mk(L->color[0], L->color[1], L->color[2]);
        v3 lpos = mk(L->position[0], L->position[1], L->position[2]);
        v3 to_light = mk(0, 0, 1);
        float atten = 1.0f, distance = 1e6f;
        if (kind > 1.5f) {
          to_light = norm3(scl(-1.0f, lpos));
        } else {
          v3 delta = sub(lpos, position);
          distance = fmaxw(len3(delta), 1e-4f);
          to_light = divs(delta, distance);
          float range = fmaxw(L->params[2], 1e-3f);
          float win = clampf(1.0f - pow4(distance / range), 0.0f, 1.0f);
          atten = (win * win) / (distance * distance + 1e-4f);
        }
        if (kind > 0.5f && kind < 1.5f) {
          v3 axis = mk(L->direction[0], L->direction[1], L->direction[2]);
          float cosA = dot3(scl(-1.0f, to_light), axis);
          float outer = L->direction[3], inner = L->params[1];
          atten *= smoothstepf(outer, fmaxw(inner, outer + 1e-3f), cosA);
        }
        float nDotL = dot3(normal, to_light);
        if (nDotL > 0 && atten > 0) {
          float shadow = 1.0f;
          float amount = L->params[3] * P->toggles[1];
          if (amount > 0) {
            float march = fminw(P->debug[2], distance);
            shadow = mixf(1.0f, contact_shadow(c, position, to_light, march, jitter,
                                               st->contact_steps),
                          amount);
          }
          v3 half = norm3(add(to_light, view_dir));
          float nDotH = fmaxw(dot3(normal, half), 0.0f);
          float spec = or_ggx_d(nDotH, rough) * or_smith_g(nDotV, nDotL, rough) * P->fog[3];
          float energy = atten * intensity * nDotL * shadow;
          radiance = add(radiance, scl(energy, mulv(lcol, add(albedo_c, mk(spec, spec, spec)))));
        }
        if (P->toggles[2] > 0 && kind < 1.5f) {
          float ray_len = len3(position);
          v3 ray_dir = divs(position, fmaxw(ray_len, 1e-5f));
          float step_len = ray_len / (float)st->vol_steps;
          for (int s = 0; s < st->vol_steps; s++) {
            float t = (((float)s + jitter) / (float)st->vol_steps) * ray_len;
            v3 sp = scl(t, ray_dir);
            v3 toL = sub(lpos, sp);
            float dist = fmaxw(len3(toL), 1e-3f);
            float range = fmaxw(L->params[2], 1e-3f);
            float win = clampf(1.0f - pow4(dist / range), 0.0f, 1.0f);
            float att = (win * win) / (dist * dist + 1e-4f);
            if (kind > 0.5f) {
              v3 axis = mk(L->direction[0], L->direction[1], L->direction[2]);
              float cosA = dot3(scl(-1.0f, divs(toL, dist)), axis);
              att *= smoothstepf(L->direction[3], fmaxw(L->params[1], L->direction[3] + 1e-3f),
                                 cosA);
            }
            scattering = add(scattering, scl(att * intensity * step_len * P->misc[2], lcol));
          }
        }
      }
      radiance = add(radiance, scl(P->toggles[2], scattering));
      float fog_amount = 1.0f - expf(-z * P->misc[2]);
      radiance = mixv(radiance, mk(P->fog[0], P->fog[1], P->fog[2]), clampf(fog_amount, 0, 1));
      radiance = scl(P->toggles[3], radiance);
      float mode = P->debug[0];
      v3 oc = radiance;
      if (mode > 0.5f && mode < 1.5f) oc = mk(disparity, disparity, disparity);
      else if (mode > 1.5f && mode < 2.5f) oc = scl(0.5f, add(normal, mk(1, 1, 1)));
      else if (mode > 2.5f && mode < 3.5f) oc = mk(ao, ao, ao);
      else if (mode > 3.5f) oc = alb_lin;
      long o = (long)py * out_w + px;
      if (hdr) {
        hdr[o * 4] = oc.x;
        hdr[o * 4 + 1] = oc.y;
        hdr[o * 4 + 2] = oc.z;
        hdr[o * 4 + 3] = 1.0f;
      }
      if (rgba8) {
        float h3[3] = {oc.x, oc.y, oc.z}, s[3];
        or_composite_px(P->grade, h3, u, v, s);
        rgba8[o * 4] = to_unorm8(s[0]);
        rgba8[o * 4 + 1] = to_unorm8(s[1]);
        rgba8[o * 4 + 2] = to_unorm8(s[2]);
        rgba8[o * 4 + 3] = 255;
      }
    }
}

/* Bilinear resize of a single-channel map (align_corners=false with edge
 * clamp), used to bring the network's disparity to render resolution when
 * shading from an upsampled depth map. */
void or_resize_bilinear(const float *src, int sw, int sh, float *dst, int dw, int dh) {
  for (int y = 0; y < dh; y++)
    for (int x = 0; x < dw; x++) {
      float u = ((float)x + 0.5f) / (float)dw, v = ((float)y + 0.5f) / (float)dh;
      float tx = u * (float)sw - 0.5f, ty = v * (float)sh - 0.5f;
      float fx0 = floorf(tx), fy0 = floorf(ty);
      float fx = tx - fx0, fy = ty - fy0;
      int x0 = clampi((int)fx0, 0, sw - 1), x1 = clampi((int)fx0 + 1, 0, sw - 1);
      int y0 = clampi((int)fy0, 0, sh - 1), y1 = clampi((int)fy0 + 1, 0, sh - 1);
      float a = src[(long)y0 * sw + x0], b = src[(long)y0 * sw + x1];
      float cc = src[(long)y1 * sw + x0], d = src[(long)y1 * sw + x1];
      float top = a + (b - a) * fx, bot = cc + (d - cc) * fx;
      dst[(long)y * dw + x] = top + (bot - top) * fy;
    }
}
