/*
 * CPU oracle for the procedural scene and the depth metrics:
 *   - a scalar float32 restatement of the ray-marched SDF scene
 *     (src/scene/procedural.ts:36-273: sdSphere, sdBox, smoothUnion, the
 *     scene map, calcNormal, softShadow, materialColor, sceneFragment) and of
 *     its uniform updates (createProceduralScene, procedural.ts:295-330);
 *   - a double-precision restatement of evaluateDepth
 *     (src/scene/metrics.ts:66-161): least-squares scale/shift in disparity
 *     space, then AbsRel, RMSE and the delta thresholds, summed in the
 *     reference's sequential order.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by the test-suite, never by the product.
 *
 * The reference renders the scene as a WebGPU fragment shader into an
 * rgba8unorm colour target and an rgba16float truth target; it has no CPU
 * version. This transcription follows the shader's f32 expression order
 * (built with -ffp-contract=off); WGSL's mix(a, b, t) is a*(1-t) + b*t and
 * clamp(x, lo, hi) is min(max(x, lo), hi). The colour is converted to 8-bit
 * as an rgba8unorm store does (round to nearest of clamp(v)*255); the truth is
 * kept in float32 (the reference's half-float texture rounds it to 11 bits).
 */
#include <math.h>
#include <stdint.h>

typedef struct { float x, y, z; } v3;

static v3 mk(float x, float y, float z) { v3 r = {x, y, z}; return r; }
static v3 add(v3 a, v3 b) { return mk(a.x + b.x, a.y + b.y, a.z + b.z); }
static v3 sub(v3 a, v3 b) { return mk(a.x - b.x, a.y - b.y, a.z - b.z); }
static v3 scl(float s, v3 a) { return mk(s * a.x, s * a.y, s * a.z); }
static v3 vmul(v3 a, v3 b) { return mk(a.x * b.x, a.y * b.y, a.z * b.z); }
static float dot3(v3 a, v3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
static float len3(v3 a) { return sqrtf(dot3(a, a)); }
static v3 norm3(v3 a) { float l = len3(a); return mk(a.x / l, a.y / l, a.z / l); }
static v3 cross3(v3 a, v3 b) {
  return mk(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}
static float clampf_(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }
static float mixf(float a, float b, float t) { return a * (1.0f - t) + b * t; }

/* sdSphere, procedural.ts:36-42 */
static float sd_sphere(v3 p, float r) { return len3(p) - r; }

/* sdBox, procedural.ts:44-53 */
static float sd_box(v3 p, v3 b) {
  v3 q = sub(mk(fabsf(p.x), fabsf(p.y), fabsf(p.z)), b);
  v3 qp = mk(fmaxf(q.x, 0.0f), fmaxf(q.y, 0.0f), fmaxf(q.z, 0.0f));
  return len3(qp) + fminf(fmaxf(q.x, fmaxf(q.y, q.z)), 0.0f);
}

/* smoothUnion, procedural.ts:56-62 */
static float smooth_union(float a, float b, float k) {
  float h = clampf_(0.5f + (0.5f * (b - a)) / k, 0.0f, 1.0f);
  return mixf(b, a, h) - k * h * (1.0f - h);
}

/* The scene map, procedural.ts:70-125: returns the distance, material in *mat. */
static float scene_map(v3 p, float t, float *mat) {
  float dist = p.y + 1.0f + 0.06f * sinf(p.x * 0.7f) * cosf(p.z * 0.6f);
  float material = 1.0f;
  float bob = 0.12f * sinf(t * 0.9f);
  float a = sd_sphere(sub(p, mk(-0.35f, -0.25f + bob, -2.1f)), 0.62f);
  float b = sd_sphere(sub(p, mk(0.4f, -0.45f + bob * 0.6f, -1.75f)), 0.42f);
  float blob = smooth_union(a, b, 0.35f);
  if (blob < dist) { dist = blob; material = 2.0f; }
  for (int i = 0; i < 4; i++) {
    float x = -2.4f + (float)i * 1.55f;
    float z = -4.6f - (float)((i * 7) % 5) * 0.55f;
    float h = 0.9f + 0.35f * (float)((i * 3) % 4);
    float box = sd_box(sub(p, mk(x, -1.0f + h, z)), mk(0.22f, h, 0.22f));
    if (box < dist) { dist = box; material = 3.0f; }
  }
  float arch = fmaxf(sd_box(sub(p, mk(0.2f, 0.6f, -8.5f)), mk(2.6f, 1.9f, 0.3f)),
                     -sd_sphere(sub(p, mk(0.2f, -0.4f, -8.5f)), 1.7f));
  if (arch < dist) { dist = arch; material = 4.0f; }
  float nr = sd_sphere(sub(p, mk(1.25f + 0.25f * sinf(t * 0.5f), 0.15f, -1.15f)), 0.28f);
  if (nr < dist) { dist = nr; material = 5.0f; }
  if (mat) *mat = material;
  return dist;
}

/* calcNormal, procedural.ts:128-137 */
static v3 calc_normal(v3 p, float t) {
  const float e = 0.0015f;
  float dx = scene_map(add(p, mk(e, 0, 0)), t, 0) - scene_map(sub(p, mk(e, 0, 0)), t, 0);
  float dy = scene_map(add(p, mk(0, e, 0)), t, 0) - scene_map(sub(p, mk(0, e, 0)), t, 0);
  float dz = scene_map(add(p, mk(0, 0, e)), t, 0) - scene_map(sub(p, mk(0, 0, e)), t, 0);
  return norm3(mk(dx, dy, dz));
}

/* softShadow, procedural.ts:140-158 */
static float soft_shadow(v3 origin, v3 dir, float time) {
  float res = 1.0f, t = 0.04f;
  for (int i = 0; i < 28; i++) {
    float h = scene_map(add(origin, scl(t, dir)), time, 0);
    res = fminf(res, (12.0f * h) / t);
    t += clampf_(h, 0.02f, 0.4f);
    if (res < 0.002f || t > 12.0f) break;
  }
  return clampf_(res, 0.0f, 1.0f);
}

/* materialColor, procedural.ts:160-175 */
static v3 material_color(float material, v3 p) {
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

/* sceneFragment, procedural.ts:191-273, at uv; params = camera[4], focus[4], options[4]. */
static void scene_fragment(const float *P, float u, float v, float rgb[3], float *depth, float *hit_out) {
  const float *cam = P, *focus = P + 4, *opt = P + 8;
  float time = cam[3];
  v3 origin = mk(cam[0], cam[1], cam[2]);
  v3 look = mk(focus[0], focus[1], focus[2]);
  v3 forward = norm3(sub(look, origin));
  v3 right = norm3(cross3(forward, mk(0, 1, 0)));
  v3 up = cross3(right, forward);
  float ndc_x = u * 2.0f - 1.0f;
  float ndc_y = 1.0f - v * 2.0f;
  v3 dir = norm3(add(add(scl(ndc_x * opt[0] * focus[3], right), scl(ndc_y * focus[3], up)), forward));

  float t = 0.02f, material = 0.0f, hit = 0.0f;
  for (int i = 0; i < 96; i++) {
    float m;
    float s = scene_map(add(origin, scl(t, dir)), time, &m);
    if (s < 0.0015f * t) { hit = 1.0f; material = m; break; }
    t += s * 0.85f;
    if (t > opt[1]) { t = opt[1]; break; }
  }

  float horizon = clampf_(dir.y * 0.5f + 0.5f, 0.0f, 1.0f);
  v3 color = mk(mixf(0.42f, 0.12f, horizon), mixf(0.47f, 0.18f, horizon), mixf(0.55f, 0.32f, horizon));
  if (hit > 0.5f) {
    v3 pos = add(origin, scl(t, dir));
    v3 n = calc_normal(pos, time);
    v3 albedo = material_color(material, pos);
    float sa = opt[2];
    v3 sun = norm3(mk(cosf(sa), 0.72f, sinf(sa)));
    float shadow = soft_shadow(add(pos, scl(0.02f, n)), sun, time);
    float diffuse = fmaxf(dot3(n, sun), 0.0f) * shadow;
    float sky = 0.5f + 0.5f * n.y;
    float bounce = fmaxf(-n.y, 0.0f) * 0.2f;
    v3 light = add(add(scl(diffuse * 1.5f, mk(1.0f, 0.94f, 0.82f)), scl(sky * 0.35f, mk(0.35f, 0.45f, 0.65f))),
                   mk(bounce * 0.25f, bounce * 0.25f, bounce * 0.25f));
    v3 lit = vmul(albedo, light);
    v3 half = norm3(sub(sun, dir));
    float spec = powf(fmaxf(dot3(n, half), 0.0f), 48.0f) * shadow * 0.35f;
    color = add(lit, mk(spec, spec, spec));
    float fog = 1.0f - expf(-t * 0.055f);
    float f = clampf_(fog, 0.0f, 1.0f);
    color = mk(mixf(color.x, 0.3f, f), mixf(color.y, 0.36f, f), mixf(color.z, 0.46f, f));
  }
  float c3[3] = {color.x, color.y, color.z};
  for (int k = 0; k < 3; k++) {
    float mapped = c3[k] / (c3[k] + 0.6f);
    rgb[k] = powf(clampf_(mapped, 0.0f, 1.0f), 1.0f / 2.2f);
  }
  *depth = t * dot3(dir, forward);
  *hit_out = hit;
}

/* Uniforms of createProceduralScene: initial values (procedural.ts:295-299)
 * when initial != 0, else update(time, orbit) (:310-318). JavaScript doubles,
 * rounded to float32 when written. */
void or_scene_params(double time, int orbit, int initial, float out[12]) {
  double tan_half = tan((58.0 * M_PI) / 180.0 / 2.0);
  if (initial) {
    float v[12] = {0.0f, 0.35f, 0.6f, 0.0f, 0.0f, -0.15f, -3.0f, (float)tan_half, 1.0f, 30.0f, 0.9f, 0.0f};
    for (int i = 0; i < 12; i++) out[i] = v[i];
    return;
  }
  double angle = orbit ? sin(time * 0.18) * 0.5 : 0.0;
  double height = 0.35 + (orbit ? sin(time * 0.11) * 0.12 : 0.0);
  out[0] = (float)(sin(angle) * 1.4);
  out[1] = (float)height;
  out[2] = (float)(0.6 + cos(angle) * 0.3);
  out[3] = (float)time;
  out[4] = 0.0f; out[5] = -0.15f; out[6] = -3.0f; out[7] = (float)tan_half;
  out[8] = 1.0f; out[9] = 30.0f; out[10] = (float)(0.9 + time * 0.03); out[11] = 0.0f;
}

/* One frame of the scene at w x h: rgb (3 x h x w planar, the 8-bit colour as
 * value/255, nullable), rgba8 (h x w x 4, nullable), truth (h x w x 2: depth
 * along the view axis, hit mask; nullable). Pixel (x, y), y down, is the
 * fragment at uv = ((x + 0.5)/w, (y + 0.5)/h). */
void or_scene_render(const float *params, int w, int h, float *rgb, uint8_t *rgba8, float *truth) {
  for (int y = 0; y < h; y++) {
    for (int x = 0; x < w; x++) {
      float c[3], dep, hit;
      scene_fragment(params, ((float)x + 0.5f) / (float)w, ((float)y + 0.5f) / (float)h, c, &dep, &hit);
      long i = (long)y * w + x;
      for (int k = 0; k < 3; k++) {
        long q = lrintf(clampf_(c[k], 0.0f, 1.0f) * 255.0f);
        if (rgb) rgb[(long)k * w * h + i] = (float)q / 255.0f;
        if (rgba8) rgba8[i * 4 + k] = (uint8_t)q;
      }
      if (rgba8) rgba8[i * 4 + 3] = 255;
      if (truth) { truth[i * 2] = dep; truth[i * 2 + 1] = hit; }
    }
  }
}

/* evaluateDepth (metrics.ts:66-161) on float32 maps: pred channel 0 of
 * pred_ch-channel texels, truth (depth, hit) pairs. out = samples, absRel,
 * rmse, delta1, delta2, delta3, scale, shift. */
void or_evaluate_depth(const float *pred, int pred_ch, const float *truth, int w, int h, double out[8]) {
  long n = 0;
  double sxx = 0, sx = 0, sxy = 0, sy = 0;
  for (int row = 0; row < h; row++) {
    for (int col = 0; col < w; col++) {
      long i = (long)row * w + col;
      double hit = truth[i * 2 + 1], depth = truth[i * 2];
      if (hit < 0.5 || !(depth > 0.05) || depth > 25) continue;
      double xv = pred[i * pred_ch], yv = 1.0 / depth;
      sxx += xv * xv;
      sx += xv;
      sxy += xv * yv;
      sy += yv;
      n++;
    }
  }
  if (n < 64) {
    out[0] = (double)n;
    out[1] = out[2] = NAN;
    out[3] = out[4] = out[5] = 0;
    out[6] = out[7] = NAN;
    return;
  }
  double det = sxx * n - sx * sx;
  double scale = fabs(det) > 1e-12 ? (n * sxy - sx * sy) / det : 1;
  double shift = fabs(det) > 1e-12 ? (sxx * sy - sx * sxy) / det : 0;
  double abs_rel = 0, sq = 0;
  long d1 = 0, d2 = 0, d3 = 0, counted = 0;
  for (int row = 0; row < h; row++) {
    for (int col = 0; col < w; col++) {
      long i = (long)row * w + col;
      double hit = truth[i * 2 + 1], depth = truth[i * 2];
      if (hit < 0.5 || !(depth > 0.05) || depth > 25) continue;
      double disparity = scale * (double)pred[i * pred_ch] + shift;
      if (!(disparity > 1e-4)) continue;
      double zhat = 1.0 / disparity, z = depth;
      abs_rel += fabs(zhat - z) / z;
      sq += (zhat - z) * (zhat - z);
      double ratio = fmax(zhat / z, z / zhat);
      if (ratio < 1.25) d1++;
      if (ratio < 1.25 * 1.25) d2++;
      if (ratio < 1.25 * 1.25 * 1.25) d3++;
      counted++;
    }
  }
  double denom = counted > 1 ? (double)counted : 1.0;
  out[0] = (double)counted;
  out[1] = abs_rel / denom;
  out[2] = sqrt(sq / denom);
  out[3] = d1 / denom;
  out[4] = d2 / denom;
  out[5] = d3 / denom;
  out[6] = scale;
  out[7] = shift;
}
