/*
 * CPU oracle for the IlluminaDepth-448 network: a scalar restatement of the
 * reference's normative CPU implementation, src/model/reference.ts.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA path: only
 * the test-suite, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load it. The product library never links or calls it.
 *
 * Numeric contract (mirrors JavaScript number semantics in reference.ts):
 *   - tensors are float32, channels-last: data[(y*W + x)*C + c];
 *   - every accumulation runs in double (JS numbers), starting from the f32
 *     bias, adding f32*f32 products (exact in double);
 *   - the activation is applied in double and the result rounded to f32 on
 *     store (Float32Array assignment);
 *   - the fused dw->pw op materialises the depthwise output as f32 between the
 *     two halves, exactly like refDepthwisePointwise (reference.ts:138-153).
 * Build with -ffp-contract=off so the compiler never fuses a*b+c.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ACT_LINEAR = 0, ACT_RELU = 1, ACT_RELU6 = 2, ACT_HARDSWISH = 3 };

/* Math.max(v, 0) / Math.min(v, 6) keep NaN; so do these. */
static double js_max(double a, double b) {
  if (a != a || b != b) return NAN;
  return a > b ? a : b;
}
static double js_min(double a, double b) {
  if (a != a || b != b) return NAN;
  return a < b ? a : b;
}

/* applyActivation, src/model/layout.ts:131-142 */
static double act_apply(int act, double v) {
  switch (act) {
    case ACT_RELU: return js_max(v, 0.0);
    case ACT_RELU6: return js_min(js_max(v, 0.0), 6.0);
    case ACT_HARDSWISH: return (v * js_min(js_max(v + 3.0, 0.0), 6.0)) / 6.0;
    default: return v;
  }
}

double or_activation(int act, double v) { return act_apply(act, v); }

static int out_extent(int in, int k, int stride) {
  int pad = (k - 1) >> 1;
  /* Math.floor((src.h + 2*pad - k) / stride) + 1, operands non-negative here */
  int num = in + 2 * pad - k;
  int q = num >= 0 ? num / stride : -((-num + stride - 1) / stride);
  return q + 1;
}

int or_out_extent(int in, int k, int stride) { return out_extent(in, k, stride); }

/* refPointwise, reference.ts:35-57 */
void or_pointwise(const float *src, long pixels, int inC, const float *w,
                  const float *bias, int outC, int act, const float *res,
                  float *out) {
  for (long p = 0; p < pixels; p++) {
    const float *x = src + p * inC;
    for (int oc = 0; oc < outC; oc++) {
      double sum = bias[oc];
      const float *wr = w + (long)oc * inC;
      for (int ic = 0; ic < inC; ic++) sum += (double)wr[ic] * (double)x[ic];
      if (res) sum += res[p * outC + oc];
      out[p * outC + oc] = (float)act_apply(act, sum);
    }
  }
}

/* refConv, reference.ts:60-96 (weights [outC][inC][k][k]) */
void or_conv(const float *src, int h, int w, int inC, const float *wt,
             const float *bias, int outC, int k, int stride, int act,
             float *out) {
  int pad = (k - 1) >> 1;
  int oh = out_extent(h, k, stride), ow = out_extent(w, k, stride);
  for (int y = 0; y < oh; y++)
    for (int x = 0; x < ow; x++)
      for (int oc = 0; oc < outC; oc++) {
        double sum = bias[oc];
        for (int ky = 0; ky < k; ky++) {
          int sy = y * stride + ky - pad;
          if (sy < 0 || sy >= h) continue;
          for (int kx = 0; kx < k; kx++) {
            int sx = x * stride + kx - pad;
            if (sx < 0 || sx >= w) continue;
            const float *px = src + ((long)sy * w + sx) * inC;
            for (int ic = 0; ic < inC; ic++)
              sum += (double)wt[(((long)oc * inC + ic) * k + ky) * k + kx] * (double)px[ic];
          }
        }
        out[((long)y * ow + x) * outC + oc] = (float)act_apply(act, sum);
      }
}

/* refDepthwise, reference.ts:99-131 (weights [C][k][k]) */
void or_depthwise(const float *src, int h, int w, int C, const float *wt,
                  const float *bias, int k, int stride, int act, float *out) {
  int pad = (k - 1) >> 1;
  int oh = out_extent(h, k, stride), ow = out_extent(w, k, stride);
  for (int y = 0; y < oh; y++)
    for (int x = 0; x < ow; x++)
      for (int c = 0; c < C; c++) {
        double sum = bias[c];
        for (int ky = 0; ky < k; ky++) {
          int sy = y * stride + ky - pad;
          if (sy < 0 || sy >= h) continue;
          for (int kx = 0; kx < k; kx++) {
            int sx = x * stride + kx - pad;
            if (sx < 0 || sx >= w) continue;
            sum += (double)wt[((long)c * k + ky) * k + kx] *
                   (double)src[((long)sy * w + sx) * C + c];
          }
        }
        out[((long)y * ow + x) * C + c] = (float)act_apply(act, sum);
      }
}

/* refDepthwisePointwise, reference.ts:138-153 */
int or_dwpw(const float *src, int h, int w, int inC, const float *dw_w,
            const float *dw_b, int mid_act, const float *pw_w,
            const float *pw_b, int outC, int k, int stride, int act,
            const float *res, float *out) {
  int oh = out_extent(h, k, stride), ow = out_extent(w, k, stride);
  float *mid = (float *)malloc(sizeof(float) * (size_t)oh * ow * inC);
  if (!mid) return -1;
  or_depthwise(src, h, w, inC, dw_w, dw_b, k, stride, mid_act, mid);
  or_pointwise(mid, (long)oh * ow, inC, pw_w, pw_b, outC, act, res, out);
  free(mid);
  return 0;
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* refUpsample2, reference.ts:161-193 (align_corners=false, taps clamped
 * independently from the unclamped floor). */
void or_upsample2(const float *src, int h, int w, int C, float *out) {
  int oh = h * 2, ow = w * 2;
  for (int y = 0; y < oh; y++) {
    double sy = (y + 0.5) / 2 - 0.5;
    double fy0 = floor(sy);
    int y0 = clampi((int)fy0, 0, h - 1), y1 = clampi((int)fy0 + 1, 0, h - 1);
    double fy = sy - fy0;
    for (int x = 0; x < ow; x++) {
      double sx = (x + 0.5) / 2 - 0.5;
      double fx0 = floor(sx);
      int x0 = clampi((int)fx0, 0, w - 1), x1 = clampi((int)fx0 + 1, 0, w - 1);
      double fx = sx - fx0;
      for (int c = 0; c < C; c++) {
        double a = src[((long)y0 * w + x0) * C + c];
        double b = src[((long)y0 * w + x1) * C + c];
        double cc = src[((long)y1 * w + x0) * C + c];
        double dd = src[((long)y1 * w + x1) * C + c];
        out[((long)y * ow + x) * C + c] =
            (float)(a * (1 - fx) * (1 - fy) + b * fx * (1 - fy) +
                    cc * (1 - fx) * fy + dd * fx * fy);
      }
    }
  }
}

/* refLateral, reference.ts:202-231. Returns -1 on a channel/shape mismatch. */
int or_lateral(const float *coarse, int ch, int cw, int coarseC,
               const float *skip, int sh, int sw, int skipC, const float *wt,
               const float *bias, int outC, int act, float *out) {
  if (coarseC != outC) return -1;
  if (ch * 2 != sh || cw * 2 != sw) return -2;
  float *up = (float *)malloc(sizeof(float) * (size_t)sh * sw * outC);
  if (!up) return -3;
  or_upsample2(coarse, ch, cw, coarseC, up);
  long pixels = (long)sh * sw;
  for (long p = 0; p < pixels; p++)
    for (int oc = 0; oc < outC; oc++) {
      double sum = (double)bias[oc] + (double)up[p * outC + oc];
      for (int ic = 0; ic < skipC; ic++)
        sum += (double)wt[(long)oc * skipC + ic] * (double)skip[p * skipC + ic];
      out[p * outC + oc] = (float)act_apply(act, sum);
    }
  free(up);
  return 0;
}

/* refHead, reference.ts:241-257: sigmoid(b + w.x), broadcast to 4 channels. */
void or_head(const float *src, long pixels, int C, const float *wt, float bias,
             float *out4) {
  for (long p = 0; p < pixels; p++) {
    double sum = bias;
    for (int ic = 0; ic < C; ic++) sum += (double)wt[ic] * (double)src[p * C + ic];
    float d = (float)(1 / (1 + exp(-sum)));
    out4[p * 4] = d;
    out4[p * 4 + 1] = d;
    out4[p * 4 + 2] = d;
    out4[p * 4 + 3] = d;
  }
}

/* Head logit (pre-sigmoid), for scale-relative checks of the last conv. */
void or_head_logit(const float *src, long pixels, int C, const float *wt,
                   float bias, double *logit) {
  for (long p = 0; p < pixels; p++) {
    double sum = bias;
    for (int ic = 0; ic < C; ic++) sum += (double)wt[ic] * (double)src[p * C + ic];
    logit[p] = sum;
  }
}

/* srgbToLinearScalar, reference.ts:264-266 */
static double srgb_to_linear(double c) {
  return c <= 0.04045 ? c / 12.92 : pow((c + 0.055) / 1.055, 2.4);
}

/* luminanceOf, reference.ts:268-270 */
static double luminance_of(double r, double g, double b) {
  return 0.2126 * r + 0.7152 * g + 0.0722 * b;
}

/* refPreprocess, reference.ts:283-308. `rgba` is size*size*4 in [0,1]. */
void or_preprocess(const float *rgba, int size, const double *mean,
                   const double *stdv, int decode_srgb, double exposure,
                   float *input, float *scene) {
  long n = (long)size * size;
  for (long p = 0; p < n; p++) {
    double lin[3];
    for (int i = 0; i < 3; i++) {
      double v = rgba[p * 4 + i];
      lin[i] = (decode_srgb ? srgb_to_linear(v) : v) * exposure;
    }
    scene[p * 4] = (float)lin[0];
    scene[p * 4 + 1] = (float)lin[1];
    scene[p * 4 + 2] = (float)lin[2];
    scene[p * 4 + 3] = 1.0f;
    for (int i = 0; i < 3; i++) input[p * 4 + i] = (float)((lin[i] - mean[i]) / stdv[i]);
    input[p * 4 + 3] = (float)luminance_of(lin[0], lin[1], lin[2]);
  }
}

/* refBilateralUpsample, reference.ts:314-353 (first frame, no history).
 * low: lh x lw x lc (channel 0 read); guide: (2*lh) x gw x gc. */
void or_bilateral(const float *low, int lh, int lw, int lc, const float *guide,
                  int gw, int gc, double range_sigma, float *out) {
  int full = lh * 2;
  double inv_sigma_den = range_sigma > 1e-4 ? range_sigma : 1e-4;
  for (int y = 0; y < full; y++)
    for (int x = 0; x < full; x++) {
      const float *gh = guide + ((long)y * gw + x) * gc;
      double luma_here = luminance_of(gh[0], gh[1], gh[2]);
      double cx = (x + 0.5) * 0.5 - 0.5;
      double cy = (y + 0.5) * 0.5 - 0.5;
      int bx = (int)floor(cx + 0.5);
      int by = (int)floor(cy + 0.5);
      double weighted = 0, total = 0;
      for (int dy = -1; dy <= 1; dy++)
        for (int dx = -1; dx <= 1; dx++) {
          int qx = clampi(bx + dx, 0, lw - 1);
          int qy = clampi(by + dy, 0, lh - 1);
          double disparity = low[((long)qy * lw + qx) * lc];
          const float *gt = guide + ((long)(qy * 2) * gw + qx * 2) * gc;
          double luma_there = luminance_of(gt[0], gt[1], gt[2]);
          double dxs = qx - cx, dys = qy - cy;
          double spatial = exp(-(dxs * dxs + dys * dys) * 0.5);
          double dl = (luma_here - luma_there) / inv_sigma_den;
          double wgt = spatial * exp(-dl * dl * 0.5);
          weighted += disparity * wgt;
          total += wgt;
        }
      out[(long)y * full + x] = (float)(weighted / (total > 1e-6 ? total : 1e-6));
    }
}

/* ------------------------------------------------------------------------
 * Deterministic initialisation, src/model/weights.ts:200-251
 * ------------------------------------------------------------------------ */

typedef struct { uint32_t a; } mb32;

/* mulberry32, weights.ts:200-209 (also test/helpers/tensors.ts:6-16) */
static double mb32_next(mb32 *s) {
  s->a = s->a + 0x6d2b79f5u;
  uint32_t t = s->a;
  t = (t ^ (t >> 15)) * (t | 1u);
  t ^= t + (t ^ (t >> 7)) * (t | 61u);
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

void or_mulberry32(uint32_t seed, long n, double *out) {
  mb32 s = {seed};
  for (long i = 0; i < n; i++) out[i] = mb32_next(&s);
}

/* gaussian, weights.ts:212-216 */
static double mb32_gaussian(mb32 *s) {
  double u = mb32_next(s);
  if (u < 1e-9) u = 1e-9;
  double v = mb32_next(s);
  return sqrt(-2 * log(u)) * cos(2 * M_PI * v);
}

/* synthesizeWeights, weights.ts:227-251. One PRNG stream consumed in spec
 * order; biases are zero and draw nothing. `fan_in[i]` and flags per tensor
 * come from the caller's restatement of weightSpecs. */
void or_synthesize(uint32_t seed, int n_specs, const long *counts,
                   const long *fan_in, const int *is_bias, const int *is_head,
                   float *blob) {
  mb32 s = {seed};
  long off = 0;
  for (int i = 0; i < n_specs; i++) {
    long n = counts[i];
    if (is_bias[i]) {
      memset(blob + off, 0, sizeof(float) * (size_t)n);
      off += n;
      continue;
    }
    double stdv = sqrt(2.0 / (double)(fan_in[i] > 1 ? fan_in[i] : 1));
    double scale = is_head[i] ? stdv * 0.05 : stdv;
    for (long j = 0; j < n; j++) blob[off + j] = (float)(mb32_gaussian(&s) * scale);
    off += n;
  }
}

/* randomFloats, test/helpers/tensors.ts:18-22: (rand()*2-1)*scale as f32.
 * The PRNG state is passed in and out so several draws can share a stream. */
uint32_t or_random_floats(uint32_t state, long n, double scale, float *out) {
  mb32 s = {state};
  for (long i = 0; i < n; i++) out[i] = (float)((mb32_next(&s) * 2 - 1) * scale);
  return s.a;
}

/* Seeded uniform [0,1) frame in NCHW order (c, y, x), float32(r). */
void or_uniform_frame(uint32_t seed, long n, float *out) {
  mb32 s = {seed};
  for (long i = 0; i < n; i++) out[i] = (float)mb32_next(&s);
}

/* halfToFloat, weights.ts:82-95 */
double or_half_to_float(uint32_t h) {
  int sign = (h & 0x8000) >> 15;
  int e = (h & 0x7c00) >> 10;
  int frac = h & 0x03ff;
  double value;
  if (e == 0) value = frac * ldexp(1.0, -24);
  else if (e == 0x1f) value = frac == 0 ? INFINITY : NAN;
  else value = (frac + 1024) * ldexp(1.0, e - 25);
  return sign ? -value : value;
}
