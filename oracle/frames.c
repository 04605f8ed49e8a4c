/* Seeded blob frames (the batched-throughput workload's input), host side.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the device generator
 * (k_gen_blobs) and the input of the timed CPU baseline.
 *
 * Workload definition (smooth procedural images): per frame seed and channel
 * c, 8 anisotropic Gaussian blobs drawn from one mulberry32 stream
 * (src/model/weights.ts:200-209) at positions d = (c*8 + b)*6 .. +5:
 * centre (u0*S, u1*S), sigma_x = 20 + 100*u2, sigma_y = 20 + 100*u3 pixels,
 * rotation u4*pi, amplitude u5. Value at pixel centre (x+0.5, y+0.5) is the
 * sum of amp*exp(-(u^2/(2 sx^2) + w^2/(2 sy^2))) over the blobs, with (u, w)
 * the rotated offset, plus N(0, 0.02) noise by Box-Muller on draws
 * 144 + 2j and 145 + 2j (j = the value's (c, y, x) index; the transform of
 * weights.ts:212-216, u clamped to 1e-9), clamped to [0, 1].
 *
 * Every operation is an IEEE-754 double add, multiply, divide, square root
 * or fused multiply-add in a fixed order, and the elementary functions are
 * written here from their series (exp: Cody-Waite reduction by ln 2 and the
 * Taylor series to r^13/13!; log: the atanh series
 * log m = 2 atanh((m-1)/(m+1)) after reducing m to [sqrt(1/2), sqrt(2)];
 * sin/cos: Taylor series on [-pi/2, pi/2]). The device generator evaluates
 * the same operations in the same order with round-to-nearest intrinsics, so
 * the two produce identical bits; the functions are within a few ulp of libm
 * (checked by the tests), so the frames are the Gaussian-blob images above.
 * Built with -ffp-contract=off: no product is fused unless written as fma().
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static double mb32_at(uint32_t seed, uint32_t j) {
  uint32_t t = seed + (j + 1u) * 0x6d2b79f5u;
  t = (t ^ (t >> 15)) * (t | 1u);
  t ^= t + (t ^ (t >> 7)) * (t | 61u);
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

static const double kLn2Hi = 0.6931471803691238;      /* 0x1.62e42feep-1: k*hi exact */
static const double kLn2Lo = 1.9082149292705877e-10;  /* ln 2 - hi */
static const double kInvLn2 = 1.4426950408889634;
static const double kPi = 3.141592653589793;
static const double kPiHalf = 1.5707963267948966;
static const double kTwoPi = 6.283185307179586;
static const double kSqrt2 = 1.4142135623730951;

static double pow2i(int k) { /* 2^k for -1022 <= k <= 1023 */
  uint64_t b = (uint64_t)(k + 1023) << 52;
  double r;
  memcpy(&r, &b, 8);
  return r;
}

/* exp(x) for x <= 0 (0 below -708). */
double or_det_exp(double x) {
  static const double c[12] = {0.5, 0.16666666666666666, 0.041666666666666664, 0.008333333333333333,
                               0.001388888888888889, 0.0001984126984126984, 2.48015873015873e-05,
                               2.7557319223985893e-06, 2.755731922398589e-07, 2.505210838544172e-08,
                               2.08767569878681e-09, 1.6059043836821613e-10};
  if (x < -708.0) return 0.0;
  double kd = floor(fma(x, kInvLn2, 0.5));
  double r = fma(-kd, kLn2Hi, x);
  r = fma(-kd, kLn2Lo, r);
  double p = c[11];
  for (int i = 10; i >= 0; i--) p = fma(p, r, c[i]);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  return p * pow2i((int)kd);
}

/* log(u) for normal u > 0. */
double or_det_log(double u) {
  static const double c[12] = {0.3333333333333333, 0.2, 0.14285714285714285, 0.1111111111111111,
                               0.09090909090909091, 0.07692307692307693, 0.06666666666666667,
                               0.058823529411764705, 0.05263157894736842, 0.047619047619047616,
                               0.043478260869565216, 0.04};
  uint64_t b;
  memcpy(&b, &u, 8);
  int e = (int)((b >> 52) & 0x7ff) - 1023;
  b = (b & 0x000fffffffffffffull) | 0x3ff0000000000000ull;
  double m;
  memcpy(&m, &b, 8);
  if (m > kSqrt2) {
    m = m * 0.5;
    e += 1;
  }
  double s = (m - 1.0) / (m + 1.0);
  double z = s * s;
  double p = c[11];
  for (int i = 10; i >= 0; i--) p = fma(p, z, c[i]);
  p = fma(p, z, 1.0);
  double lm = (s + s) * p;
  double ed = (double)e;
  return fma(ed, kLn2Hi, fma(ed, kLn2Lo, lm));
}

/* cos(t), sin(t) for |t| <= pi/2 */
static double cos_poly(double t) {
  static const double c[12] = {-0.5, 0.041666666666666664, -0.001388888888888889, 2.48015873015873e-05,
                               -2.755731922398589e-07, 2.08767569878681e-09, -1.1470745597729725e-11,
                               4.779477332387385e-14, -1.5619206968586225e-16, 4.110317623312165e-19,
                               -8.896791392450574e-22, 1.6117375710961184e-24};
  double z = t * t;
  double p = c[11];
  for (int i = 10; i >= 0; i--) p = fma(p, z, c[i]);
  return fma(p, z, 1.0);
}

static double sin_poly(double t) {
  static const double c[11] = {-0.16666666666666666, 0.008333333333333333, -0.0001984126984126984,
                               2.7557319223985893e-06, -2.505210838544172e-08, 1.6059043836821613e-10,
                               -7.647163731819816e-13, 2.8114572543455206e-15, -8.22063524662433e-18,
                               1.9572941063391263e-20, -3.868170170630684e-23};
  double z = t * t;
  double p = c[10];
  for (int i = 9; i >= 0; i--) p = fma(p, z, c[i]);
  p = fma(p, z, 1.0);
  return t * p;
}

/* cos and sin of th in [0, pi): th = t + pi/2 with |t| <= pi/2. */
void or_det_sincos(double th, double *s, double *c) {
  double t = th - kPiHalf;
  *c = -sin_poly(t);
  *s = cos_poly(t);
}

/* cos(2 pi v) for v in [0, 1) (v a multiple of 2^-32: the reductions are exact). */
double or_det_cos2pi(double v) {
  double w = v - floor(v + 0.5);
  double a = fabs(w);
  if (a <= 0.25) return cos_poly(a * kTwoPi);
  return -cos_poly((0.5 - a) * kTwoPi);
}

typedef struct {
  double cx, cy, hx, hy, cs, sn, amp;
} Blob;

static void blob_params(uint32_t seed, int c, int b, int S, Blob *o) {
  uint32_t d = (uint32_t)((c * 8 + b) * 6);
  o->cx = mb32_at(seed, d) * (double)S;
  o->cy = mb32_at(seed, d + 1) * (double)S;
  double sx = fma(mb32_at(seed, d + 2), 100.0, 20.0);
  double sy = fma(mb32_at(seed, d + 3), 100.0, 20.0);
  o->hx = 0.5 / (sx * sx);
  o->hy = 0.5 / (sy * sy);
  or_det_sincos(mb32_at(seed, d + 4) * kPi, &o->sn, &o->cs);
  o->amp = mb32_at(seed, d + 5);
}

/* One [3][S][S] blob frame of `seed`. */
void or_blob_frame(uint32_t seed, int S, float *out) {
  for (int c = 0; c < 3; c++) {
    Blob bl[8];
    for (int b = 0; b < 8; b++) blob_params(seed, c, b, S, &bl[b]);
    for (int y = 0; y < S; y++)
      for (int x = 0; x < S; x++) {
        double v = 0.0;
        const double px = (double)x + 0.5, py = (double)y + 0.5;
        for (int b = 0; b < 8; b++) {
          const Blob *B = &bl[b];
          double dx = px - B->cx, dy = py - B->cy;
          double u = fma(B->cs, dx, B->sn * dy);
          double w = fma(B->cs, dy, -(B->sn * dx));
          double q = fma(u * u, B->hx, (w * w) * B->hy);
          v = fma(B->amp, or_det_exp(-q), v);
        }
        uint32_t j = (uint32_t)(((long)c * S + y) * S + x);
        uint32_t nd = 144u + 2u * j;
        double uu = mb32_at(seed, nd);
        if (uu < 1e-9) uu = 1e-9;
        double g = sqrt(-2.0 * or_det_log(uu)) * or_det_cos2pi(mb32_at(seed, nd + 1));
        v = fma(0.02, g, v);
        v = v < 0.0 ? 0.0 : (v > 1.0 ? 1.0 : v);
        out[((long)c * S + y) * S + x] = (float)v;
      }
  }
}
