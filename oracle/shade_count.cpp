// Op-counting build of the shading restatement (oracle/shade.c).
//
// TEST / MEASUREMENT INFRASTRUCTURE ONLY: it produces the algorithmic FLOP
// count per pixel of the depth-aware shading + tone-map pass that the
// benchmark divides by the measured kernel time; nothing in the product
// loads it.
//
// shade.c is compiled here as C++ with `float` replaced by a type that
// performs the same float32 operation and counts it: + - * / and each
// comparison, min/max, floor and fabs count 1, a fused multiply-add 2, and
// each transcendental or root (sqrt, exp, pow, sin, cos) 1. Integer index
// arithmetic is not counted. or_shade_flops runs or_shade over a band of
// rows and returns the operations per shaded pixel.
#include <cmath>
#include <cstdint>
#include <math.h>
#include <stdint.h>

namespace {
thread_local unsigned long long g_ops = 0;

struct cf {
  float v;
  cf() : v(0.0f) {}
  cf(float x) : v(x) {}  // NOLINT: literals and ints convert implicitly, as in C
  cf(double x) : v((float)x) {}
  cf(int x) : v((float)x) {}
  explicit operator int() const { return (int)v; }
  explicit operator uint8_t() const { return (uint8_t)v; }
  cf &operator+=(cf o) { ++g_ops; v += o.v; return *this; }
  cf &operator-=(cf o) { ++g_ops; v -= o.v; return *this; }
  cf &operator*=(cf o) { ++g_ops; v *= o.v; return *this; }
  cf &operator/=(cf o) { ++g_ops; v /= o.v; return *this; }
};
inline cf operator+(cf a, cf b) { ++g_ops; return cf(a.v + b.v); }
inline cf operator-(cf a, cf b) { ++g_ops; return cf(a.v - b.v); }
inline cf operator*(cf a, cf b) { ++g_ops; return cf(a.v * b.v); }
inline cf operator/(cf a, cf b) { ++g_ops; return cf(a.v / b.v); }
inline cf operator-(cf a) { return cf(-a.v); }
inline bool operator<(cf a, cf b) { ++g_ops; return a.v < b.v; }
inline bool operator>(cf a, cf b) { ++g_ops; return a.v > b.v; }
inline bool operator<=(cf a, cf b) { ++g_ops; return a.v <= b.v; }
inline bool operator>=(cf a, cf b) { ++g_ops; return a.v >= b.v; }
inline bool operator!(cf a) { return !a.v; }
inline cf sqrtf(cf a) { ++g_ops; return cf(std::sqrt(a.v)); }
inline cf floorf(cf a) { ++g_ops; return cf(std::floor(a.v)); }
inline cf fabsf(cf a) { ++g_ops; return cf(std::fabs(a.v)); }
inline cf expf(cf a) { ++g_ops; return cf(std::exp(a.v)); }
inline cf powf(cf a, cf b) { ++g_ops; return cf(std::pow(a.v, b.v)); }
inline cf sinf(cf a) { ++g_ops; return cf(std::sin(a.v)); }
inline cf cosf(cf a) { ++g_ops; return cf(std::cos(a.v)); }
inline cf fmaf(cf a, cf b, cf c) { g_ops += 2; return cf(std::fma(a.v, b.v, c.v)); }
}  // namespace

#define float cf
#define or_ggx_d count_ggx_d
#define or_smith_g count_smith_g
#define or_composite_px count_composite_px
#define or_shade count_shade
#define or_resize_bilinear count_resize_bilinear
#include "shade.c"
#undef float

// (the resize is not part of the counted pass; referenced so the build has no unused function)
void *const kResizeUnused = reinterpret_cast<void *>(&count_resize_bilinear);

// Operations per pixel of or_shade over rows [row0, row1) (inputs as or_shade's).
extern "C" double or_shade_flops(const float *depth, int dw, int dh, const float *albedo, int aw, int ah,
                                 const or_light *lights, int n_lights, const or_shade_params *P,
                                 const or_steps *st, int out_w, int out_h, int row0, int row1) {
  static_assert(sizeof(cf) == sizeof(float), "counting float has float's layout");
  g_ops = 0;
  // the counting type has float's layout, so the float arrays are read in place
  count_shade(reinterpret_cast<const cf *>(depth), dw, dh, reinterpret_cast<const cf *>(albedo), aw, ah, lights,
              n_lights, P, st, out_w, out_h, row0, row1, nullptr, nullptr);
  const double px = (double)(row1 - row0) * out_w;
  return px > 0 ? (double)g_ops / px : 0.0;
}
