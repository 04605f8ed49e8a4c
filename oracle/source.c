/*
 * CPU oracle for the source-texture read of makePreprocess
 * (src/model/kernels/io.ts:64-118): an 8-bit RGBA source of any size sampled
 * at the network's resolution with the uv transform
 *   uv = ((x + 0.5) / size, (y + 0.5) / size) * uvScale + uvOffset
 * (io.ts:76-84, runner.ts:181-182), u mirrored first when asked (blit.ts:57-60),
 * through a linear-filtering, clamp-to-edge sampler (runner.ts:177): texel
 * coordinate uv * extent - 0.5, the two neighbouring texels clamped to the
 * image, weights from the fractional part; texels read as unorm (v / 255).
 * And cropTransform (src/scene/blit.ts:80-86) in double, stored as float.
 *
 * TEST INFRASTRUCTURE ONLY. Float32 arithmetic, -ffp-contract=off. WebGPU
 * samplers filter with implementation-defined (often 8-bit) weight precision;
 * this restatement uses exact float32 weights, as the product does.
 */
#include <math.h>
#include <stdint.h>

static float clampf_s(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }

void or_sample_source(const uint8_t *rgba8, int n, int sw, int sh, const float *uv_scale, const float *uv_offset,
                      int mirror, int size, float *frames) {
  const float fs = (float)size;
  const long plane = (long)size * size;
  for (int f = 0; f < n; f++) {
    const uint8_t *img = rgba8 + (long)f * sw * sh * 4;
    for (int y = 0; y < size; y++) {
      for (int x = 0; x < size; x++) {
        float u = ((float)x + 0.5f) / fs, v = ((float)y + 0.5f) / fs;
        if (mirror) u = 1.0f - u;
        float uu = u * uv_scale[0] + uv_offset[0], vv = v * uv_scale[1] + uv_offset[1];
        float tx = uu * (float)sw - 0.5f, ty = vv * (float)sh - 0.5f;
        float fx0 = floorf(tx), fy0 = floorf(ty);
        float ax = tx - fx0, ay = ty - fy0;
        int x0 = (int)clampf_s(fx0, 0.0f, (float)(sw - 1)), x1 = (int)clampf_s(fx0 + 1.0f, 0.0f, (float)(sw - 1));
        int y0 = (int)clampf_s(fy0, 0.0f, (float)(sh - 1)), y1 = (int)clampf_s(fy0 + 1.0f, 0.0f, (float)(sh - 1));
        float w00 = (1.0f - ax) * (1.0f - ay), w10 = ax * (1.0f - ay), w01 = (1.0f - ax) * ay, w11 = ax * ay;
        const uint8_t *a = img + ((long)y0 * sw + x0) * 4, *b = img + ((long)y0 * sw + x1) * 4;
        const uint8_t *c = img + ((long)y1 * sw + x0) * 4, *d = img + ((long)y1 * sw + x1) * 4;
        for (int k = 0; k < 3; k++) {
          float s = ((float)a[k] / 255.0f) * w00;
          s = s + ((float)b[k] / 255.0f) * w10;
          s = s + ((float)c[k] / 255.0f) * w01;
          s = s + ((float)d[k] / 255.0f) * w11;
          frames[((long)f * 3 + k) * plane + (long)y * size + x] = s;
        }
      }
    }
  }
}

void or_crop_transform(int width, int height, float out[4]) {
  if (width <= 0 || height <= 0) {
    out[0] = 1, out[1] = 1, out[2] = 0, out[3] = 0;
    return;
  }
  double sx = width > height ? (double)height / width : 1.0;
  double sy = height > width ? (double)width / height : 1.0;
  out[0] = (float)sx, out[1] = (float)sy, out[2] = (float)((1 - sx) / 2), out[3] = (float)((1 - sy) / 2);
}
