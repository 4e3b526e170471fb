// eg_host.cpp -- host-side parts of libemberglass_cuda: the reference's
// quantisers (bit-exact, JS double semantics), RoPE tables, and the seeded
// synthetic-weight generator.  Compiled with -ffp-contract=off so every
// double/float operation is rounded exactly as written.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "emberglass.h"
#include "eg_host.h"

namespace eg {

static inline uint64_t sm_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
uint64_t stream_at(uint64_t seed, uint64_t k) { return sm_mix(seed + (k + 1) * 0x9E3779B97F4A7C15ULL); }
static inline double u01(uint64_t z) { return (double)(z >> 11) * 0x1.0p-53; }

// Element e of the normal stream: Box-Muller over stream outputs 2e, 2e+1.
void fill_normal(float* out, int64_t n, uint64_t seed, double stdv, int64_t start) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) {
    const uint64_t e = (uint64_t)(start + i);
    const double a = 1.0 - u01(stream_at(seed, 2 * e));
    const double b = u01(stream_at(seed, 2 * e + 1));
    const double r = sqrt(-2.0 * log(a));
    const double c = cos(6.283185307179586 * b);
    out[i] = (float)(stdv * (r * c));
  }
}

// JS Math.round: nearest, halves toward +infinity (quantize.js:42, :97).
static inline double js_round(double x) {
  double r = floor(x);
  if (x - r >= 0.5) r += 1.0;
  return r;
}

void rope_tables(int max_ctx, int hd, double theta, float* cosT, float* sinT) {
  const int half = hd / 2;
  for (int p = 0; p < max_ctx; p++)
    for (int i = 0; i < half; i++) {  // _buildRope, runtime.js:572-590
      const double a = p / pow(theta, (2.0 * i) / hd);
      const double cc = cos(a), ss = sin(a);
      cosT[(int64_t)p * hd + i] = (float)cc;
      cosT[(int64_t)p * hd + half + i] = (float)cc;
      sinT[(int64_t)p * hd + i] = (float)ss;
      sinT[(int64_t)p * hd + half + i] = (float)ss;
    }
}

}  // namespace eg

extern "C" {

// quantizeInt4Group (quantize.js:81-111): amax, s = amax/7 and inv = 1/s in
// double; the stored scale is f32(s) while inv keeps the unrounded s.
EG_API eg_status eg_quantize_int4_group(const float* W, int N, int K, int group, uint32_t* packed,
                                        float* scale) {
  if (!W || !packed || !scale || N < 0 || K <= 0 || group <= 0 || K % group || group % 8)
    return eg::fail(EG_ERR_ARG, "quantizeInt4Group: need K % group == 0 and group % 8 == 0");
  const int gpr = K / group;
#pragma omp parallel for schedule(static)
  for (int o = 0; o < N; o++) {
    for (int g = 0; g < gpr; g++) {
      const float* src = W + (int64_t)o * K + (int64_t)g * group;
      double amax = 0;
      for (int i = 0; i < group; i++) {
        const double a = fabs((double)src[i]);
        if (a > amax) amax = a;
      }
      const double s = amax > 0 ? amax / 7 : 1;
      scale[(int64_t)o * gpr + g] = (float)s;
      const double inv = 1 / s;
      uint32_t* dst = packed + ((int64_t)o * K + (int64_t)g * group) / 8;
      for (int w = 0; w < group / 8; w++) {
        uint32_t acc = 0;
        for (int j = 0; j < 8; j++) {
          double v = eg::js_round((double)src[w * 8 + j] * inv);
          if (v > 7) v = 7;
          else if (v < -8) v = -8;
          acc |= ((uint32_t)(int32_t)v & 0xFu) << (4 * j);
        }
        dst[w] = acc;
      }
    }
  }
  return EG_OK;
}

// quantizeInt8RowMajor (quantize.js:28-57).
EG_API eg_status eg_quantize_int8_rows(const float* W, int N, int K, uint32_t* packed, float* scale) {
  if (!W || !packed || !scale || N < 0 || K <= 0 || K % 4)
    return eg::fail(EG_ERR_ARG, "quantizeInt8RowMajor: need K % 4 == 0");
#pragma omp parallel for schedule(static)
  for (int o = 0; o < N; o++) {
    const float* src = W + (int64_t)o * K;
    double amax = 0;
    for (int i = 0; i < K; i++) {
      const double a = fabs((double)src[i]);
      if (a > amax) amax = a;
    }
    const double s = amax > 0 ? amax / 127 : 1;
    scale[o] = (float)s;
    const double inv = 1 / s;
    uint8_t* dst = reinterpret_cast<uint8_t*>(packed + (int64_t)o * K / 4);
    for (int i = 0; i < K; i++) {
      double v = eg::js_round((double)src[i] * inv);
      if (v > 127) v = 127;
      else if (v < -128) v = -128;
      dst[i] = (uint8_t)(int8_t)v;
    }
  }
  return EG_OK;
}

// Synthetic-input stream exposed for cross-checks (same generator the
// synthetic model build uses).
EG_API void eg_synth_normal(float* out, int64_t n, uint64_t seed, double stdv, int64_t start) {
  eg::fill_normal(out, n, seed, stdv, start);
}
EG_API uint64_t eg_synth_stream_at(uint64_t seed, uint64_t k) { return eg::stream_at(seed, k); }

}  // extern "C"
