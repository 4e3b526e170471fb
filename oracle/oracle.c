/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement, in plain C, of the Emberglass reference's int4 decode hot
 * path (maceip/vibethinker-webgpu-lora).  It is the parity checker for the CUDA
 * library and the timed CPU baseline in bench.py; nothing in the product path
 * links, imports or calls it.  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may load it.
 *
 * The reference path is JavaScript + WGSL and cannot execute here (no node, no
 * WebGPU), so every routine below restates the reference algorithm and cites
 * the file:line it follows (paths relative to the reference project root).
 * Parity of this restatement is pinned by the reference's own known-answer
 * tests (test/topk_argmax_ties.js:114-129, test/gemm_test.js:21-60) which
 * tests/test_oracle_golden.py replays, plus hand-derived quantiser cases.
 *
 * Numerics ("mimic" mode): every reduction is done in float32 in the order the
 * WGSL kernel writes it per thread; cross-thread reduction trees of the
 * WebGPU kernels are replaced by a sequential f32 sum (the only freedom left).
 * Quantiser arithmetic is JS double, exactly as quantize.js runs it.
 * The f16 staging path (setUseF16 / RMSNORM_F16 / ROPE_QK_F16 /
 * ATTN_*_F16) rounds through IEEE binary16 with one rounding per WGSL f16 op.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

/* One rounding of an exactly-representable double to binary16 (RNE). */
static inline float h16(double v) { return (float)(_Float16)v; }

/* ------------------------------------------------------------------------ */
/* Synthetic inputs: SplitMix64 stream in counter form + Box-Muller.         */
/* (Test-input generator; not a reference algorithm.)                        */
/* ------------------------------------------------------------------------ */
static inline uint64_t sm_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
/* k-th output of the SplitMix64 stream whose state starts at `seed`. */
static inline uint64_t sm_at(uint64_t seed, uint64_t k) {
  return sm_mix(seed + (k + 1) * 0x9E3779B97F4A7C15ULL);
}
static inline double u01(uint64_t z) { return (double)(z >> 11) * 0x1.0p-53; }

ORC_API uint64_t orc_stream_at(uint64_t seed, uint64_t k) { return sm_at(seed, k); }

/* out[i] = std * N(0,1) for element index (start + i) of stream `seed`. */
ORC_API void orc_fill_normal(float* out, int64_t n, uint64_t seed, double stdv, int64_t start) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) {
    uint64_t e = (uint64_t)(start + i);
    double a = 1.0 - u01(sm_at(seed, 2 * e));
    double b = u01(sm_at(seed, 2 * e + 1));
    double r = sqrt(-2.0 * log(a));
    double c = cos(6.283185307179586 * b);
    out[i] = (float)(stdv * (r * c));
  }
}
ORC_API void orc_fill_uniform(float* out, int64_t n, uint64_t seed) {
  for (int64_t i = 0; i < n; i++) out[i] = (float)u01(sm_at(seed, (uint64_t)i));
}
ORC_API void orc_fill_ids(uint32_t* out, int64_t n, uint64_t seed, uint32_t vocab) {
  for (int64_t i = 0; i < n; i++) out[i] = (uint32_t)(sm_at(seed, (uint64_t)i) % vocab);
}

/* ------------------------------------------------------------------------ */
/* Quantisers (src/qwgpu/quantize.js)                                        */
/* ------------------------------------------------------------------------ */
/* JS Math.round: nearest integer, halves toward +infinity. */
static inline double js_round(double x) {
  double r = floor(x);
  if (x - r >= 0.5) r += 1.0;
  return r;
}

/* quantizeInt4Group, src/qwgpu/quantize.js:81-111.  amax/scale/inv/w*inv in
 * double; stored scale is the f32 rounding of s while inv uses unrounded s. */
ORC_API int orc_quantize_int4_group(const float* W, int N, int K, int group, uint32_t* packed,
                                    float* scale) {
  if (N < 0 || K <= 0 || group <= 0 || K % group || K % 8) return -1;
  const int gpr = K / group;
#pragma omp parallel for schedule(static)
  for (int o = 0; o < N; o++) {
    int8_t q[8];
    for (int g = 0; g < gpr; g++) {
      const float* src = W + (int64_t)o * K + (int64_t)g * group;
      double amax = 0;
      for (int i = 0; i < group; i++) {
        double a = fabs((double)src[i]);
        if (a > amax) amax = a;
      }
      double s = amax > 0 ? amax / 7 : 1;
      scale[(int64_t)o * gpr + g] = (float)s;
      double inv = 1 / s;
      uint32_t* dst = packed + ((int64_t)o * K + (int64_t)g * group) / 8;
      for (int w = 0; w < group / 8; w++) {
        uint32_t acc = 0;
        for (int j = 0; j < 8; j++) {
          double v = js_round((double)src[w * 8 + j] * inv);
          if (v > 7) v = 7;
          else if (v < -8) v = -8;
          q[j] = (int8_t)v;
          acc |= ((uint32_t)q[j] & 0xFu) << (4 * j); /* quantize.js:107 */
        }
        dst[w] = acc;
      }
    }
  }
  return 0;
}

/* quantizeInt8RowMajor, src/qwgpu/quantize.js:28-57: one scale per row,
 * 4 int8 per u32 little-endian. */
ORC_API int orc_quantize_int8_rows(const float* W, int N, int K, uint32_t* packed, float* scale) {
  if (N < 0 || K <= 0 || K % 4) return -1;
#pragma omp parallel for schedule(static)
  for (int o = 0; o < N; o++) {
    const float* src = W + (int64_t)o * K;
    double amax = 0;
    for (int i = 0; i < K; i++) {
      double a = fabs((double)src[i]);
      if (a > amax) amax = a;
    }
    double s = amax > 0 ? amax / 127 : 1;
    scale[o] = (float)s;
    double inv = 1 / s;
    uint8_t* dst = (uint8_t*)(packed + (int64_t)o * K / 4);
    for (int i = 0; i < K; i++) {
      double v = js_round((double)src[i] * inv);
      if (v > 127) v = 127;
      else if (v < -128) v = -128;
      dst[i] = (uint8_t)(int8_t)v;
    }
  }
  return 0;
}

/* Dequantise int4 (test/q4_accuracy.mjs:27-30): deq = nib * scale, f32. */
ORC_API void orc_dequant_int4(const uint32_t* packed, const float* scale, int N, int K, int group,
                              float* out) {
  const int gpr = K / group;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < N; r++)
    for (int c = 0; c < K; c++) {
      int64_t wi = (int64_t)r * K + c;
      int nib = (packed[wi >> 3] >> ((wi & 7) * 4)) & 0xF;
      if (nib > 7) nib -= 16;
      out[wi] = (float)nib * scale[(int64_t)r * gpr + c / group];
    }
}

static inline float nib_at(uint32_t word, int j) { return (float)((int32_t)(word << (28 - 4 * j)) >> 28); }

/* ------------------------------------------------------------------------ */
/* GEMVs                                                                     */
/* ------------------------------------------------------------------------ */
/* GEMV4 / GEMV4_ADD, src/qwgpu/kernels.js:884-971.  Per word the eight
 * products are summed first, then scaled by the group scale (bk>>7). */
/* Summation order of the reductions (GEMV row words, RMSNorm sum of
 * squares, attention q.k dot and weighted-V sum): 0 = ascending (the order
 * one WGSL thread walks them), 1 = descending.  Both are f32 restatements
 * of the same sums; the second exists to measure how far two valid
 * reduction orders of the reference part -- the numerical noise floor an
 * independent implementation is held to. */
static int g_sum_order = 0;
ORC_API void orc_set_sum_order(int order) { g_sum_order = order; }

static float gemv4_row(const float* x, const uint32_t* w, const float* scale, int n, int K,
                       int gpr) {
  const int K8 = K / 8;
  const uint32_t* rw = w + (int64_t)n * K8;
  const float* rs = scale + (int64_t)n * gpr;
  float acc = 0.0f;
  for (int cc = 0; cc < K8; cc++) {
    const int c = g_sum_order ? K8 - 1 - cc : cc;
    uint32_t word = rw[c];
    int bk = c * 8;
    float sc = rs[bk >> 7];
    float p = 0.0f;
    for (int j = 0; j < 8; j++) p = p + x[bk + j] * nib_at(word, j);
    acc = acc + p * sc;
  }
  return acc;
}

static float lora_delta(const float* d, const float* B, int rank, int N, int n) {
  float dl = 0.0f;
  for (int r = 0; r < rank; r++) dl = dl + d[r] * B[(int64_t)r * N + n];
  return dl;
}

/* y = W4 x (+bias) (+scaleLo * d.B);  add != 0 gives y += (...). */
ORC_API void orc_gemv_q4(const float* x, const uint32_t* w, const float* scale, const float* bias,
                         const float* loraD, const float* loraB, int rank, float scaleLo, int N,
                         int K, int gpr, int add, float* y) {
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; n++) {
    float o = gemv4_row(x, w, scale, n, K, gpr);
    if (bias) o = o + bias[n];
    if (loraB && rank > 0) o = o + scaleLo * lora_delta(loraD, loraB, rank, N, n);
    y[n] = add ? y[n] + o : o;
  }
}

/* GEMV (int8 rows), src/qwgpu/kernels.js:20-59: sum first, scale last. */
ORC_API void orc_gemv_q8(const float* x, const uint32_t* w, const float* scale, const float* bias,
                         int N, int K, float* y) {
  const int K4 = K / 4;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; n++) {
    const int8_t* rw = (const int8_t*)(w + (int64_t)n * K4);
    float acc = 0.0f;
    for (int k = 0; k < K4; k++) {
      const int kk = 4 * k;
      acc = acc + x[kk] * (float)rw[kk] + x[kk + 1] * (float)rw[kk + 1] +
            x[kk + 2] * (float)rw[kk + 2] + x[kk + 3] * (float)rw[kk + 3];
    }
    float o = acc * scale[n];
    if (bias) o = o + bias[n];
    y[n] = o;
  }
}

/* GATE_UP_SILU_GEMV4, src/qwgpu/kernels.js:1021-1072.  Rows n and N+n of the
 * packed [gate;up] matrix (runtime.js:640-651); silu(g)*u.  The gate and up
 * halves are passed as separate row bases so callers need not concatenate. */
static void gate_up_silu2(const float* x, const uint32_t* wg, const float* sg, const uint32_t* wu,
                          const float* su, const float* gD, const float* gB, int gRank,
                          float gScale, const float* uD, const float* uB, int uRank, float uScale,
                          int N, int K, int gpr, float* y) {
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; n++) {
    float g = gemv4_row(x, wg, sg, n, K, gpr);
    float u = gemv4_row(x, wu, su, n, K, gpr);
    if (gB && gRank > 0) g = g + gScale * lora_delta(gD, gB, gRank, N, n);
    if (uB && uRank > 0) u = u + uScale * lora_delta(uD, uB, uRank, N, n);
    y[n] = (g / (1.0f + expf(-g))) * u;
  }
}
ORC_API void orc_gate_up_silu(const float* x, const uint32_t* w, const float* scale,
                              const float* gD, const float* gB, int gRank, float gScale,
                              const float* uD, const float* uB, int uRank, float uScale, int N,
                              int K, int gpr, float* y) {
  gate_up_silu2(x, w, scale, w + (int64_t)N * (K / 8), scale + (int64_t)N * gpr, gD, gB, gRank,
                gScale, uD, uB, uRank, uScale, N, K, gpr, y);
}

/* LORA_A, src/qwgpu/kernels.js:60-78: d[r] = sum_k x[k] A[r][k]. */
ORC_API void orc_lora_a(const float* x, const float* A, int K, int rank, float* d) {
  for (int r = 0; r < rank; r++) {
    float acc = 0.0f;
    for (int k = 0; k < K; k++) acc = acc + x[k] * A[(int64_t)r * K + k];
    d[r] = acc;
  }
}

/* ------------------------------------------------------------------------ */
/* Norm, RoPE, embedding                                                     */
/* ------------------------------------------------------------------------ */
/* RMSNORM (kernels.js:128-144) and RMSNORM_F16 (kernels.js:145-166). */
ORC_API void orc_rmsnorm(const float* x, const float* g, int K, float eps, int f16, float* y) {
  float s = 0.0f;
  for (int kk = 0; kk < K; kk++) {
    const int k = g_sum_order ? K - 1 - kk : kk;
    s = s + x[k] * x[k];
  }
  /* inverseSqrt: WGSL leaves its rounding to the device; restated as an
   * IEEE f32 sqrt followed by an IEEE f32 divide. */
  float inv = 1.0f / sqrtf(s / (float)K + eps);
  if (!f16) {
    for (int k = 0; k < K; k++) y[k] = x[k] * inv * g[k];
  } else {
    float inv16 = h16(inv);
    for (int k = 0; k < K; k++) y[k] = h16((double)h16((double)h16(x[k]) * inv16) * h16(g[k]));
  }
}

/* _buildRope, src/qwgpu/runtime.js:572-590: tables in double, stored f32. */
ORC_API void orc_rope_tables(int max_ctx, int hd, double theta, float* cosT, float* sinT) {
  const int half = hd / 2;
  for (int p = 0; p < max_ctx; p++)
    for (int i = 0; i < half; i++) {
      double a = p / pow(theta, (2.0 * i) / hd);
      double cc = cos(a), ss = sin(a);
      cosT[(int64_t)p * hd + i] = (float)cc;
      cosT[(int64_t)p * hd + half + i] = (float)cc;
      sinT[(int64_t)p * hd + i] = (float)ss;
      sinT[(int64_t)p * hd + half + i] = (float)ss;
    }
}

/* One rotate-half pair, ROPE_QK (kernels.js:205-230) / ROPE_QK_F16 (231-257):
 * two separately rounded products, then one add. */
static void rope_pair(float* lo, float* hi, float c, float s, int f16) {
  float xl = *lo, xh = *hi;
  if (!f16) {
    float a = xl * c, b = (-xh) * s;
    float d = xh * c, e = xl * s;
    *lo = a + b;
    *hi = d + e;
  } else {
    double hc = h16(c), hs = h16(s), hl = h16(xl), hh = h16(xh);
    *lo = h16((double)h16(hl * hc) + (double)h16(-hh * hs));
    *hi = h16((double)h16(hh * hc) + (double)h16(hl * hs));
  }
}
ORC_API void orc_rope_qk(float* q, float* k, int nq, int nkv, int hd, int pos, const float* cosT,
                         const float* sinT, int f16) {
  const int half = hd / 2;
  for (int h = 0; h < nq + nkv; h++) {
    float* x = h < nq ? q + h * hd : k + (h - nq) * hd;
    for (int j = 0; j < half; j++) {
      int64_t off = (int64_t)pos * hd + j;
      rope_pair(&x[j], &x[j + half], cosT[off], sinT[off], f16);
    }
  }
}

/* EMBED / EMBED_BUF, kernels.js:524-550: f32(q8[id][k]) * scale[id]. */
ORC_API void orc_embed(const uint32_t* w, const float* scale, uint32_t id, int H, float* out) {
  const int8_t* row = (const int8_t*)(w + (int64_t)id * (H / 4));
  for (int k = 0; k < H; k++) out[k] = (float)row[k] * scale[id];
}

/* ------------------------------------------------------------------------ */
/* Split-K decode attention                                                  */
/* ------------------------------------------------------------------------ */
/* ATTN_PARTIAL (kernels.js:258-298) + ATTN_COMBINE (346-365), and the f16
 * staging pair ATTN_PARTIAL_F16 (299-345) + ATTN_COMBINE_F16 (366-388).
 * kc/vc: [ctx][nkv*hd] f32.  chunk = runtime CHUNK (runtime.js:330 => 128). */
ORC_API void orc_attention(const float* q, const float* kc, const float* vc, int nh, int nkv,
                           int ctx, int hd, int chunk, int f16, float* out) {
  const int nsplit = (ctx + chunk - 1) / chunk;
  const int stride = nkv * hd;
  const float scale = 1.0f / sqrtf((float)hd);
  float* pm = (float*)malloc(sizeof(float) * nsplit);
  float* pz = (float*)malloc(sizeof(float) * nsplit);
  float* po = (float*)malloc(sizeof(float) * (size_t)nsplit * hd);
  float* sc = (float*)malloc(sizeof(float) * chunk);
  for (int h = 0; h < nh; h++) {
    const int kvh = h / (nh / nkv);
    const float* qh = q + h * hd;
    for (int s = 0; s < nsplit; s++) {
      int t0 = s * chunk, t1 = t0 + chunk;
      if (t1 > ctx) t1 = ctx;
      float M = -1e30f;
      for (int t = t0; t < t1; t++) {
        const float* kr = kc + (int64_t)t * stride + kvh * hd;
        float dot = 0.0f;
        for (int dd = 0; dd < hd; dd++) {
          const int d = g_sum_order ? hd - 1 - dd : dd;
          dot = dot + (f16 ? h16(qh[d]) * h16(kr[d]) : qh[d] * kr[d]);
        }
        sc[t - t0] = dot * scale;
        if (sc[t - t0] > M) M = sc[t - t0];
      }
      float Z = 0.0f;
      for (int t = t0; t < t1; t++) {
        float ev = expf(sc[t - t0] - M);
        sc[t - t0] = ev;
        Z = Z + ev;
      }
      for (int d = 0; d < hd; d++) {
        float acc = 0.0f;
        for (int tt = t0; tt < t1; tt++) {
          const int t = g_sum_order ? t0 + t1 - 1 - tt : tt;
          float v = vc[(int64_t)t * stride + kvh * hd + d];
          acc = acc + sc[t - t0] * (f16 ? h16(v) : v);
        }
        po[(int64_t)s * hd + d] = acc;
      }
      pm[s] = M;
      pz[s] = Z;
    }
    float M = -1e30f;
    for (int s = 0; s < nsplit; s++) M = fmaxf(M, pm[s]);
    float Z = 0.0f;
    for (int s = 0; s < nsplit; s++) Z = Z + pz[s] * expf(pm[s] - M);
    float invZ = 1.0f / Z;
    for (int d = 0; d < hd; d++) {
      float acc = 0.0f;
      for (int s = 0; s < nsplit; s++) {
        float p = po[(int64_t)s * hd + d];
        acc = acc + expf(pm[s] - M) * (f16 ? h16(p) : p);
      }
      out[h * hd + d] = acc * invZ;
    }
  }
  free(pm);
  free(pz);
  free(po);
  free(sc);
}

/* ------------------------------------------------------------------------ */
/* Whole-prompt prefill (prefillBatch)                                       */
/* ------------------------------------------------------------------------ */
/* GEMM4 / GEMM4_ADD_T, kernels.js:389-473: per word the eight weights are
 * dequantised first (f32(nibble) * scale), the eight products summed left to
 * right, the sum added to the running accumulator. */
static float gemm4_row(const float* x, const uint32_t* w, const float* scale, int n, int K, int gpr) {
  const int K8 = K / 8;
  const uint32_t* rw = w + (int64_t)n * K8;
  const float* rs = scale + (int64_t)n * gpr;
  float acc = 0.0f;
  for (int cc = 0; cc < K8; cc++) {
    const int c = g_sum_order ? K8 - 1 - cc : cc;
    const uint32_t word = rw[c];
    const float sc = rs[(c * 8) >> 7];
    const float* a = x + c * 8;
    float p = a[0] * (nib_at(word, 0) * sc);
    for (int j = 1; j < 8; j++) p = p + a[j] * (nib_at(word, j) * sc);
    acc = acc + p;
  }
  return acc;
}

/* Y[t] = W4 X[t] + bias (GEMM4) or Y[t] = Y[t] + W4 X[t] + bias (GEMM4_ADD_T). */
ORC_API void orc_gemm4(const float* X, int T, const uint32_t* w, const float* scale, const float* bias, int N,
                       int K, int add, float* Y) {
  const int gpr = K / 128;
#pragma omp parallel for collapse(2) schedule(static)
  for (int t = 0; t < T; t++)
    for (int n = 0; n < N; n++) {
      const float acc = gemm4_row(X + (int64_t)t * K, w, scale, n, K, gpr);
      const float bv = bias ? bias[n] : 0.0f;
      float* y = Y + (int64_t)t * N + n;
      *y = add ? (*y + acc) + bv : acc + bv;
    }
}

/* loraBatchDelta (runtime.js:1814-1843): LORA_A_BATCH (kernels.js:79-97)
 * d[t][r] = sum_k X[t][k] A[r][k], then LORA_B_ADD_T (kernels.js:98-112)
 * Y[t][n] += scale * sum_r d[t][r] B[r][n]. */
ORC_API void orc_lora_batch_delta(const float* X, int T, const float* A, const float* B, int rank, float scale,
                                  int K, int N, float* Y) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; t++) {
    float d[256];
    for (int r = 0; r < rank; r++) {
      float acc = 0.0f;
      for (int k = 0; k < K; k++) acc = acc + X[(int64_t)t * K + k] * A[(int64_t)r * K + k];
      d[r] = acc;
    }
    for (int n = 0; n < N; n++) {
      float acc = 0.0f;
      for (int r = 0; r < rank; r++) acc = acc + d[r] * B[(int64_t)r * N + n];
      Y[(int64_t)t * N + n] = Y[(int64_t)t * N + n] + scale * acc;
    }
  }
}

/* SILUMUL / SILUMUL_F16, kernels.js:499-523: silu in f32; the f16 variant
 * rounds silu(g) and u to f16 and multiplies in f16. */
ORC_API void orc_silu_mul(float* gate, const float* up, int64_t n, int f16) {
  for (int64_t i = 0; i < n; i++) {
    const float v = gate[i];
    const float sg = v / (1.0f + expf(-v));
    gate[i] = f16 ? h16((double)h16(sg) * (double)h16(up[i])) : sg * up[i];
  }
}

/* ROPE_T / ROPE_T_F16, kernels.js:588-618: rows t of x (nh heads) at
 * position pos0 + t, the decode pair rotation. */
ORC_API void orc_rope_t(float* x, int T, int nh, int hd, int pos0, const float* cosT, const float* sinT,
                        int f16) {
  const int half = hd / 2;
  for (int t = 0; t < T; t++)
    for (int h = 0; h < nh; h++) {
      float* r = x + ((int64_t)t * nh + h) * hd;
      for (int j = 0; j < half; j++) {
        const int64_t off = (int64_t)(pos0 + t) * hd + j;
        rope_pair(&r[j], &r[j + half], cosT[off], sinT[off], f16);
      }
    }
}

/* ATTN_PREFILL_BLOCK, kernels.js:684-770: query row t (absolute position
 * qStart + t) over keys 0..ctx-1 in blocks of 128 with an online softmax:
 * per block the running max moves to max(m, block max), the running sum
 * and the accumulator are rescaled by exp(m_old - m_new), then the block's
 * exp(s - m_new) weights are added; keys past the query are masked.
 * q [T][nh*hd], kc / vc [ctx][nkv*hd], out [T][nh*hd]. */
ORC_API void orc_attn_prefill(const float* q, const float* kc, const float* vc, int nh, int nkv, int hd, int T,
                              int qStart, int ctx, float* out) {
  const int stride = nkv * hd, BK = 128;
  const float scl = 1.0f / sqrtf((float)hd);
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int t = 0; t < T; t++)
    for (int h = 0; h < nh; h++) {
      const int kvh = h / (nh / nkv), absQ = qStart + t;
      const float* qr = q + ((int64_t)t * nh + h) * hd;
      float acc[256], p[128];
      for (int d = 0; d < hd; d++) acc[d] = 0.0f;
      float mrun = -1e30f, lrun = 0.0f;
      for (int kb = 0; kb < ctx; kb += BK) {
        float bm = -1e30f;
        for (int j = 0; j < BK; j++) {
          const int kk = kb + j;
          p[j] = -1e30f;
          if (kk < ctx && kk <= absQ) {
            const float* kr = kc + (int64_t)kk * stride + kvh * hd;
            float dot = 0.0f;
            for (int dd = 0; dd < hd; dd++) {
              const int d = g_sum_order ? hd - 1 - dd : dd;
              dot = dot + qr[d] * kr[d];
            }
            p[j] = dot * scl;
          }
          bm = fmaxf(bm, p[j]);
        }
        const float mnew = fmaxf(mrun, bm), corr = expf(mrun - mnew);
        float bs = 0.0f;
        for (int j = 0; j < BK; j++) {
          const int kk = kb + j;
          p[j] = (kk < ctx && kk <= absQ) ? expf(p[j] - mnew) : 0.0f;
          bs = bs + p[j];
        }
        lrun = lrun * corr + bs;
        mrun = mnew;
        const int bcount = ctx - kb < BK ? ctx - kb : BK;
        for (int d = 0; d < hd; d++) {
          float a = acc[d] * corr;
          for (int jj = 0; jj < bcount; jj++) {
            const int j = g_sum_order ? bcount - 1 - jj : jj;
            a = a + p[j] * vc[(int64_t)(kb + j) * stride + kvh * hd + d];
          }
          acc[d] = a;
        }
      }
      const float invL = 1.0f / lrun;
      for (int d = 0; d < hd; d++) out[((int64_t)t * nh + h) * hd + d] = acc[d] * invL;
    }
}

/* ------------------------------------------------------------------------ */
/* Sampling                                                                  */
/* ------------------------------------------------------------------------ */
static inline int beats(float x, uint32_t i, float v, uint32_t idx) {
  return x > v || (x == v && i < idx);
}
/* ARGMAX, kernels.js:771-784: max, ties to the lowest index, NaN never wins. */
ORC_API uint32_t orc_argmax(const float* logits, int n) {
  float v = -1e30f;
  uint32_t idx = 0xFFFFFFFFu;
  for (int i = 0; i < n; i++)
    if (beats(logits[i], (uint32_t)i, v, idx)) {
      v = logits[i];
      idx = (uint32_t)i;
    }
  return idx;
}

/* TOPK_SELECT, kernels.js:785-813 (driven k times, runtime.js:1648-1678). */
ORC_API void orc_topk(const float* logits, int n, int k, uint32_t* ids, float* vals) {
  for (int sel = 0; sel < k; sel++) {
    float v = -1e30f;
    uint32_t idx = 0xFFFFFFFFu;
    for (int i = 0; i < n; i++) {
      int taken = 0;
      for (int j = 0; j < sel; j++)
        if (ids[j] == (uint32_t)i) {
          taken = 1;
          break;
        }
      if (!taken && beats(logits[i], (uint32_t)i, v, idx)) {
        v = logits[i];
        idx = (uint32_t)i;
      }
    }
    ids[sel] = idx;
    vals[sel] = v;
  }
}

/* SAMPLE_TOPK, kernels.js:814-883: exp without max subtraction, 64-slot
 * pairwise tree sum, Hillis-Steele inclusive prefix, first j with r <= P_j. */
ORC_API uint32_t orc_sample_topk(const uint32_t* ids, const float* vals, int k, float temp,
                                 float r) {
  float s[64], red[64];
  const float t = temp <= 0.0f ? 1.0f : temp;
  for (int tid = 0; tid < 64; tid++) {
    float v = -1e30f;
    if (tid < k) {
      v = vals[tid];
      if (t != 1.0f) v = vals[tid] / t;
    }
    float ev = tid < k ? expf(v) : 0.0f;
    s[tid] = ev;
    red[tid] = ev;
  }
  for (int stride = 32; stride > 0; stride /= 2)
    for (int tid = 0; tid < stride; tid++) red[tid] = red[tid] + red[tid + stride];
  const float sum = red[0];
  const float invSum = sum > 0.0f ? 1.0f / sum : 0.0f;
  for (int tid = 0; tid < 64; tid++) s[tid] = tid < k ? s[tid] * invSum : 0.0f;
  for (int stride = 1; stride < 64; stride *= 2) {
    float add[64];
    for (int tid = 0; tid < 64; tid++) add[tid] = tid >= stride ? s[tid - stride] : 0.0f;
    for (int tid = stride; tid < 64; tid++) s[tid] = s[tid] + add[tid];
  }
  uint32_t chosen = k > 0 ? (uint32_t)(k - 1) : 0u;
  if (sum > 0.0f)
    for (int j = 0; j < k; j++)
      if (r <= s[j]) {
        chosen = (uint32_t)j;
        break;
      }
  return k > 0 ? ids[chosen] : 0u;
}

/* ------------------------------------------------------------------------ */
/* Whole-model decode step (src/qwgpu/runtime.js:1466-1571, default flags:    */
/* unfused q/k/v GEMV4 + ROPE_QK, fused gate_up+SiLU, fused residual).       */
/* ------------------------------------------------------------------------ */
typedef struct {
  int hidden, layers, heads, kv_heads, head_dim, inter, vocab;
  float eps;
  double theta;
} orc_cfg;

typedef struct {
  float *A, *B; /* A [r][in], B [r][out] (src/lora_gpu.js:96-107) */
  int rank;
  float scale;
} orc_lora_mod;

typedef struct {
  orc_cfg c;
  int max_ctx, f16, chunk;
  /* int8 tied embedding / LM head */
  uint32_t* emb_w;
  float* emb_s;
  float* final_norm;
  /* per layer: 7 int4 projections (q,k,v,o,gate,up,down) */
  uint32_t** w[7];
  float** s[7];
  float** bias[3];
  float** in_norm;
  float** post_norm;
  float *kc, *vc; /* [layers][max_ctx][kvd] */
  float *cosT, *sinT;
  orc_lora_mod* lora; /* [layers*7] or NULL */
  /* scratch */
  float *hidden, *normed, *q, *k, *v, *attn, *tmp, *logits, *d1, *d2;
} orc_model;

static void proj_dims(const orc_cfg* c, int p, int* N, int* K) {
  const int H = c->hidden, QD = c->heads * c->head_dim, KVD = c->kv_heads * c->head_dim,
            I = c->inter;
  switch (p) {
    case 0: *N = QD; *K = H; break;
    case 1: *N = KVD; *K = H; break;
    case 2: *N = KVD; *K = H; break;
    case 3: *N = H; *K = QD; break;
    case 4: *N = I; *K = H; break;
    case 5: *N = I; *K = H; break;
    default: *N = H; *K = I; break;
  }
}

/* Synthetic-model tensor ids: embed 0; layer i projection p (0..6) at
 * 16i+1+p; q/k/v biases at 16i+8+{0,1,2}.  seed_t = stream(base)[t]. */
ORC_API uint64_t orc_tensor_seed(uint64_t base, int tensor_id) { return sm_at(base, (uint64_t)tensor_id); }

static void* xmalloc(size_t n) {
  void* p = malloc(n ? n : 1);
  return p;
}

ORC_API void orc_model_free(void* mp);

/* Build the synthetic model: all matrices and q/k/v biases N(0, std_w),
 * norms 1, int4 g128 projections, int8-row tied embedding. */
ORC_API void* orc_model_create(const orc_cfg* cfg, int max_ctx, int f16, uint64_t seed,
                               double std_w) {
  orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
  if (!m) return NULL;
  m->c = *cfg;
  m->max_ctx = max_ctx;
  m->f16 = f16;
  m->chunk = 128;
  const orc_cfg* c = cfg;
  const int H = c->hidden, L = c->layers, hd = c->head_dim;
  const int KVD = c->kv_heads * hd, QD = c->heads * hd;
  /* embedding, generated in row chunks (quantisation is per row) */
  m->emb_w = (uint32_t*)xmalloc((size_t)c->vocab * H);
  m->emb_s = (float*)xmalloc(sizeof(float) * c->vocab);
  {
    const int rows = 4096;
    float* tmp = (float*)xmalloc(sizeof(float) * (size_t)rows * H);
    uint64_t sd = orc_tensor_seed(seed, 0);
    for (int r0 = 0; r0 < c->vocab; r0 += rows) {
      int nr = c->vocab - r0 < rows ? c->vocab - r0 : rows;
      orc_fill_normal(tmp, (int64_t)nr * H, sd, std_w, (int64_t)r0 * H);
      orc_quantize_int8_rows(tmp, nr, H, m->emb_w + (size_t)r0 * H / 4, m->emb_s + r0);
    }
    free(tmp);
  }
  m->final_norm = (float*)xmalloc(sizeof(float) * H);
  for (int i = 0; i < H; i++) m->final_norm[i] = 1.0f;
  for (int p = 0; p < 7; p++) {
    m->w[p] = (uint32_t**)calloc(L, sizeof(void*));
    m->s[p] = (float**)calloc(L, sizeof(void*));
  }
  for (int b = 0; b < 3; b++) m->bias[b] = (float**)calloc(L, sizeof(void*));
  m->in_norm = (float**)calloc(L, sizeof(void*));
  m->post_norm = (float**)calloc(L, sizeof(void*));
  size_t maxel = 0;
  for (int p = 0; p < 7; p++) {
    int N, K;
    proj_dims(c, p, &N, &K);
    if ((size_t)N * K > maxel) maxel = (size_t)N * K;
  }
  float* tmp = (float*)xmalloc(sizeof(float) * maxel);
  for (int i = 0; i < L; i++) {
    for (int p = 0; p < 7; p++) {
      int N, K;
      proj_dims(c, p, &N, &K);
      m->w[p][i] = (uint32_t*)xmalloc((size_t)N * K / 2);
      m->s[p][i] = (float*)xmalloc(sizeof(float) * (size_t)N * (K / 128));
      orc_fill_normal(tmp, (int64_t)N * K, orc_tensor_seed(seed, 16 * i + 1 + p), std_w, 0);
      orc_quantize_int4_group(tmp, N, K, 128, m->w[p][i], m->s[p][i]);
    }
    for (int b = 0; b < 3; b++) {
      int N = b == 0 ? QD : KVD;
      m->bias[b][i] = (float*)xmalloc(sizeof(float) * N);
      orc_fill_normal(m->bias[b][i], N, orc_tensor_seed(seed, 16 * i + 8 + b), std_w, 0);
    }
    m->in_norm[i] = (float*)xmalloc(sizeof(float) * H);
    m->post_norm[i] = (float*)xmalloc(sizeof(float) * H);
    for (int k = 0; k < H; k++) m->in_norm[i][k] = m->post_norm[i][k] = 1.0f;
  }
  free(tmp);
  m->kc = (float*)calloc((size_t)L * max_ctx * KVD, sizeof(float));
  m->vc = (float*)calloc((size_t)L * max_ctx * KVD, sizeof(float));
  m->cosT = (float*)xmalloc(sizeof(float) * (size_t)max_ctx * hd);
  m->sinT = (float*)xmalloc(sizeof(float) * (size_t)max_ctx * hd);
  orc_rope_tables(max_ctx, hd, c->theta, m->cosT, m->sinT);
  const int I = c->inter;
  m->hidden = (float*)xmalloc(sizeof(float) * H);
  m->normed = (float*)xmalloc(sizeof(float) * H);
  m->q = (float*)xmalloc(sizeof(float) * QD);
  m->k = (float*)xmalloc(sizeof(float) * KVD);
  m->v = (float*)xmalloc(sizeof(float) * KVD);
  m->attn = (float*)xmalloc(sizeof(float) * QD);
  m->tmp = (float*)xmalloc(sizeof(float) * I);
  m->logits = (float*)xmalloc(sizeof(float) * c->vocab);
  m->d1 = (float*)xmalloc(sizeof(float) * 256);
  m->d2 = (float*)xmalloc(sizeof(float) * 256);
  return m;
}

ORC_API void orc_model_set_chunk(void* mp, int chunk) { ((orc_model*)mp)->chunk = chunk; }

/* Pointer to a quantised tensor for cross-checks: which = 0..6 projection
 * words, 7..13 projection scales, 14 embed words, 15 embed scales,
 * 16..18 q/k/v bias. */
ORC_API const void* orc_model_tensor(void* mp, int layer, int which) {
  orc_model* m = (orc_model*)mp;
  if (which < 7) return m->w[which][layer];
  if (which < 14) return m->s[which - 7][layer];
  if (which == 14) return m->emb_w;
  if (which == 15) return m->emb_s;
  return m->bias[which - 16][layer];
}

static void free_lora(orc_model* m) {
  if (!m->lora) return;
  for (int i = 0; i < m->c.layers * 7; i++) {
    free(m->lora[i].A);
    free(m->lora[i].B);
  }
  free(m->lora);
  m->lora = NULL;
}

/* Synthetic adapter on all 7 projections of every layer (module index
 * 7i+p): A ~ N(0, stdA) [rank][in], B ~ N(0, stdB) [rank][out]; module
 * streams 2(7i+p) and 2(7i+p)+1 of `seed`.  scale as lora_gpu.js:100-108. */
ORC_API void orc_model_lora_synth(void* mp, uint64_t seed, int rank, float scale, double stdA,
                                  double stdB) {
  orc_model* m = (orc_model*)mp;
  free_lora(m);
  const int L = m->c.layers;
  m->lora = (orc_lora_mod*)calloc((size_t)L * 7, sizeof(orc_lora_mod));
  for (int i = 0; i < L; i++)
    for (int p = 0; p < 7; p++) {
      int N, K;
      proj_dims(&m->c, p, &N, &K);
      orc_lora_mod* md = &m->lora[7 * i + p];
      md->rank = rank;
      md->scale = scale;
      md->A = (float*)xmalloc(sizeof(float) * (size_t)rank * K);
      md->B = (float*)xmalloc(sizeof(float) * (size_t)rank * N);
      orc_fill_normal(md->A, (int64_t)rank * K, sm_at(seed, 2 * (uint64_t)(7 * i + p)), stdA, 0);
      orc_fill_normal(md->B, (int64_t)rank * N, sm_at(seed, 2 * (uint64_t)(7 * i + p) + 1), stdB, 0);
    }
}
ORC_API void orc_model_lora_clear(void* mp) { free_lora((orc_model*)mp); }

static orc_lora_mod* lmod(orc_model* m, int i, int p) { return m->lora ? &m->lora[7 * i + p] : NULL; }

static void proj(orc_model* m, int i, int p, const float* x, const float* bias, int add,
                 float* y) {
  int N, K;
  proj_dims(&m->c, p, &N, &K);
  orc_lora_mod* md = lmod(m, i, p);
  if (md) orc_lora_a(x, md->A, K, md->rank, m->d1);
  orc_gemv_q4(x, m->w[p][i], m->s[p][i], bias, m->d1, md ? md->B : NULL, md ? md->rank : 0,
              md ? md->scale : 0.0f, N, K, K / 128, add, y);
}

/* embed(id) then step(pos): token() at runtime.js:1735-1741 -> step()
 * runtime.js:1466-1571.  Writes logits (vocab floats) if non-NULL. */
ORC_API int orc_model_step(void* mp, uint32_t id, int pos, float* logits_out) {
  orc_model* m = (orc_model*)mp;
  const orc_cfg* c = &m->c;
  if (pos < 0 || pos >= m->max_ctx || id >= (uint32_t)c->vocab) return -1;
  const int H = c->hidden, hd = c->head_dim, KVD = c->kv_heads * hd, I = c->inter;
  orc_embed(m->emb_w, m->emb_s, id, H, m->hidden);
  for (int i = 0; i < c->layers; i++) {
    orc_rmsnorm(m->hidden, m->in_norm[i], H, c->eps, m->f16, m->normed);
    proj(m, i, 0, m->normed, m->bias[0][i], 0, m->q);
    proj(m, i, 1, m->normed, m->bias[1][i], 0, m->k);
    proj(m, i, 2, m->normed, m->bias[2][i], 0, m->v);
    orc_rope_qk(m->q, m->k, c->heads, c->kv_heads, hd, pos, m->cosT, m->sinT, m->f16);
    float* kc = m->kc + (size_t)i * m->max_ctx * KVD;
    float* vc = m->vc + (size_t)i * m->max_ctx * KVD;
    memcpy(kc + (size_t)pos * KVD, m->k, sizeof(float) * KVD); /* runtime.js:1512-1513 */
    memcpy(vc + (size_t)pos * KVD, m->v, sizeof(float) * KVD);
    orc_attention(m->q, kc, vc, c->heads, c->kv_heads, pos + 1, hd, m->chunk, m->f16, m->attn);
    proj(m, i, 3, m->attn, NULL, 1, m->hidden);
    orc_rmsnorm(m->hidden, m->post_norm[i], H, c->eps, m->f16, m->normed);
    {
      orc_lora_mod* g = lmod(m, i, 4);
      orc_lora_mod* u = lmod(m, i, 5);
      if (g) orc_lora_a(m->normed, g->A, H, g->rank, m->d1);
      if (u) orc_lora_a(m->normed, u->A, H, u->rank, m->d2);
      /* packed [gate;up] = gate rows then up rows (runtime.js:640-651) */
      gate_up_silu2(m->normed, m->w[4][i], m->s[4][i], m->w[5][i], m->s[5][i], m->d1,
                    g ? g->B : NULL, g ? g->rank : 0, g ? g->scale : 0.0f, m->d2,
                    u ? u->B : NULL, u ? u->rank : 0, u ? u->scale : 0.0f, I, H, H / 128, m->tmp);
    }
    proj(m, i, 6, m->tmp, NULL, 1, m->hidden);
  }
  orc_rmsnorm(m->hidden, m->final_norm, H, c->eps, m->f16, m->normed);
  orc_gemv_q8(m->normed, m->emb_w, m->emb_s, NULL, c->vocab, H, m->logits);
  if (logits_out) memcpy(logits_out, m->logits, sizeof(float) * c->vocab);
  return 0;
}

/* One projection of a prefill pass: GEMM4(_ADD_T) then the adapter's batch
 * delta (gemm4 / gemm4AddT, runtime.js:1800-1813). */
static void proj_t(orc_model* m, int i, int p, const float* X, int T, const float* bias, int add, float* Y) {
  int N, K;
  proj_dims(&m->c, p, &N, &K);
  orc_gemm4(X, T, m->w[p][i], m->s[p][i], bias, N, K, add, Y);
  orc_lora_mod* md = lmod(m, i, p);
  if (md) orc_lora_batch_delta(X, T, md->A, md->B, md->rank, md->scale, K, N, Y);
}

/* prefillBatch(ids), runtime.js:1936-2087: chunk <= 0 or T <= chunk runs
 * _prefillFull (one pass over the whole prompt), else _prefillChunked
 * (passes of `chunk` positions, each attending to every earlier row).  Per
 * pass and layer: RMSNORM_T, GEMM4 q/k/v (+bias, +LoRA), ROPE_T, the K/V rows
 * into the cache, ATTN_PREFILL_BLOCK, GEMM4_ADD_T o, RMSNORM_T, GEMM4
 * gate/up, SILUMUL, GEMM4_ADD_T down.  Then the last row's final norm and
 * LM-head GEMV.  Leaves the cache filled to T - 1 and hidden = the last row. */
ORC_API int orc_model_prefill(void* mp, const uint32_t* ids, int T, int chunk, float* logits_out) {
  orc_model* m = (orc_model*)mp;
  const orc_cfg* c = &m->c;
  if (T <= 0 || T > m->max_ctx) return -1;
  for (int t = 0; t < T; t++)
    if (ids[t] >= (uint32_t)c->vocab) return -1;
  const int H = c->hidden, hd = c->head_dim, QD = c->heads * hd, KVD = c->kv_heads * hd, I = c->inter;
  const int CT = (chunk > 0 && T > chunk) ? chunk : T;
  float* hid = (float*)xmalloc(sizeof(float) * (size_t)CT * H);
  float* nrm = (float*)xmalloc(sizeof(float) * (size_t)CT * H);
  float* q = (float*)xmalloc(sizeof(float) * (size_t)CT * QD);
  float* k = (float*)xmalloc(sizeof(float) * (size_t)CT * KVD);
  float* v = (float*)xmalloc(sizeof(float) * (size_t)CT * KVD);
  float* at = (float*)xmalloc(sizeof(float) * (size_t)CT * QD);
  float* g = (float*)xmalloc(sizeof(float) * (size_t)CT * I);
  float* u = (float*)xmalloc(sizeof(float) * (size_t)CT * I);
  for (int off = 0; off < T; off += CT) {
    const int n = T - off < CT ? T - off : CT, end = off + n;
    for (int t = 0; t < n; t++) orc_embed(m->emb_w, m->emb_s, ids[off + t], H, hid + (size_t)t * H);
    for (int i = 0; i < c->layers; i++) {
      for (int t = 0; t < n; t++)
        orc_rmsnorm(hid + (size_t)t * H, m->in_norm[i], H, c->eps, m->f16, nrm + (size_t)t * H);
      proj_t(m, i, 0, nrm, n, m->bias[0][i], 0, q);
      proj_t(m, i, 1, nrm, n, m->bias[1][i], 0, k);
      proj_t(m, i, 2, nrm, n, m->bias[2][i], 0, v);
      orc_rope_t(q, n, c->heads, hd, off, m->cosT, m->sinT, m->f16);
      orc_rope_t(k, n, c->kv_heads, hd, off, m->cosT, m->sinT, m->f16);
      float* kc = m->kc + (size_t)i * m->max_ctx * KVD;
      float* vc = m->vc + (size_t)i * m->max_ctx * KVD;
      memcpy(kc + (size_t)off * KVD, k, sizeof(float) * (size_t)n * KVD);
      memcpy(vc + (size_t)off * KVD, v, sizeof(float) * (size_t)n * KVD);
      orc_attn_prefill(q, kc, vc, c->heads, c->kv_heads, hd, n, off, end, at);
      proj_t(m, i, 3, at, n, NULL, 1, hid);
      for (int t = 0; t < n; t++)
        orc_rmsnorm(hid + (size_t)t * H, m->post_norm[i], H, c->eps, m->f16, nrm + (size_t)t * H);
      proj_t(m, i, 4, nrm, n, NULL, 0, g);
      proj_t(m, i, 5, nrm, n, NULL, 0, u);
      orc_silu_mul(g, u, (int64_t)n * I, m->f16);
      proj_t(m, i, 6, g, n, NULL, 1, hid);
    }
    if (end == T) memcpy(m->hidden, hid + (size_t)(n - 1) * H, sizeof(float) * H);
  }
  orc_rmsnorm(m->hidden, m->final_norm, H, c->eps, m->f16, m->normed);
  orc_gemv_q8(m->normed, m->emb_w, m->emb_s, NULL, c->vocab, H, m->logits);
  if (logits_out) memcpy(logits_out, m->logits, sizeof(float) * c->vocab);
  free(hid);
  free(nrm);
  free(q);
  free(k);
  free(v);
  free(at);
  free(g);
  free(u);
  return 0;
}

ORC_API const float* orc_model_hidden(void* mp) { return ((orc_model*)mp)->hidden; }
ORC_API const float* orc_model_logits(void* mp) { return ((orc_model*)mp)->logits; }

/* Greedy continuation: prompt tokens are stepped one at a time (the decode
 * semantics prefillBatch reproduces), then n_gen argmax tokens are chained
 * as decodeBatch does (runtime.js:1776-1793). margins[i] = top1 - top2 logit
 * at each generated step (NULL to skip). */
ORC_API int orc_model_generate(void* mp, const uint32_t* prompt, int n_prompt, int n_gen,
                               uint32_t* out_ids, float* margins) {
  orc_model* m = (orc_model*)mp;
  if (n_prompt <= 0 || n_prompt + n_gen > m->max_ctx) return -1;
  for (int t = 0; t < n_prompt; t++) orc_model_step(m, prompt[t], t, NULL);
  int pos = n_prompt;
  for (int g = 0; g < n_gen; g++) {
    uint32_t ids[2];
    float vals[2];
    orc_topk(m->logits, m->c.vocab, 2, ids, vals);
    out_ids[g] = orc_argmax(m->logits, m->c.vocab);
    if (margins) margins[g] = vals[0] - vals[1];
    if (g + 1 < n_gen) orc_model_step(m, out_ids[g], pos++, NULL);
  }
  return 0;
}

ORC_API void orc_model_free(void* mp) {
  orc_model* m = (orc_model*)mp;
  if (!m) return;
  free_lora(m);
  for (int p = 0; p < 7; p++) {
    for (int i = 0; i < m->c.layers; i++) {
      free(m->w[p][i]);
      free(m->s[p][i]);
    }
    free(m->w[p]);
    free(m->s[p]);
  }
  for (int b = 0; b < 3; b++) {
    for (int i = 0; i < m->c.layers; i++) free(m->bias[b][i]);
    free(m->bias[b]);
  }
  for (int i = 0; i < m->c.layers; i++) {
    free(m->in_norm[i]);
    free(m->post_norm[i]);
  }
  free(m->in_norm);
  free(m->post_norm);
  free(m->emb_w);
  free(m->emb_s);
  free(m->final_norm);
  free(m->kc);
  free(m->vc);
  free(m->cosT);
  free(m->sinT);
  free(m->hidden);
  free(m->normed);
  free(m->q);
  free(m->k);
  free(m->v);
  free(m->attn);
  free(m->tmp);
  free(m->logits);
  free(m->d1);
  free(m->d2);
  free(m);
}

ORC_API int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
