// eg_kernels.cu -- sm_100a kernels for the Emberglass batch-1 decode path.
//
// GEMVs: the weights stay in the reference's packed layouts (int4 group-128,
// f32 group scales, quantize.js:81-111; int8 rows, quantize.js:28-57).  Each
// warp streams 16-row tiles with 128-bit loads, turns nibbles/bytes into
// exact f16 integers with one LOP3 + one HSUB2 per pair, and uses the
// m16n8k16 tensor-core op as a dot-product engine: the activation vector is
// split into f16 (hi, lo) columns so the result keeps ~f32 accuracy.  The
// per-group scale is applied to each 128-wide group sum (the reference
// applies it per 8-wide word: same value up to f32 rounding).
//
// Attention: split-K decode over the KV cache (ATTN_PARTIAL/ATTN_COMBINE,
// kernels.js:258-388) with RoPE (ROPE_QK, kernels.js:205-257) and the KV
// append (runtime.js:1509-1514) fused into the partial kernel.
#include <float.h>
#include <math.h>

#include <algorithm>

#include "eg_common.cuh"
#include "eg_kernels.h"

namespace eg {

static int g_sm_count = 0;
int sm_count() {
  if (!g_sm_count) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (g_sm_count <= 0) g_sm_count = 148;
  }
  return g_sm_count;
}

template <typename Kern, typename... Args>
static void launch(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, k, args...);
}

// ======================================================================
// Block reductions
// ======================================================================
__device__ float block_sum(float v, float* sbuf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sbuf[warp] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < nw; i++) r += sbuf[i];  // fixed order: deterministic
  return r;
}
__device__ float block_max(float v, float* sbuf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) sbuf[warp] = v;
  __syncthreads();
  float r = sbuf[0];
  for (int i = 1; i < nw; i++) r = fmaxf(r, sbuf[i]);
  return r;
}

// ======================================================================
// GEMV prologue: resolve the input vector (plain / RMSNorm / embed+RMSNorm)
// ======================================================================
struct XCtx {
  int mode, f16;
  const float* x;
  const float* g;
  const int8_t* erow;
  float escale, inv;
  __half inv16;
};

__device__ __forceinline__ float raw_at(const XCtx& c, int k) {
  return c.mode == X_EMBED_RMS ? (float)c.erow[k] * c.escale : c.x[k];
}
// RMSNORM: y = x*inv*g (kernels.js:143); RMSNORM_F16: f16(f16(x)*inv)*f16(g)
// (kernels.js:165) with inv rounded to f16.
__device__ __forceinline__ float xval(const XCtx& c, int k) {
  const float r = raw_at(c, k);
  if (c.mode == X_PLAIN) return r;
  if (!c.f16) return __fmul_rn(__fmul_rn(r, c.inv), c.g[k]);
  __half t = __hmul_rn(__float2half_rn(r), c.inv16);
  t = __hmul_rn(t, __float2half_rn(c.g[k]));
  return __half2float(t);
}

__device__ void setup_x(const XSrc& s, int K, XCtx& c, float* sred) {
  c.mode = s.mode;
  c.f16 = s.f16;
  c.x = s.x;
  c.g = s.norm_g;
  c.erow = nullptr;
  c.escale = 0.f;
  c.inv = 1.f;
  c.inv16 = __float2half_rn(1.f);
  if (s.mode == X_EMBED_RMS) {
    const uint32_t id = s.ids[*s.pos];
    c.erow = reinterpret_cast<const int8_t*>(s.emb_w + (size_t)id * (K / 4));
    c.escale = s.emb_s[id];
    if (blockIdx.x == 0 && s.hidden_out)
      for (int k = threadIdx.x; k < K; k += blockDim.x) s.hidden_out[k] = raw_at(c, k);
  }
  if (s.mode != X_PLAIN) {
    float ss = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const float v = raw_at(c, k);
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
    ss = block_sum(ss, sred);
    c.inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), s.eps)));
    c.inv16 = __float2half_rn(c.inv);
  }
}

// Power-of-two shift keeping |x| * 2^-e inside the f16 range.
__device__ __forceinline__ int shift_for(float amax) {
  if (!(amax > 16384.f)) return 0;
  int e;
  frexpf(amax / 16384.f, &e);
  return e;
}

// Register-staged prologue.  Thread i owns the 8-element units
// u = i, i + blockDim, ... (k = 8u..8u+7); every global load of the input
// (and of the norm weight) is issued before any is consumed, so the whole
// prologue costs one memory latency.  The values are then transformed
// (RMSNorm), range-checked and written once as MMA B fragments:
//   fmt 4: int4 layout (see write_int4_word), fmt 8: int8 layout.
template <int MAXU>
__device__ int stage_x(const XSrc& s, int K, int fmt, void* smem, float* sred) {
  const int K8 = K / 8;
  float v[MAXU][8];
  float gw[MAXU][8];
  const int8_t* erow = nullptr;
  float escale = 0.f;
  if (s.mode == X_EMBED_RMS) {
    const uint32_t id = s.ids[*s.pos];
    erow = reinterpret_cast<const int8_t*>(s.emb_w + (size_t)id * (K / 4));
    escale = s.emb_s[id];
  }
#pragma unroll
  for (int i = 0; i < MAXU; i++) {
    const int u = threadIdx.x + i * blockDim.x;
    const bool ok = u < K8;
    if (s.mode == X_EMBED_RMS) {
      const uint2 b = ok ? *reinterpret_cast<const uint2*>(erow + 8 * u) : make_uint2(0, 0);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int8_t q = (int8_t)(((j < 4 ? b.x : b.y) >> (8 * (j & 3))) & 0xFF);
        v[i][j] = __fmul_rn((float)q, escale);  // EMBED_BUF: f32(q8) * scale[id]
      }
    } else {
      const float4 a = ok ? *reinterpret_cast<const float4*>(s.x + 8 * u) : make_float4(0, 0, 0, 0);
      const float4 b = ok ? *reinterpret_cast<const float4*>(s.x + 8 * u + 4) : make_float4(0, 0, 0, 0);
      v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
      v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
    }
    if (s.mode != X_PLAIN) {
      const float4 a = ok ? __ldg(reinterpret_cast<const float4*>(s.norm_g + 8 * u)) : make_float4(0, 0, 0, 0);
      const float4 b = ok ? __ldg(reinterpret_cast<const float4*>(s.norm_g + 8 * u + 4)) : make_float4(0, 0, 0, 0);
      gw[i][0] = a.x; gw[i][1] = a.y; gw[i][2] = a.z; gw[i][3] = a.w;
      gw[i][4] = b.x; gw[i][5] = b.y; gw[i][6] = b.z; gw[i][7] = b.w;
    }
  }
  if (s.mode == X_EMBED_RMS && blockIdx.x == 0 && s.hidden_out) {
#pragma unroll
    for (int i = 0; i < MAXU; i++) {
      const int u = threadIdx.x + i * blockDim.x;
      if (u < K8) {
        *reinterpret_cast<float4*>(s.hidden_out + 8 * u) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        *reinterpret_cast<float4*>(s.hidden_out + 8 * u + 4) = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
      }
    }
  }
  if (s.mode != X_PLAIN) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXU; i++)
#pragma unroll
      for (int j = 0; j < 8; j++) ss = __fadd_rn(ss, __fmul_rn(v[i][j], v[i][j]));
    ss = block_sum(ss, sred);
    // RMSNORM: inverseSqrt(sum/K + eps) (kernels.js:142), IEEE sqrt + divide
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), s.eps)));
    const __half inv16 = __float2half_rn(inv);
#pragma unroll
    for (int i = 0; i < MAXU; i++)
#pragma unroll
      for (int j = 0; j < 8; j++) {
        if (!s.f16) {
          v[i][j] = __fmul_rn(__fmul_rn(v[i][j], inv), gw[i][j]);
        } else {  // RMSNORM_F16: f16(f16(x) * inv) * f16(g)
          __half t = __hmul_rn(__float2half_rn(v[i][j]), inv16);
          t = __hmul_rn(t, __float2half_rn(gw[i][j]));
          v[i][j] = __half2float(t);
        }
      }
  }
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < MAXU; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) am = fmaxf(am, fabsf(v[i][j]));
  const int e = shift_for(block_max(am, sred));
#pragma unroll
  for (int i = 0; i < MAXU; i++) {
    const int u = threadIdx.x + i * blockDim.x;
    if (u >= K8) continue;
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; j++) x[j] = e ? ldexpf(v[i][j], -e) : v[i][j];
    if (fmt == 4) {
      uint4* xs = reinterpret_cast<uint4*>(smem);
      uint4* lo = xs + K8 + 4;
      uint4 h, l;
      split_h2(x[0], x[4], h.x, l.x);
      split_h2(x[1] * 0.0625f, x[5] * 0.0625f, h.y, l.y);
      split_h2(x[2], x[6], h.z, l.z);
      split_h2(x[3] * 0.0625f, x[7] * 0.0625f, h.w, l.w);
      const int slot = (u & ~15) + 4 * (u & 3) + ((u >> 2) & 3);
      xs[slot] = h;
      lo[slot] = l;
    } else {
      uint2* xs2 = reinterpret_cast<uint2*>(smem);
      uint2* lo = xs2 + K / 4 + 2;
      uint2 h, l;
      split_h2(x[0], x[2], h.x, l.x);
      split_h2(x[1], x[3], h.y, l.y);
      xs2[2 * u] = h;
      lo[2 * u] = l;
      split_h2(x[4], x[6], h.x, l.x);
      split_h2(x[5], x[7], h.y, l.y);
      xs2[2 * u + 1] = h;
      lo[2 * u + 1] = l;
    }
  }
  __syncthreads();
  return e;
}

// ======================================================================
// Epilogues (GEMV4 / GEMV4_ADD / GATE_UP_SILU_GEMV4, kernels.js:884-1072)
// ======================================================================
__device__ __forceinline__ float lora_dot(const Epi& e, int m, int nm, int Nm) {
  const LoraMod md = e.mods[m];
  if (md.rank <= 0 || !md.B) return 0.f;
  const float* d = e.lora_d + m * kMaxRank;
  float dl = 0.f;
  for (int r = 0; r < md.rank; r++) dl = __fadd_rn(dl, __fmul_rn(d[r], md.B[(size_t)r * Nm + nm]));
  return __fmul_rn(md.scale, dl);
}

__device__ __forceinline__ void epilogue_row(const Epi& e, int n, float v, float v2) {
  if (n >= e.N) return;
  if (e.mode == EPI_SILU) {
    float g = v, u = v2;
    if (e.mods) {
      g = __fadd_rn(g, lora_dot(e, 0, n, e.N));
      u = __fadd_rn(u, lora_dot(e, 1, n, e.N));
    }
    e.y[n] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
    return;
  }
  float o = v;
  if (e.bias) o = __fadd_rn(o, e.bias[n]);
  if (e.mods) {
    int m = 0, nm = n, Nm = e.split1;
    if (n >= e.split2) {
      m = 2;
      nm = n - e.split2;
      Nm = e.N - e.split2;
    } else if (n >= e.split1) {
      m = 1;
      nm = n - e.split1;
      Nm = e.split2 - e.split1;
    }
    o = __fadd_rn(o, lora_dot(e, m, nm, Nm));
  }
  e.y[n] = e.mode == EPI_ADD ? __fadd_rn(e.y[n], o) : o;
}

// ======================================================================
// int4 GEMV
// ======================================================================
// R = row tiles per block (2 for the gate/up pair), U = groups in flight per
// warp, W = warps (split-K over the 128-wide groups).  The first U groups of
// weights are requested before the activation prologue (they do not depend on
// the previous kernel), so their HBM latency overlaps the wait and the
// x-staging; later groups are fetched one batch ahead of the math.
template <int R, int U>
struct WBatch {
  uint4 a[U][R], b[U][R];
};

template <int R, int U, int W>
__device__ __forceinline__ void load_batch(WBatch<R, U>& wb, const uint32_t* __restrict__ w, int K8,
                                           int gpr, int G0, const int (&row_a)[R],
                                           const int (&row_b)[R], const bool (&va)[R],
                                           const bool (&vb)[R], int t) {
#pragma unroll
  for (int u = 0; u < U; u++) {
    const int G = G0 + u * W;
#pragma unroll
    for (int r = 0; r < R; r++) {
      const bool ok = G < gpr;
      wb.a[u][r] = (ok && va[r]) ? ldg_stream(w + (size_t)row_a[r] * K8 + 16 * G + 4 * t)
                                 : make_uint4(0, 0, 0, 0);
      wb.b[u][r] = (ok && vb[r]) ? ldg_stream(w + (size_t)row_b[r] * K8 + 16 * G + 4 * t)
                                 : make_uint4(0, 0, 0, 0);
    }
  }
}

template <int R, int U, int W, int MAXU>
__global__ void __launch_bounds__(W * 32) gemv_q4_kernel(const uint32_t* __restrict__ w,
                                                         const float* __restrict__ s, int N,
                                                         int K, XSrc xsrc, Epi epi, int pdl) {
  extern __shared__ uint4 smem[];
  __shared__ float sred[32];
  __shared__ float red[W][R][16];
  const int K8 = K / 8, gpr = K / kGroup;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, t = lane & 3;
  const int tile = blockIdx.x;

  int row_a[R], row_b[R];
  bool va[R], vb[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const int base = tile * 16 + (r ? N : 0);  // r = 1: the "up" half of [gate;up]
    row_a[r] = base + gq;
    row_b[r] = base + gq + 8;
    va[r] = (tile * 16 + gq) < N;
    vb[r] = (tile * 16 + gq + 8) < N;
  }
  WBatch<R, U> cur;
  load_batch<R, U, W>(cur, w, K8, gpr, warp, row_a, row_b, va, vb, t);

  if (pdl) pdl_wait();
  const int e = stage_x<MAXU>(xsrc, K, 4, smem, sred);
  if (pdl) pdl_launch_dependents();

  const uint4* xs = gq == 0 ? smem : smem + K8 + 4;
  const bool bl = gq < 2;
  float acc[R][2];
#pragma unroll
  for (int r = 0; r < R; r++) acc[r][0] = acc[r][1] = 0.f;

  for (int G0 = warp; G0 < gpr; G0 += W * U) {
    WBatch<R, U> nxt;
    const bool more = G0 + W * U < gpr;
    if (more) load_batch<R, U, W>(nxt, w, K8, gpr, G0 + W * U, row_a, row_b, va, vb, t);
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int G = G0 + u * W;
      if (G >= gpr) break;
      float c[R][4];
#pragma unroll
      for (int r = 0; r < R; r++) c[r][0] = c[r][1] = c[r][2] = c[r][3] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const uint4 xb = bl ? xs[16 * G + 4 * j + t] : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int r = 0; r < R; r++) {
          const uint4& A = cur.a[u][r];
          const uint4& B = cur.b[u][r];
          const uint32_t wa = j == 0 ? A.x : j == 1 ? A.y : j == 2 ? A.z : A.w;
          const uint32_t wbw = j == 0 ? B.x : j == 1 ? B.y : j == 2 ? B.z : B.w;
          uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
          deq_int4(wa, a0, a1, a2, a3);
          deq_int4(wbw, b0, b1, b2, b3);
          mma16816(c[r], a0, b0, a1, b1, xb.x, xb.y);
          mma16816(c[r], a2, b2, a3, b3, xb.z, xb.w);
        }
      }
      if (t == 0) {
#pragma unroll
        for (int r = 0; r < R; r++) {
          const float sa = va[r] ? __ldg(s + (size_t)row_a[r] * gpr + G) : 0.f;
          const float sb = vb[r] ? __ldg(s + (size_t)row_b[r] * gpr + G) : 0.f;
          acc[r][0] = fmaf(sa, c[r][0] + c[r][1], acc[r][0]);
          acc[r][1] = fmaf(sb, c[r][2] + c[r][3], acc[r][1]);
        }
      }
    }
    if (more) cur = nxt;
  }
  if (t == 0) {
#pragma unroll
    for (int r = 0; r < R; r++) {
      red[warp][r][gq] = acc[r][0];
      red[warp][r][gq + 8] = acc[r][1];
    }
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int i = threadIdx.x;
    float v[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      float a = 0.f;
      for (int ww = 0; ww < W; ww++) a += red[ww][r][i];
      v[r] = e ? ldexpf(a, e) : a;
    }
    epilogue_row(epi, tile * 16 + i, v[0], R == 2 ? v[R - 1] : 0.f);
  }
}

// Units of 8 activations per thread (256 threads) the prologue holds.
static int maxu_for(int K) {
  const int u = (K / 8 + 255) / 256;
  return u <= 1 ? 1 : u <= 2 ? 2 : 6;  // K <= 12288
}

template <int R, int U, int MAXU>
static void gemv_q4_go(const uint32_t* w, const float* s, int N, int K, const XSrc& x, const Epi& e,
                       cudaStream_t st, bool pdl) {
  const int tiles = (N + 15) / 16;
  const size_t smem = (size_t)(2 * (K / 8) + 8) * sizeof(uint4);
  auto k = gemv_q4_kernel<R, U, 8, MAXU>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch(k, dim3(tiles), dim3(256), smem, st, pdl, w, s, N, K, x, e, (int)pdl);
}

template <int R, int U>
static void gemv_q4_k(const uint32_t* w, const float* s, int N, int K, const XSrc& x, const Epi& e,
                      cudaStream_t st, bool pdl) {
  switch (maxu_for(K)) {
    case 1: gemv_q4_go<R, U, 1>(w, s, N, K, x, e, st, pdl); break;
    case 2: gemv_q4_go<R, U, 2>(w, s, N, K, x, e, st, pdl); break;
    default: gemv_q4_go<R, U, 6>(w, s, N, K, x, e, st, pdl); break;
  }
}

void gemv_q4(const uint32_t* w, const float* s, int N, int K, const XSrc& x, const Epi& e,
             cudaStream_t st, bool pdl) {
  if (e.mode == EPI_SILU)
    gemv_q4_k<2, 2>(w, s, N, K, x, e, st, pdl);
  else
    gemv_q4_k<1, 4>(w, s, N, K, x, e, st, pdl);
}

// ======================================================================
// int8 GEMV (tied LM head, GEMV kernels.js:20-59) + fused argmax tail
// ======================================================================
template <int U>
struct W8Batch {
  uint4 a[U], b[U];
};
template <int U, int W>
__device__ __forceinline__ void load8(W8Batch<U>& wb, const uint32_t* __restrict__ w, int K4, int nch,
                                      int N, int tile, int C0, int gq, int t) {
  const int ra = tile * 16 + gq, rb = ra + 8;
#pragma unroll
  for (int u = 0; u < U; u++) {
    const int Ch = C0 + u * W;
    wb.a[u] = (Ch < nch && ra < N) ? ldg_stream(w + (size_t)ra * K4 + 16 * Ch + 4 * t) : make_uint4(0, 0, 0, 0);
    wb.b[u] = (Ch < nch && rb < N) ? ldg_stream(w + (size_t)rb * K4 + 16 * Ch + 4 * t) : make_uint4(0, 0, 0, 0);
  }
}

// Grid-stride over 16-row tiles; the activation prologue runs once per block
// and the next tile's first batch of weights is in flight while the current
// tile is reduced.
template <int U, int W, int MAXU>
__global__ void __launch_bounds__(W * 32) gemv_q8_kernel(const uint32_t* __restrict__ w,
                                                         const float* __restrict__ s, int N,
                                                         int K, XSrc xsrc, float* __restrict__ y,
                                                         StepTail tail, int has_tail, int pdl) {
  extern __shared__ uint4 smem4[];
  uint2* smem = reinterpret_cast<uint2*>(smem4);
  __shared__ float sred[32];
  __shared__ float red[W][16];
  __shared__ float best_v[16];
  __shared__ uint32_t best_i[16];
  __shared__ bool last;
  const int K4 = K / 4, nch = K / 64;  // 64-wide chunks
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, t = lane & 3;
  const int tiles = (N + 15) / 16;

  W8Batch<U> cur;
  if (blockIdx.x < tiles) load8<U, W>(cur, w, K4, nch, N, blockIdx.x, warp, gq, t);
  if (pdl) pdl_wait();
  const int e = stage_x<MAXU>(xsrc, K, 8, smem4, sred);
  if (pdl) pdl_launch_dependents();
  const uint2* xs = gq == 0 ? smem : smem + K4 + 2;
  const bool bl = gq < 2;
  float bv = -1e30f;
  uint32_t bi = 0xffffffffu;

  for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    for (int C0 = warp; C0 < nch; C0 += W * U) {
      W8Batch<U> nxt;
      const bool tail_batch = C0 + W * U >= nch;
      const int ntile = tile + gridDim.x;
      if (!tail_batch)
        load8<U, W>(nxt, w, K4, nch, N, tile, C0 + W * U, gq, t);
      else if (ntile < tiles)
        load8<U, W>(nxt, w, K4, nch, N, ntile, warp, gq, t);
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int Ch = C0 + u * W;
        if (Ch >= nch) break;
        const uint4* xp = reinterpret_cast<const uint4*>(xs + 16 * Ch + 4 * t);
        const uint4 x01 = bl ? xp[0] : make_uint4(0, 0, 0, 0);
        const uint4 x23 = bl ? xp[1] : make_uint4(0, 0, 0, 0);
        uint32_t a0, a1, b0, b1;
        deq_int8(cur.a[u].x, a0, a1);
        deq_int8(cur.b[u].x, b0, b1);
        mma16816(c, a0, b0, a1, b1, x01.x, x01.y);
        deq_int8(cur.a[u].y, a0, a1);
        deq_int8(cur.b[u].y, b0, b1);
        mma16816(c, a0, b0, a1, b1, x01.z, x01.w);
        deq_int8(cur.a[u].z, a0, a1);
        deq_int8(cur.b[u].z, b0, b1);
        mma16816(c, a0, b0, a1, b1, x23.x, x23.y);
        deq_int8(cur.a[u].w, a0, a1);
        deq_int8(cur.b[u].w, b0, b1);
        mma16816(c, a0, b0, a1, b1, x23.z, x23.w);
      }
      cur = nxt;
    }
    if (t == 0) {
      red[warp][gq] = c[0] + c[1];
      red[warp][gq + 8] = c[2] + c[3];
    }
    __syncthreads();
    if (threadIdx.x < 16) {
      const int n = tile * 16 + threadIdx.x;
      float a = 0.f;
      for (int ww = 0; ww < W; ww++) a += red[ww][threadIdx.x];
      if (n < N) {
        const float o = __fmul_rn(e ? ldexpf(a, e) : a, __ldg(s + n));  // sum first, scale last
        y[n] = o;
        if (beats(o, (uint32_t)n, bv, bi)) {
          bv = o;
          bi = (uint32_t)n;
        }
      }
    }
    __syncthreads();
  }
  if (!has_tail) return;
  // ---- fused argmax + position advance (ARGMAX kernels.js:771-784, then
  // decodeBatch's copy of s.amax into the id buffer, runtime.js:1783-1785)
  if (threadIdx.x < 16) {
    best_v[threadIdx.x] = bv;
    best_i[threadIdx.x] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = -1e30f;
    uint32_t id = 0xffffffffu;
    for (int i = 0; i < 16; i++)
      if (beats(best_v[i], best_i[i], v, id)) {
        v = best_v[i];
        id = best_i[i];
      }
    tail.cand_v[blockIdx.x] = v;
    tail.cand_i[blockIdx.x] = id;
    __threadfence();
    const unsigned prev = atomicAdd(tail.counter, 1u);
    last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  float v = -1e30f;
  uint32_t id = 0xffffffffu;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
    const float cv = __ldcg(tail.cand_v + b);
    const uint32_t ci = __ldcg(tail.cand_i + b);
    if (beats(cv, ci, v, id)) {
      v = cv;
      id = ci;
    }
  }
  // warp + block argmax reduction, ties to the lower index
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, id, o);
    if (beats(ov, oi, v, id)) {
      v = ov;
      id = oi;
    }
  }
  if (lane == 0) {
    best_v[warp] = v;
    best_i[warp] = id;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    v = best_v[0];
    id = best_i[0];
    for (int i = 1; i < W; i++)
      if (beats(best_v[i], best_i[i], v, id)) {
        v = best_v[i];
        id = best_i[i];
      }
    const int p = *tail.pos;
    if (tail.greedy) {
      *tail.amax = id;
      tail.ids[p + 1] = id;
      const int k = *tail.out_idx;
      tail.out_ids[k] = id;
      *tail.out_idx = k + 1;
    }
    *tail.pos = p + 1;
    *tail.counter = 0u;
  }
}

template <int MAXU>
static void gemv_q8_go(const uint32_t* w, const float* s, int N, int K, const XSrc& x, float* y,
                       const StepTail* tail, cudaStream_t st, bool pdl) {
  const int tiles = (N + 15) / 16;
  const int grid = std::min(tiles, sm_count() * 4);
  const size_t smem = (size_t)(2 * (K / 4) + 4) * sizeof(uint2);
  auto k = gemv_q8_kernel<4, 8, MAXU>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  StepTail tl = {};
  if (tail) tl = *tail;
  launch(k, dim3(grid), dim3(256), smem, st, pdl, w, s, N, K, x, y, tl, tail ? 1 : 0, (int)pdl);
}

void gemv_q8(const uint32_t* w, const float* s, int N, int K, const XSrc& x, float* y,
             const StepTail* tail, cudaStream_t st, bool pdl) {
  switch (maxu_for(K)) {
    case 1: gemv_q8_go<1>(w, s, N, K, x, y, tail, st, pdl); break;
    case 2: gemv_q8_go<2>(w, s, N, K, x, y, tail, st, pdl); break;
    default: gemv_q8_go<6>(w, s, N, K, x, y, tail, st, pdl); break;
  }
}

// ======================================================================
// LoRA A: d[m][r] = A_m[r] . x  (LORA_A, kernels.js:60-78)
// ======================================================================
__global__ void lora_a_kernel(XSrc xsrc, int K, const LoraMod* mods, float* d, int pdl) {
  __shared__ float sred[32];
  extern __shared__ float xsh[];
  const int m = blockIdx.y, r = blockIdx.x;
  if (pdl) pdl_wait();
  const LoraMod md = mods[m];
  if (r >= md.rank || !md.A) return;
  XCtx c;
  setup_x(xsrc, K, c, sred);
  float acc = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x)
    acc = __fadd_rn(acc, __fmul_rn(xval(c, k), md.A[(size_t)r * K + k]));
  acc = block_sum(acc, sred);
  if (threadIdx.x == 0) d[m * kMaxRank + r] = acc;
  (void)xsh;
}

void lora_a(const XSrc& x, int K, const LoraMod* mods, int nmods, int max_rank, float* d,
            cudaStream_t st, bool pdl) {
  if (max_rank <= 0) return;
  launch(lora_a_kernel, dim3(max_rank, nmods), dim3(256), 0, st, pdl, x, K, mods, d, (int)pdl);
}

// ======================================================================
// Attention: RoPE + KV append + split-K partials, then combine
// ======================================================================
// RoPE pair (kernels.js:224-227 / 251-254): two separately rounded products
// then one add; the f16 variant rounds inputs, products and sum to f16.
__device__ __forceinline__ void rope_pair(float& lo, float& hi, float c, float s, int f16) {
  if (!f16) {
    const float a = __fmul_rn(lo, c), b = __fmul_rn(-hi, s);
    const float d = __fmul_rn(hi, c), e = __fmul_rn(lo, s);
    lo = __fadd_rn(a, b);
    hi = __fadd_rn(d, e);
  } else {
    const __half hc = __float2half_rn(c), hs = __float2half_rn(s);
    const __half xl = __float2half_rn(lo), xh = __float2half_rn(hi);
    lo = __half2float(__hadd_rn(__hmul_rn(xl, hc), __hmul_rn(__hneg(xh), hs)));
    hi = __half2float(__hadd_rn(__hmul_rn(xh, hc), __hmul_rn(xl, hs)));
  }
}

__device__ __forceinline__ int attn_chunk(int ctx, int fixed) {
  if (fixed > 0) return fixed;
  int c = (ctx + 63) / 64;          // aim for ~64 splits per KV head
  c = (c + 15) & ~15;
  return c < 16 ? 16 : (c > 64 ? 64 : c);
}
int attn_max_splits(int max_ctx) { return std::max(64, (max_ctx + 15) / 16); }

constexpr int kAttnMaxChunk = 64;
constexpr int kAttnMaxGroup = 8;

template <typename KVT>
__device__ __forceinline__ float kv_load(const KVT* p);
template <>
__device__ __forceinline__ float kv_load<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float kv_load<__half>(const __half* p) { return __half2float(*p); }
template <typename KVT>
__device__ __forceinline__ KVT kv_cvt(float v);
template <>
__device__ __forceinline__ float kv_cvt<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half kv_cvt<__half>(float v) { return __float2half_rn(v); }

template <typename KVT>
__device__ __forceinline__ void kv_row4(const KVT* p, float* dst);  // 4 consecutive values
template <>
__device__ __forceinline__ void kv_row4<float>(const float* p, float* dst) {
  *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ void kv_row4<__half>(const __half* p, float* dst) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  *reinterpret_cast<float4*>(dst) = make_float4(a.x, a.y, b.x, b.y);
}

constexpr int kKsStride = kHeadDim + 4;  // padded K rows (keeps float4 alignment)

// One block per (split, kv head): RoPE on the group's q heads, RoPE + append
// of the new k/v row when this split holds position pos, split-K partials for
// the group's q heads (one warp per head), then the last block of the KV head
// to finish merges all splits (ATTN_COMBINE) and writes the output.
template <typename KVT>
__global__ void __launch_bounds__(256) attn_partial_kernel(AttnArgs a, int pdl) {
  __shared__ __align__(16) float qs[kAttnMaxGroup][kHeadDim];
  extern __shared__ __align__(16) float attn_smem[];
  __shared__ float sc[kAttnMaxGroup][kAttnMaxChunk];
  __shared__ __align__(16) float knew[kHeadDim];
  __shared__ __align__(16) float vnew[kHeadDim];
  __shared__ bool last;
  float* ks = attn_smem;                              // [chunk][kKsStride]
  float* vs = attn_smem + kAttnMaxChunk * kKsStride;  // [chunk][128]
  if (pdl) pdl_wait();
  const int pos = a.pos ? *a.pos : a.fixed_pos;
  const int ctx = pos + 1;
  const int chunk = attn_chunk(ctx, a.chunk);
  const int nsplit = (ctx + chunk - 1) / chunk;
  const int split = blockIdx.x, kvh = blockIdx.y;
  if (split >= nsplit) return;
  if (pdl) pdl_launch_dependents();
  const int G = a.nh / a.nkv, hd = kHeadDim, half = hd / 2;
  const int kvd = a.nkv * hd;
  const int f16 = a.kv_f16;
  const float* cs = a.cosT + (size_t)pos * hd;
  const float* sn = a.sinT + (size_t)pos * hd;
  for (int idx = threadIdx.x; idx < G * half; idx += blockDim.x) {
    const int hh = idx / half, j = idx % half;
    const float* q = a.qkv + (kvh * G + hh) * hd;
    float lo = q[j], hi = q[j + half];
    rope_pair(lo, hi, cs[j], sn[j], f16);
    if (f16) {  // ATTN_PARTIAL_F16 reads q through f16
      lo = round_h(lo);
      hi = round_h(hi);
    }
    qs[hh][j] = lo;
    qs[hh][j + half] = hi;
  }
  const int t0 = split * chunk;
  const int t1 = min(t0 + chunk, ctx);
  const int len = t1 - t0;
  KVT* kc = reinterpret_cast<KVT*>(a.kc);
  KVT* vc = reinterpret_cast<KVT*>(a.vc);
  const bool has_new = pos >= t0 && pos < t1;
  if (has_new) {  // ROPE_QK on k, then the KV append (runtime.js:1509-1514)
    const float* k = a.qkv + a.nh * hd + kvh * hd;
    const float* v = a.qkv + a.nh * hd + kvd + kvh * hd;
    for (int j = threadIdx.x; j < half; j += blockDim.x) {
      float lo = k[j], hi = k[j + half];
      rope_pair(lo, hi, cs[j], sn[j], f16);
      knew[j] = f16 ? round_h(lo) : lo;
      knew[j + half] = f16 ? round_h(hi) : hi;
      kc[(size_t)pos * kvd + kvh * hd + j] = kv_cvt<KVT>(lo);
      kc[(size_t)pos * kvd + kvh * hd + j + half] = kv_cvt<KVT>(hi);
    }
    for (int j = threadIdx.x; j < hd; j += blockDim.x) {
      vnew[j] = f16 ? round_h(v[j]) : v[j];
      vc[(size_t)pos * kvd + kvh * hd + j] = kv_cvt<KVT>(v[j]);
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < len * (hd / 4); idx += blockDim.x) {
    const int tt = idx / (hd / 4), d = 4 * (idx % (hd / 4)), t = t0 + tt;
    if (t == pos) {
      *reinterpret_cast<float4*>(ks + tt * kKsStride + d) = *reinterpret_cast<const float4*>(knew + d);
      *reinterpret_cast<float4*>(vs + tt * hd + d) = *reinterpret_cast<const float4*>(vnew + d);
    } else {
      kv_row4<KVT>(kc + (size_t)t * kvd + kvh * hd + d, ks + tt * kKsStride + d);
      kv_row4<KVT>(vc + (size_t)t * kvd + kvh * hd + d, vs + tt * hd + d);
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float scale = 1.0f / sqrtf((float)hd);
  for (int hh = warp; hh < G; hh += blockDim.x / 32) {
    const float4 q4 = *reinterpret_cast<const float4*>(&qs[hh][4 * lane]);
    float m = -1e30f;
    for (int tt = 0; tt < len; tt++) {
      const float4 k4 = *reinterpret_cast<const float4*>(ks + tt * kKsStride + 4 * lane);
      float p = __fmul_rn(q4.x, k4.x);
      p = __fadd_rn(p, __fmul_rn(q4.y, k4.y));
      p = __fadd_rn(p, __fmul_rn(q4.z, k4.z));
      p = __fadd_rn(p, __fmul_rn(q4.w, k4.w));
      const float sv = __fmul_rn(warp_sum(p), scale);
      if (lane == 0) sc[hh][tt] = sv;
      m = fmaxf(m, sv);
    }
    __syncwarp();
    float z = 0.f;
    for (int tt = lane; tt < len; tt += 32) {
      const float ev = expf(sc[hh][tt] - m);
      sc[hh][tt] = ev;
      z += ev;
    }
    z = warp_sum(z);
    __syncwarp();
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int tt = 0; tt < len; tt++) {
      const float ev = sc[hh][tt];
      const float4 v4 = *reinterpret_cast<const float4*>(vs + tt * hd + 4 * lane);
      acc.x = __fadd_rn(acc.x, __fmul_rn(ev, v4.x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(ev, v4.y));
      acc.z = __fadd_rn(acc.z, __fmul_rn(ev, v4.z));
      acc.w = __fadd_rn(acc.w, __fmul_rn(ev, v4.w));
    }
    const int h = kvh * G + hh;
    *reinterpret_cast<float4*>(a.po + ((size_t)h * a.max_splits + split) * hd + 4 * lane) = acc;
    if (lane == 0) {
      a.pm[h * a.max_splits + split] = m;
      a.pz[h * a.max_splits + split] = z;
    }
  }
  // ---- last block of this KV head merges the splits (ATTN_COMBINE[_F16],
  // kernels.js:346-388)
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(a.counters + kvh, 1u);
    last = prev == (unsigned)nsplit - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int hh = warp; hh < G; hh += blockDim.x / 32) {
    const int h = kvh * G + hh;
    const float* pm = a.pm + h * a.max_splits;
    const float* pz = a.pz + h * a.max_splits;
    float M = -1e30f;
    for (int s2 = 0; s2 < nsplit; s2++) M = fmaxf(M, __ldcg(pm + s2));
    float Z = 0.f;
    for (int s2 = 0; s2 < nsplit; s2++) Z = __fadd_rn(Z, __fmul_rn(__ldcg(pz + s2), expf(__ldcg(pm + s2) - M)));
    const float invZ = 1.0f / Z;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s2 = 0; s2 < nsplit; s2++) {
      const float wgt = expf(__ldcg(pm + s2) - M);
      float4 p = __ldcg(reinterpret_cast<const float4*>(a.po + ((size_t)h * a.max_splits + s2) * hd + 4 * lane));
      if (f16) {
        p.x = round_h(p.x);
        p.y = round_h(p.y);
        p.z = round_h(p.z);
        p.w = round_h(p.w);
      }
      acc.x = __fadd_rn(acc.x, __fmul_rn(wgt, p.x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(wgt, p.y));
      acc.z = __fadd_rn(acc.z, __fmul_rn(wgt, p.z));
      acc.w = __fadd_rn(acc.w, __fmul_rn(wgt, p.w));
    }
    *reinterpret_cast<float4*>(a.out + h * hd + 4 * lane) =
        make_float4(__fmul_rn(acc.x, invZ), __fmul_rn(acc.y, invZ), __fmul_rn(acc.z, invZ),
                    __fmul_rn(acc.w, invZ));
  }
  if (threadIdx.x == 0) a.counters[kvh] = 0u;  // ready for the next launch
}

void attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl) {
  dim3 grid(a.max_splits, a.nkv);
  const int smem = kAttnMaxChunk * (kKsStride + kHeadDim) * (int)sizeof(float);
  if (a.kv_f16) {
    cudaFuncSetAttribute(attn_partial_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    launch(attn_partial_kernel<__half>, grid, dim3(256), smem, st, pdl, a, (int)pdl);
  } else {
    cudaFuncSetAttribute(attn_partial_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    launch(attn_partial_kernel<float>, grid, dim3(256), smem, st, pdl, a, (int)pdl);
  }
}

// ======================================================================
// Standalone small ops (single-op C-ABI entry points)
// ======================================================================
__global__ void rmsnorm_kernel(const float* x, const float* g, int K, float eps, int f16, float* y) {
  __shared__ float sred[32];
  XSrc s = {};
  s.mode = X_RMS;
  s.x = x;
  s.norm_g = g;
  s.eps = eps;
  s.f16 = f16;
  XCtx c;
  setup_x(s, K, c, sred);
  for (int k = threadIdx.x; k < K; k += blockDim.x) y[k] = xval(c, k);
}
void rmsnorm(const float* x, const float* g, int K, float eps, int f16, float* y, cudaStream_t st) {
  rmsnorm_kernel<<<1, 256, 0, st>>>(x, g, K, eps, f16, y);
}

__global__ void rope_qk_kernel(float* q, float* k, int nq, int nkv, int pos, const float* cosT,
                               const float* sinT, int f16) {
  const int half = kHeadDim / 2;
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (nq + nkv) * half) return;
  const int h = g / half, j = g % half;
  float* x = h < nq ? q + h * kHeadDim : k + (h - nq) * kHeadDim;
  float lo = x[j], hi = x[j + half];
  rope_pair(lo, hi, cosT[(size_t)pos * kHeadDim + j], sinT[(size_t)pos * kHeadDim + j], f16);
  x[j] = lo;
  x[j + half] = hi;
}
void rope_qk(float* q, float* k, int nq, int nkv, int pos, const float* cosT, const float* sinT,
             int f16, cudaStream_t st) {
  const int n = (nq + nkv) * kHeadDim / 2;
  rope_qk_kernel<<<(n + 255) / 256, 256, 0, st>>>(q, k, nq, nkv, pos, cosT, sinT, f16);
}

__global__ void embed_kernel(const uint32_t* w, const float* s, const uint32_t* id_dev, int H, float* out) {
  const uint32_t id = *id_dev;
  const int8_t* row = reinterpret_cast<const int8_t*>(w + (size_t)id * (H / 4));
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < H; k += gridDim.x * blockDim.x)
    out[k] = __fmul_rn((float)row[k], s[id]);
}
void embed_rows(const uint32_t* w, const float* s, const uint32_t* id_dev, int H, float* out,
                cudaStream_t st) {
  embed_kernel<<<(H + 255) / 256, 256, 0, st>>>(w, s, id_dev, H, out);
}

__global__ void copy_u32_kernel(const uint32_t* src, uint32_t* dst) { *dst = *src; }
void copy_u32(const uint32_t* src, uint32_t* dst, cudaStream_t st) {
  copy_u32_kernel<<<1, 1, 0, st>>>(src, dst);
}

// ======================================================================
// Sampling: ARGMAX / TOPK_SELECT / SAMPLE_TOPK (kernels.js:771-883)
// ======================================================================
__device__ void block_best(float& v, uint32_t& id, float* sv, uint32_t* si) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, id, o);
    if (beats(ov, oi, v, id)) {
      v = ov;
      id = oi;
    }
  }
  __syncthreads();
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = id;
  }
  __syncthreads();
  v = sv[0];
  id = si[0];
  for (int i = 1; i < nw; i++)
    if (beats(sv[i], si[i], v, id)) {
      v = sv[i];
      id = si[i];
    }
}

int topk_cand_blocks(int n) { return std::max(1, std::min(kCandMax, (n + 1023) / 1024)); }

// Stage 1: per-block argmax candidates.  Stage 2 (one block) merges them.
__global__ void argmax_stage1(const float* logits, int n, float* cv, uint32_t* ci) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  const int per = (n + gridDim.x - 1) / gridDim.x;
  const int b0 = blockIdx.x * per, b1 = min(n, b0 + per);
  float v = -1e30f;
  uint32_t id = 0xffffffffu;
  for (int i = b0 + threadIdx.x; i < b1; i += blockDim.x)
    if (beats(logits[i], (uint32_t)i, v, id)) {
      v = logits[i];
      id = (uint32_t)i;
    }
  block_best(v, id, sv, si);
  if (threadIdx.x == 0) {
    cv[blockIdx.x] = v;
    ci[blockIdx.x] = id;
  }
}
__global__ void argmax_stage2(const float* cv, const uint32_t* ci, int nc, uint32_t* out) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  float v = -1e30f;
  uint32_t id = 0xffffffffu;
  for (int i = threadIdx.x; i < nc; i += blockDim.x)
    if (beats(cv[i], ci[i], v, id)) {
      v = cv[i];
      id = ci[i];
    }
  block_best(v, id, sv, si);
  if (threadIdx.x == 0) *out = id;
}
void argmax(const float* logits, int n, uint32_t* out, float* cand_v, uint32_t* cand_i,
            cudaStream_t st) {
  const int nb = topk_cand_blocks(n);
  argmax_stage1<<<nb, 256, 0, st>>>(logits, n, cand_v, cand_i);
  argmax_stage2<<<1, 256, 0, st>>>(cand_v, cand_i, nb, out);
}

// Top-k in the reference's order (value desc, index asc): each block extracts
// its local top-k by k rounds of block argmax over not-yet-taken elements,
// then one block merges the candidates the same way.  Selecting by this total
// order is exactly the sequence of TOPK_SELECT rounds (kernels.js:785-813).
constexpr int kTopkPer = 8;  // elements per thread in stage 1 (256 threads)
__global__ void topk_stage1(const float* logits, int n, int k, float* cv, uint32_t* ci) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  const int per = (n + gridDim.x - 1) / gridDim.x;
  const int b0 = blockIdx.x * per, b1 = min(n, b0 + per);
  float val[kTopkPer];
  uint32_t idx[kTopkPer];
#pragma unroll
  for (int j = 0; j < kTopkPer; j++) {
    const int i = b0 + threadIdx.x + j * blockDim.x;
    val[j] = i < b1 ? logits[i] : -INFINITY;
    idx[j] = i < b1 ? (uint32_t)i : 0xffffffffu;
  }
  for (int r = 0; r < k; r++) {
    float v = -1e30f;
    uint32_t id = 0xffffffffu;
#pragma unroll
    for (int j = 0; j < kTopkPer; j++)
      if (beats(val[j], idx[j], v, id)) {
        v = val[j];
        id = idx[j];
      }
    block_best(v, id, sv, si);
#pragma unroll
    for (int j = 0; j < kTopkPer; j++)
      if (idx[j] == id && id != 0xffffffffu) val[j] = -INFINITY;  // taken
    if (threadIdx.x == 0) {
      cv[blockIdx.x * k + r] = v;
      ci[blockIdx.x * k + r] = id;
    }
  }
}
__global__ void topk_stage2(const float* cv_in, const uint32_t* ci_in, int nc, int k, uint32_t* ids,
                            float* vals) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  extern __shared__ float cand[];
  float* cvs = cand;
  uint32_t* cis = reinterpret_cast<uint32_t*>(cand + nc);
  for (int i = threadIdx.x; i < nc; i += blockDim.x) {
    cvs[i] = cv_in[i];
    cis[i] = ci_in[i];
  }
  __syncthreads();
  for (int r = 0; r < k; r++) {
    float v = -1e30f;
    uint32_t id = 0xffffffffu;
    int slot = -1;
    for (int i = threadIdx.x; i < nc; i += blockDim.x)
      if (cis[i] != 0xffffffffu && beats(cvs[i], cis[i], v, id)) {
        v = cvs[i];
        id = cis[i];
        slot = i;
      }
    block_best(v, id, sv, si);
    // the owner of the winning slot removes it
    if (slot >= 0 && cis[slot] == id && id != 0xffffffffu) cis[slot] = 0xffffffffu;
    if (threadIdx.x == 0) {
      ids[r] = id;
      vals[r] = v;
    }
    __syncthreads();
  }
}
void topk(const float* logits, int n, int k, uint32_t* ids, float* vals, float* cand_v,
          uint32_t* cand_i, cudaStream_t st) {
  int nb = topk_cand_blocks(n);
  while ((long long)nb * 256 * kTopkPer < n) nb++;
  nb = std::min(nb, kCandMax);
  topk_stage1<<<nb, 256, 0, st>>>(logits, n, k, cand_v, cand_i);
  const int nc = nb * k;
  cudaFuncSetAttribute(topk_stage2, cudaFuncAttributeMaxDynamicSharedMemorySize, nc * 8);
  topk_stage2<<<1, 256, (size_t)nc * 8, st>>>(cand_v, cand_i, nc, k, ids, vals);
}

// SAMPLE_TOPK restated literally: 64 slots, exp without max subtraction,
// pairwise tree sum, Hillis-Steele inclusive prefix, first j with r <= P_j.
__global__ void sample_topk_kernel(const uint32_t* ids, const float* vals, int k, float temp, float r,
                                   uint32_t* out, uint32_t* out2) {
  __shared__ float s[64], red[64];
  const int tid = threadIdx.x;
  const float t = temp <= 0.f ? 1.f : temp;
  float v = -1e30f;
  if (tid < k) {
    const float lv = vals[tid];
    v = lv;
    if (t != 1.f) v = __fdiv_rn(lv, t);
  }
  const float ev = tid < k ? expf(v) : 0.f;
  s[tid] = ev;
  red[tid] = ev;
  __syncthreads();
  for (int stride = 32; stride > 0; stride /= 2) {
    if (tid < stride) red[tid] = __fadd_rn(red[tid], red[tid + stride]);
    __syncthreads();
  }
  const float sum = red[0];
  const float invSum = sum > 0.f ? __fdiv_rn(1.f, sum) : 0.f;
  s[tid] = tid < k ? __fmul_rn(s[tid], invSum) : 0.f;
  __syncthreads();
  for (int stride = 1; stride < 64; stride *= 2) {
    const float add = tid >= stride ? s[tid - stride] : 0.f;
    __syncthreads();
    if (tid >= stride) s[tid] = __fadd_rn(s[tid], add);
    __syncthreads();
  }
  if (tid == 0) {
    uint32_t chosen = k > 0 ? (uint32_t)(k - 1) : 0u;
    if (sum > 0.f)
      for (int j = 0; j < k; j++)
        if (r <= s[j]) {
          chosen = (uint32_t)j;
          break;
        }
    const uint32_t o = k > 0 ? ids[chosen] : 0u;
    *out = o;
    if (out2) *out2 = o;
  }
}
void sample_topk(const uint32_t* ids, const float* vals, int k, float temp, float r, uint32_t* out,
                 uint32_t* out2, cudaStream_t st) {
  sample_topk_kernel<<<1, 64, 0, st>>>(ids, vals, k, temp, r, out, out2);
}

}  // namespace eg
