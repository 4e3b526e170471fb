// eg_device.cuh -- device building blocks shared by the per-op kernels
// (eg_kernels.cu) and the persistent fused decode kernel (eg_fused.cu):
// mbarrier / bulk-copy helpers, block reductions, the activation prologues
// that build MMA B fragments (f16 hi/lo split for the fused kernel, digit
// planes for the integer-MMA GEMVs), GEMV epilogues and one attention work
// item of the fused kernel.
#pragma once
#include <float.h>
#include <math.h>

#include "eg_common.cuh"
#include "eg_kernels.h"

namespace eg {


// ======================================================================
// mbarriers and bulk copies (shared-memory rings fed by cp.async.bulk)
// ======================================================================
constexpr long long kSpinLimit = 1LL << 24;  // polls before a wait gives up

__device__ __forceinline__ bool err_set(const int* err) { return *(volatile const int*)err != 0; }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// One try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or about kWaitSliceNs pass, instead of re-polling (polling warps
// take issue slots from the warps doing the math).
constexpr uint32_t kWaitSliceNs = 20000;
constexpr long long kWaitSlices = 1LL << 17;  // ~2.6 s at most
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(a), "r"(parity), "r"(kWaitSliceNs)
      : "memory");
  return done != 0;
}

// Bounded mbarrier phase wait; false = gave up (error recorded or seen).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t a = smem_addr(bar);
  for (long long i = 0;; i++) {
    if (mbar_try(a, parity)) return true;
    // the error word is a global load (an L2 round trip): only on long waits
    if ((i & 15) == 15 && err_set(err)) return false;
    if (i > kWaitSlices) {
      atomicExch(err, 1);
      return false;
    }
  }
}

// Bounded wait that ignores the error word (draining copies in flight).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  for (long long i = 0; i <= kWaitSlices; i++)
    if (mbar_try(a, parity)) return true;
  return false;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
// global -> shared bulk copy completing on bar (16-byte aligned, size % 16 == 0)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ======================================================================
// Block reductions
// ======================================================================
__device__ __forceinline__ float block_sum(float v, float* sbuf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = kCtaThreads >> 5;
  v = warp_sum(v);
  cta_sync();
  if (lane == 0) sbuf[warp] = v;
  cta_sync();
  float r = 0.f;
  for (int i = 0; i < nw; i++) r += sbuf[i];  // fixed order: deterministic
  return r;
}
// block_sum over the NT threads of named barrier 1 (NT a multiple of 32).
template <int NT>
__device__ __forceinline__ void bar_sync_n() {
  asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}
template <int NT>
__device__ __forceinline__ float block_max_n(float v, float* sbuf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  bar_sync_n<NT>();
  if (lane == 0) sbuf[warp] = v;
  bar_sync_n<NT>();
  float r = sbuf[0];
  for (int i = 1; i < NT / 32; i++) r = fmaxf(r, sbuf[i]);
  return r;
}
template <int NT>
__device__ __forceinline__ float block_sum_n(float v, float* sbuf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  bar_sync_n<NT>();
  if (lane == 0) sbuf[warp] = v;
  bar_sync_n<NT>();
  float r = 0.f;
  for (int i = 0; i < NT / 32; i++) r += sbuf[i];  // fixed order: deterministic
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

__device__ __forceinline__ void setup_x(const XSrc& s, int K, XCtx& c, float* sred) {
  c.mode = s.mode;
  c.f16 = s.f16;
  c.x = s.x;
  c.g = s.norm_g;
  c.erow = nullptr;
  c.escale = 0.f;
  c.inv = 1.f;
  c.inv16 = __float2half_rn(1.f);
  if (s.mode == X_EMBED_RMS) {
    const uint32_t id =
        s.use_fixed_id ? s.fixed_id : __ldcg(s.ids + (s.pos ? __ldcg(s.pos) : s.fixed_pos));
    c.erow = reinterpret_cast<const int8_t*>(s.emb_w + (size_t)id * (K / 4));
    c.escale = s.emb_s[id];
    if (blockIdx.x == 0 && s.hidden_out)
      for (int k = threadIdx.x; k < K; k += kCtaThreads) s.hidden_out[k] = raw_at(c, k);
  }
  if (s.mode != X_PLAIN) {
    float ss = 0.f;
    for (int k = threadIdx.x; k < K; k += kCtaThreads) {
      const float v = raw_at(c, k);
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
    ss = block_sum(ss, sred);
    c.inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), s.eps)));
    c.inv16 = __float2half_rn(c.inv);
  }
}


// Activation prologue of the integer-MMA int4 GEMV.  The vector is put in
// fixed point with one exponent f (from its largest |x|): even elements
// (they meet the low nibbles of the weights) as X = round(x * 2^f), |X| <
// 2^30, odd elements (they meet the high nibbles, which the consumers use in
// place as 16 (q + 8) bytes, without a shift) as X = round(x * 2^(f-4)), so
// both halves carry the same scale into one accumulator.  X is written as
// four balanced base-256 digits d_p in [-128, 127] (X = sum_p d_p 256^p;
// bytes of (X + 0x80808080) ^ 0x80808080), one s8 plane per MMA column:
//   xb:   the m16n8k32 B fragments, uint2 [G][p][t][m] (lane (p, t) of MMA m
//         holds plane p of elements 8(4m+t) + {0,2,4,6} and + {1,3,5,7}),
//   xcor: per group and column pair (2i, 2i+1): the weight-offset correction
//         8 (W_{2i} + 256 W_{2i+1}), W_p = sum over the group of plane p of the
//         even elements + 16 x that of the odd elements,
//   *xf:  f; a row's dot product is 2^-f (C_0 + 65536 C_1), C_i the sum over
//         groups of scale * (column pair i value - xcor).
// pdl: the norm weights are read first, then griddepcontrol.wait, then the
// input (which the previous kernel writes).
// xtc (optional): the same planes also as the tcgen05 B operand (see
// BatchPlanes::xtc), this vector at columns tc_col0 .. tc_col0 + 3 of
// tc_ncol.
// xh (optional, instead of all of the above but *xf): the f16 operand of
// the whole-prompt GEMM, this vector as column xh_col of a 128-column tile
// (the tile's group G at xh + G * 64 KB): x' = x * 2^f with max |x'| < 2^15
// split into f16 hi = f16(x') and lo = f16(x' - hi), stacked along k (hi
// elements 0..127, lo 128..255), K-major 8 x 16-byte core matrices, the 32
// eight-element k-chunks 2 KB apart; *xf = f.
// Staged LoRA A side (optional): d[m * kMaxRank + r] = sum_k x[k] A_m[r][k]
// (LORA_A over the normalised input, kernels.js:60-97) for the nlm modules
// at mods, at most kStageLoraRows rows in all; lsm: kStageLoraRows x NT/32
// floats + kStageLoraRows ints of shared memory.
constexpr int kStageLoraRows = 96;
struct StageLora {
  const LoraMod* mods;
  int nmods;
  float* d;
  float* lsm;
};

template <int MAXU, bool NORM, int NT = kCtaThreads>
__device__ void stage_xd(const XSrc& s, int K, uint2* xb, int* xcor, int* xf, float* sred,
                         int pdl, unsigned char* xtc = nullptr, int tc_ncol = 0,
                         int tc_col0 = 0, unsigned char* xh = nullptr, int xh_col = 0,
                         const StageLora* lora = nullptr) {
  const int K8 = K / 8;
  float v[MAXU][8];
  float gw[NORM ? MAXU : 1][8];
  if (NORM && s.mode != X_PLAIN) {
#pragma unroll
    for (int i = 0; i < MAXU; i++) {
      const int u = threadIdx.x + i * NT;
      const bool ok = u < K8;
      const float4 a = ok ? __ldg(reinterpret_cast<const float4*>(s.norm_g + 8 * u)) : make_float4(0, 0, 0, 0);
      const float4 b = ok ? __ldg(reinterpret_cast<const float4*>(s.norm_g + 8 * u + 4)) : make_float4(0, 0, 0, 0);
      gw[NORM ? i : 0][0] = a.x; gw[NORM ? i : 0][1] = a.y; gw[NORM ? i : 0][2] = a.z; gw[NORM ? i : 0][3] = a.w;
      gw[NORM ? i : 0][4] = b.x; gw[NORM ? i : 0][5] = b.y; gw[NORM ? i : 0][6] = b.z; gw[NORM ? i : 0][7] = b.w;
    }
  }
  if (pdl) pdl_wait();
  const int8_t* erow = nullptr;
  float escale = 0.f;
  if (NORM && s.mode == X_EMBED_RMS) {
    const uint32_t id =
        s.use_fixed_id ? s.fixed_id : __ldcg(s.ids + (s.pos ? __ldcg(s.pos) : s.fixed_pos));
    erow = reinterpret_cast<const int8_t*>(s.emb_w + (size_t)id * (K / 4));
    escale = s.emb_s[id];
  }
#pragma unroll
  for (int i = 0; i < MAXU; i++) {
    const int u = threadIdx.x + i * NT;
    const bool ok = u < K8;
    if (NORM && s.mode == X_EMBED_RMS) {
      const uint2 b = ok ? *reinterpret_cast<const uint2*>(erow + 8 * u) : make_uint2(0, 0);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int8_t q = (int8_t)(((j < 4 ? b.x : b.y) >> (8 * (j & 3))) & 0xFF);
        v[i][j] = __fmul_rn((float)q, escale);  // EMBED_BUF: f32(q8) * scale[id]
      }
    } else {
      const float4 a = ok ? __ldcg(reinterpret_cast<const float4*>(s.x + 8 * u)) : make_float4(0, 0, 0, 0);
      const float4 b = ok ? __ldcg(reinterpret_cast<const float4*>(s.x + 8 * u + 4)) : make_float4(0, 0, 0, 0);
      v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
      v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
    }
  }
  if (NORM && s.mode == X_EMBED_RMS && blockIdx.x == 0 && s.hidden_out) {
#pragma unroll
    for (int i = 0; i < MAXU; i++) {
      const int u = threadIdx.x + i * NT;
      if (u < K8) {
        *reinterpret_cast<float4*>(s.hidden_out + 8 * u) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        *reinterpret_cast<float4*>(s.hidden_out + 8 * u + 4) = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
      }
    }
  }
  if (NORM && s.mode != X_PLAIN) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXU; i++)
#pragma unroll
      for (int j = 0; j < 8; j++) ss = __fadd_rn(ss, __fmul_rn(v[i][j], v[i][j]));
    ss = block_sum_n<NT>(ss, sred);
    // RMSNORM: inverseSqrt(sum/K + eps) (kernels.js:142), IEEE sqrt + divide
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), s.eps)));
    const __half inv16 = __float2half_rn(inv);
#pragma unroll
    for (int i = 0; i < MAXU; i++)
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        if (!s.f16) {
          v[i][j] = __fmul_rn(__fmul_rn(v[i][j], inv), gw[NORM ? i : 0][j]);
          v[i][j + 1] = __fmul_rn(__fmul_rn(v[i][j + 1], inv), gw[NORM ? i : 0][j + 1]);
        } else {  // RMSNORM_F16: f16(f16(x) * inv) * f16(g), two lanes at a time
          __half2 t = __hmul2_rn(__floats2half2_rn(v[i][j], v[i][j + 1]), __half2half2(inv16));
          t = __hmul2_rn(t, __floats2half2_rn(gw[NORM ? i : 0][j], gw[NORM ? i : 0][j + 1]));
          const float2 r = __half22float2(t);
          v[i][j] = r.x;
          v[i][j + 1] = r.y;
        }
      }
  }
  if (lora) {  // the adapter's A rows against the vector this block holds
    constexpr int NW = NT / 32;
    float* part = lora->lsm;
    int* slot = reinterpret_cast<int*>(part + kStageLoraRows * NW);
    const int w = threadIdx.x >> 5, ln = threadIdx.x & 31;
    int row = 0;
    for (int m = 0; m < lora->nmods; m++) {
      const LoraMod md = lora->mods[m];
      if (!md.A) continue;
      const int rk = min(md.rank, kStageLoraRows - row);
      // four rows at a time: their loads are in flight together
      for (int r0 = 0; r0 < rk; r0 += 4) {
        float p[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < MAXU; i++) {
          const int u = threadIdx.x + i * NT;
          if (u >= K8) continue;
          float4 a0[4], a1[4];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const float* Ar = md.A + (size_t)min(r0 + q, rk - 1) * K + 8 * u;
            a0[q] = __ldg(reinterpret_cast<const float4*>(Ar));
            a1[q] = __ldg(reinterpret_cast<const float4*>(Ar + 4));
          }
#pragma unroll
          for (int q = 0; q < 4; q++) {
            p[q] = fmaf(v[i][0], a0[q].x, p[q]); p[q] = fmaf(v[i][1], a0[q].y, p[q]);
            p[q] = fmaf(v[i][2], a0[q].z, p[q]); p[q] = fmaf(v[i][3], a0[q].w, p[q]);
            p[q] = fmaf(v[i][4], a1[q].x, p[q]); p[q] = fmaf(v[i][5], a1[q].y, p[q]);
            p[q] = fmaf(v[i][6], a1[q].z, p[q]); p[q] = fmaf(v[i][7], a1[q].w, p[q]);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int q = 0; q < 4; q++) p[q] += __shfl_xor_sync(0xffffffffu, p[q], o);
#pragma unroll
        for (int q = 0; q < 4; q++)
          if (r0 + q < rk) {
            if (ln == 0) part[(row + r0 + q) * NW + w] = p[q];
            if (threadIdx.x == 0) slot[row + r0 + q] = m * kMaxRank + r0 + q;
          }
      }
      row += rk;
    }
    bar_sync_n<NT>();
    for (int q = threadIdx.x; q < row; q += NT) {
      float t = 0.f;
#pragma unroll
      for (int ww = 0; ww < NW; ww++) t = __fadd_rn(t, part[q * NW + ww]);
      lora->d[slot[q]] = t;
    }
  }
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < MAXU; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) am = fmaxf(am, fabsf(v[i][j]));
  am = block_max_n<NT>(am, sred);
  if (xh) {
    // am < 2^ex; f = 15 - ex puts max |x'| below 2^15 (f = 0 for a zero vector)
    const int ex = ((__float_as_int(am) >> 23) & 0xFF) - 126;
    const int f = am > 0.f ? max(-126, min(126, 15 - ex)) : 0;
    const float sc = __int_as_float((127 + f) << 23);
    if (threadIdx.x == 0) *xf = f;
#pragma unroll
    for (int i = 0; i < MAXU; i++) {
      const int u = threadIdx.x + i * NT;
      if (u >= K8) continue;
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float a = __fmul_rn(v[i][j], sc), b = __fmul_rn(v[i][j + 1], sc);
        const __half2 h = __floats2half2_rn(a, b);
        const float2 hf = __half22float2(h);
        const __half2 l = __floats2half2_rn(__fsub_rn(a, hf.x), __fsub_rn(b, hf.y));
        hi[j / 2] = *reinterpret_cast<const uint32_t*>(&h);
        lo[j / 2] = *reinterpret_cast<const uint32_t*>(&l);
      }
      const int G = u >> 4, q = u & 15;
      unsigned char* gb = xh + (size_t)G * 65536 + (xh_col >> 3) * 128 + (xh_col & 7) * 16;
      *reinterpret_cast<uint4*>(gb + q * 2048) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(gb + (16 + q) * 2048) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    bar_sync_n<NT>();
    return;
  }
  // am < 2^ex, ex from the exponent field (0 and subnormals: f = 126)
  const int ex = ((__float_as_int(am) >> 23) & 0xFF) - 126;
  const int f = min(30 - ex, 126);
  const float se = __int_as_float((127 + f) << 23);  // 2^f (even elements)
  const float so = __int_as_float((123 + f) << 23);  // 2^(f-4) (odd elements)
  if (threadIdx.x == 0) *xf = f;
#pragma unroll
  for (int i = 0; i < MAXU; i++) {
    const int u = threadIdx.x + i * NT;
    uint32_t D[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int X = __float2int_rn(v[i][j] * ((j & 1) ? so : se));  // exact scaling
      D[j] = ((uint32_t)X + 0x80808080u) ^ 0x80808080u;            // balanced base-256 digits
    }
    int W[4];
    uint2 pl[4];
#pragma unroll
    for (int p = 0; p < 4; p++) {
      const uint32_t sel = (uint32_t)(p | ((p + 4) << 4));
      const uint32_t e0 = __byte_perm(D[0], D[2], sel), e1 = __byte_perm(D[4], D[6], sel);
      const uint32_t o0 = __byte_perm(D[1], D[3], sel), o1 = __byte_perm(D[5], D[7], sel);
      pl[p].x = __byte_perm(e0, e1, 0x5410);
      pl[p].y = __byte_perm(o0, o1, 0x5410);
      W[p] = __dp4a((int)pl[p].x, 0x01010101, 16 * __dp4a((int)pl[p].y, 0x01010101, 0));
    }
    // the 16 units of a group sit in 16 consecutive lanes (K8 % 16 == 0)
#pragma unroll
    for (int p = 0; p < 4; p++)
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) W[p] += __shfl_xor_sync(0xffffffffu, W[p], o);
    if (u >= K8) continue;
    const int G = u >> 4, q = u & 15, m = q >> 2, t = q & 3;
#pragma unroll
    for (int p = 0; p < 4; p++) xb[((G * 4 + p) * 4 + t) * 4 + m] = pl[p];
    if (xtc) {  // unit q = k bytes 8q .. 8q + 7: k-chunk q / 2, half q & 1
      unsigned char* gb = xtc + (size_t)G * tc_ncol * 128 + (size_t)(q >> 1) * (tc_ncol / 8) * 128 + (q & 1) * 8;
#pragma unroll
      for (int p = 0; p < 4; p++) {
        const int n = tc_col0 + p;
        *reinterpret_cast<uint2*>(gb + (n >> 3) * 128 + (n & 7) * 16) = pl[p];
      }
    }
    if (q == 0) {
      xcor[2 * G] = 8 * (W[0] + 256 * W[1]);
      xcor[2 * G + 1] = 8 * (W[2] + 256 * W[3]);
    }
  }
  bar_sync_n<NT>();
}

// The same fixed-point digit planes for the int8 (m16n8k32 s8.s8) GEMV:
// units of 4 consecutive elements, 32 units per 128-wide group (one warp).
// Lane (p, t) of MMA m holds plane p of elements 32m + 4t + {0..3} (b0) and
// 32m + 16 + 4t + {0..3} (b1): xb as uint32 [G][p][t][m][2].  The weights
// are signed, so no offset correction is needed; xmul as in stage_xd.
// K: the input length; Kp: K rounded up to 128 (the zero tail is staged too).
template <int MAXU, bool NORM, int NT>
__device__ void stage_xd8(const XSrc& s, int K, int Kp, uint32_t* xb, float* xmul, float* sred,
                          int pdl) {
  const int K4 = K / 4, Kp4 = Kp / 4;
  float v[MAXU][4];
  float gw[NORM ? MAXU : 1][4];
  if (NORM && s.mode != X_PLAIN) {
#pragma unroll
    for (int i = 0; i < MAXU; i++) {
      const int u = threadIdx.x + i * NT;
      const float4 a = u < K4 ? __ldg(reinterpret_cast<const float4*>(s.norm_g + 4 * u)) : make_float4(0, 0, 0, 0);
      gw[NORM ? i : 0][0] = a.x; gw[NORM ? i : 0][1] = a.y; gw[NORM ? i : 0][2] = a.z; gw[NORM ? i : 0][3] = a.w;
    }
  }
  if (pdl) pdl_wait();
#pragma unroll
  for (int i = 0; i < MAXU; i++) {
    const int u = threadIdx.x + i * NT;
    const float4 a = u < K4 ? __ldcg(reinterpret_cast<const float4*>(s.x + 4 * u)) : make_float4(0, 0, 0, 0);
    v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
  }
  if (NORM && s.mode != X_PLAIN) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXU; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) ss = __fadd_rn(ss, __fmul_rn(v[i][j], v[i][j]));
    ss = block_sum_n<NT>(ss, sred);
    // RMSNORM: inverseSqrt(sum/K + eps) (kernels.js:142), IEEE sqrt + divide
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), s.eps)));
    const __half inv16 = __float2half_rn(inv);
#pragma unroll
    for (int i = 0; i < MAXU; i++)
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        if (!s.f16) {
          v[i][j] = __fmul_rn(__fmul_rn(v[i][j], inv), gw[NORM ? i : 0][j]);
          v[i][j + 1] = __fmul_rn(__fmul_rn(v[i][j + 1], inv), gw[NORM ? i : 0][j + 1]);
        } else {  // RMSNORM_F16: f16(f16(x) * inv) * f16(g)
          __half2 t = __hmul2_rn(__floats2half2_rn(v[i][j], v[i][j + 1]), __half2half2(inv16));
          t = __hmul2_rn(t, __floats2half2_rn(gw[NORM ? i : 0][j], gw[NORM ? i : 0][j + 1]));
          const float2 r = __half22float2(t);
          v[i][j] = r.x;
          v[i][j + 1] = r.y;
        }
      }
  }
#pragma unroll
  for (int i = 0; i < MAXU; i++) {
    const int u = threadIdx.x + i * NT;
    float am = fmaxf(fmaxf(fabsf(v[i][0]), fabsf(v[i][1])), fmaxf(fabsf(v[i][2]), fabsf(v[i][3])));
    am = warp_max(am);  // the 32 units of a group are one warp (Kp4 % 32 == 0)
    const int ex = ((__float_as_int(am) >> 23) & 0xFF) - 126;
    const int f = min(30 - ex, 126);
    const float sf = __int_as_float((127 + f) << 23);  // 2^f
    uint32_t D[4];
#pragma unroll
    for (int j = 0; j < 4; j++)
      D[j] = ((uint32_t)__float2int_rn(v[i][j] * sf) + 0x80808080u) ^ 0x80808080u;
    if (u >= Kp4) continue;
    const int G = u >> 5, q = u & 31, m = q >> 3, t = q & 3, hf = (q >> 2) & 1;
#pragma unroll
    for (int p = 0; p < 4; p++) {
      const uint32_t sel = (uint32_t)(p | ((p + 4) << 4));
      const uint32_t w = __byte_perm(__byte_perm(D[0], D[1], sel), __byte_perm(D[2], D[3], sel), 0x5410);
      xb[((((G * 4 + p) * 4 + t) * 4 + m) << 1) + hf] = w;
    }
    if (q == 0) {
      xmul[2 * G] = __int_as_float((127 - f) << 23);      // 2^-f
      xmul[2 * G + 1] = __int_as_float((143 - f) << 23);  // 2^(16-f)
    }
  }
  bar_sync_n<NT>();
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
  e.y[n] = e.mode == EPI_ADD ? __fadd_rn(__ldcg(e.y + n), o) : o;
}

// The global value an epilogue row reads (residual y[n] or bias[n]), loaded
// ahead of time so the epilogue itself does no memory round trip.
__device__ __forceinline__ float epi_pre(const Epi& e, int n) {
  if (n >= e.N) return 0.f;
  if (e.mode == EPI_ADD) return __ldcg(e.y + n);
  if (e.mode == EPI_STORE && e.bias) return __ldg(e.bias + n);
  return 0.f;
}
// epilogue_row with the epi_pre value supplied (no LoRA: fused path).
__device__ __forceinline__ void epilogue_row_pre(const Epi& e, int n, float v, float v2, float pre) {
  if (n >= e.N) return;
  if (e.mode == EPI_SILU) {
    e.y[n] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.f, expf(-v))), v2);
    return;
  }
  if (e.mode == EPI_ADD) {
    e.y[n] = __fadd_rn(pre, v);
    return;
  }
  e.y[n] = e.bias ? __fadd_rn(v, pre) : v;
}

// RoPE pair (kernels.js:224-227 / 251-254): two separately rounded products
// then one add; the f16 variant rounds inputs, products and sum to f16.
__device__ __forceinline__ void rope_pair(float& lo, float& hi, float c, float s, int f16) {
  if (!f16) {
    const float a = __fmul_rn(lo, c), b = __fmul_rn(-hi, s);
    const float d = __fmul_rn(hi, c), e = __fmul_rn(lo, s);
    lo = __fadd_rn(a, b);
    hi = __fadd_rn(d, e);
  } else {
    // (xl*c + -(xh*s), xh*c + xl*s), each product and sum rounded to f16
    const __half2 cs = __floats2half2_rn(c, s);
    const __half2 x = __floats2half2_rn(lo, hi);                     // (xl, xh)
    const __half2 p = __hmul2_rn(x, __low2half2(cs));                 // (xl*c, xh*c)
    const __half2 q = __hmul2_rn(__lowhigh2highlow(x), __high2half2(cs));  // (xh*s, xl*s)
    const __half2 r = __hadd2_rn(p, __halves2half2(__hneg(__low2half(q)), __high2half(q)));
    const float2 f = __half22float2(r);
    lo = f.x;
    hi = f.y;
  }
}

template <typename KVT>
__device__ __forceinline__ KVT kv_cvt(float v);
template <>
__device__ __forceinline__ float kv_cvt<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half kv_cvt<__half>(float v) { return __float2half_rn(v); }


__device__ __forceinline__ void block_best(float& v, uint32_t& id, float* sv, uint32_t* si) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = kCtaThreads >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, id, o);
    if (beats(ov, oi, v, id)) {
      v = ov;
      id = oi;
    }
  }
  cta_sync();
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = id;
  }
  cta_sync();
  v = sv[0];
  id = si[0];
  for (int i = 1; i < nw; i++)
    if (beats(sv[i], si[i], v, id)) {
      v = sv[i];
      id = si[i];
    }
}

// ---- warp-level f16 tensor-core fragments and asynchronous copies (the
// prefill attention and the long-context decode attention)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// d += a (16x16, row) * b (16x8, col), f16 in, f32 accumulate
// not volatile: independent MMAs may be interleaved by the compiler
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 16-byte global -> shared copy; src_bytes 0 fills zeros
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
// (x, y) = hi + lo, each an f16 pair (low half = x)
__device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 f = __half22float2(h);
  hi = h2_bits(h);
  lo = h2_bits(__floats2half2_rn(__fsub_rn(x, f.x), __fsub_rn(y, f.y)));
}
}  // namespace eg
