// eg_prefill.cu -- whole-prompt prefill kernels (prefillBatch,
// runtime.js:1936-2087): token embedding, RoPE + K/V rows into the cache,
// and the causal prefill attention on the tensor cores.
//
// Prefill attention (ATTN_PREFILL_BLOCK, kernels.js:684-770).  One CTA owns
// one KV head and a tile of query rows; its 8 warps are (query head of the
// GQA group, 16-row sub-tile) pairs, so every K/V tile staged in shared
// memory serves the whole group.  Keys go in blocks of 128 aligned at key 0,
// exactly the reference's BK blocks, and each block does the reference's
// online-softmax update: scores S = q.k * 1/sqrt(128) (causal mask), block
// max, m' = max(m, block max), l = l * exp(m - m') + sum exp(s - m'),
// acc = acc * exp(m - m') + P V, out = acc * (1 / l).
//
// The two products run as mma.sync m16n8k16 f16 MMAs with f32 accumulation.
// To keep f32 accuracy every f32 operand x is split into f16 hi = f16(x) and
// lo = f16(x - hi) (x = hi + lo to about 2^-22 relative): QK uses
// qh.kh + ql.kh + qh.kl and PV ph.vh + pl.vh + ph.vl; with the f16 cache
// (kv_f16) q, K and V are f16 values already (ROPE_T_F16 rounds q and k; the
// cache stores V as f16), so QK is one MMA and PV two.  Operands must stay
// inside the f16 range (|x| < 65504), as the f16 cache requires anyway.
#include <math.h>
#include <algorithm>
#include <type_traits>

#include "eg_common.cuh"
#include "eg_device.cuh"
#include "eg_prefill.h"
#include "eg_stream.cuh"

namespace eg {

namespace {

constexpr int kPfThreads = 256;  // 8 warps
constexpr int kPfPitch = 136;    // halfs per shared row (272 B: ldmatrix rows hit distinct banks)
constexpr int kPfTileBytes = 128 * kPfPitch * 2;

__global__ void prefill_embed_kernel(const uint32_t* ids, const uint32_t* w, const float* s, int H, float* out) {
  const int t = blockIdx.x;
  const uint32_t id = ids[t];
  const int8_t* row = reinterpret_cast<const int8_t*>(w + (size_t)id * (H / 4));
  const float sc = s[id];
  for (int k = threadIdx.x; k < H; k += blockDim.x) out[(size_t)t * H + k] = __fmul_rn((float)row[k], sc);
}

template <typename KVT>
__global__ void prefill_rope_append_kernel(float* qkv, int stride, int nh, int nkv, int pos0, const float* cosT,
                                           const float* sinT, int f16, KVT* kc, KVT* vc) {
  const int t = blockIdx.x, lane = threadIdx.x & 31, pos = pos0 + t;
  const int kvd = nkv * kHeadDim;
  float cj[4], sj[4];
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const int j = (4 * lane + c) & (kHeadDim / 2 - 1);
    cj[c] = __ldg(cosT + (size_t)pos * kHeadDim + j);
    sj[c] = __ldg(sinT + (size_t)pos * kHeadDim + j);
  }
  float* row = qkv + (size_t)t * stride;
  for (int hh = threadIdx.x >> 5; hh < nh + 2 * nkv; hh += blockDim.x >> 5) {
    float4* x = reinterpret_cast<float4*>(row + hh * kHeadDim + 4 * lane);
    float4 v = *x;
    KVT* dst;
    if (hh < nh) {
      *x = rope_lane4(v, cj, sj, f16, f16 != 0);
      continue;
    } else if (hh < nh + nkv) {
      v = rope_lane4(v, cj, sj, f16, false);
      dst = kc + (size_t)pos * kvd + (hh - nh) * kHeadDim + 4 * lane;
    } else {
      dst = vc + (size_t)pos * kvd + (hh - nh - nkv) * kHeadDim + 4 * lane;
    }
    dst[0] = kv_cvt<KVT>(v.x);
    dst[1] = kv_cvt<KVT>(v.y);
    dst[2] = kv_cvt<KVT>(v.z);
    dst[3] = kv_cvt<KVT>(v.w);
  }
}

// four f32 values into shared memory as f16 hi (and lo when `lo` is set)
__device__ __forceinline__ void put4(__half* hi, __half* lo, float4 v) {
  uint32_t h0, l0, h1, l1;
  split2(v.x, v.y, h0, l0);
  split2(v.z, v.w, h1, l1);
  *reinterpret_cast<uint2*>(hi) = make_uint2(h0, h1);
  if (lo) *reinterpret_cast<uint2*>(lo) = make_uint2(l0, l1);
}

template <typename KVT>
__global__ void __launch_bounds__(kPfThreads, 1) attn_prefill_kernel(PrefillAttn a, int hw, int nsub, int hc) {
  constexpr bool F32 = std::is_same<KVT, float>::value;
  constexpr int NQ = F32 ? 2 : 1, NK = F32 ? 2 : 1;  // f16 parts of q and of K / V
  constexpr int TILE = 128 * kPfPitch;                // halfs per shared tile
  extern __shared__ __align__(16) unsigned char pf_sm[];
  // f32 cache: q hi/lo, K hi/lo, V hi/lo.  f16 cache: q, then two buffers of
  // (K, V): block b + 1 is copied (cp.async) while block b computes.
  __half* Qs = reinterpret_cast<__half*>(pf_sm);  // [NQ][128 rows][pitch]
  __half* Ks = Qs + NQ * TILE;                     // [NK][128 keys][pitch] (buffer 0)
  __half* Vs = Ks + NK * TILE;                     // [NK][128 keys][pitch] (buffer 0)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gsz = a.nh / a.nkv, qt = 16 * nsub;
  const int tile = gridDim.x - 1 - blockIdx.x;  // the longest rows start first
  const int kvh = blockIdx.y / hc, hci = blockIdx.y % hc;
  const int hl = warp % hw, sub = warp / hw;
  const bool active = sub < nsub && hci * hw + hl < gsz;
  const int h = kvh * gsz + hci * hw + hl;
  const int t0 = tile * qt + sub * 16;  // this warp's first query row
  const int kvd = a.nkv * kHeadDim;

  // q rows of this warp (16 x 128) as f16 hi (and lo)
  for (int i = 0; i < 16; i++) {
    const int t = t0 + i;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (active && t < a.T)
      v = __ldcg(reinterpret_cast<const float4*>(a.qkv + (size_t)t * a.qkv_stride + h * kHeadDim) + lane);
    __half* d = Qs + (warp * 16 + i) * kPfPitch + 4 * lane;
    put4(d, NQ == 2 ? d + TILE : nullptr, v);
  }

  const int tend = min(a.T, (tile + 1) * qt);   // rows of the CTA: < tend
  const int kend = min(a.ctx, a.q_start + tend);  // keys any of them sees: < kend
  const int nblk = (kend + 127) / 128;
  const float scl = __fdiv_rn(1.f, __fsqrt_rn((float)kHeadDim));
  const int g = lane >> 2, tq = lane & 3;
  const int abs0 = a.q_start + t0 + g, abs1 = abs0 + 8;  // rows of c[0..1] and c[2..3]
  float O[16][4];
#pragma unroll
  for (int j = 0; j < 16; j++) O[j][0] = O[j][1] = O[j][2] = O[j][3] = 0.f;
  float m0 = -1e30f, m1 = -1e30f, l0 = 0.f, l1 = 0.f;
  const uint32_t qa_addr = smem_addr(Qs + (warp * 16 + (lane & 15)) * kPfPitch + (lane >> 4) * 8);
  const uint32_t kb_addr = smem_addr(Ks + ((lane & 7) + ((lane >> 4) << 3)) * kPfPitch + ((lane >> 3) & 1) * 8);
  const uint32_t vb_addr = smem_addr(Vs + ((lane & 7) + (((lane >> 3) & 1) << 3)) * kPfPitch + (lane >> 4) * 8);

  // f16 cache: K / V rows of block b into buffer buf (rows past kend zero)
  auto issue_f16 = [&](int b, int buf) {
    const __half* kc = static_cast<const __half*>(a.kc);
    const __half* vc = static_cast<const __half*>(a.vc);
    __half* kd = Ks + buf * 2 * TILE;
    __half* vd = kd + TILE;
    for (int i = threadIdx.x; i < 128 * 16; i += kPfThreads) {
      const int r = i >> 4, c8 = i & 15, key = b * 128 + r;
      const bool ok = key < kend;
      const size_t off = ok ? (size_t)key * kvd + kvh * kHeadDim + 8 * c8 : 0;
      cp_async16(kd + r * kPfPitch + 8 * c8, kc + off, ok ? 16 : 0);
      cp_async16(vd + r * kPfPitch + 8 * c8, vc + off, ok ? 16 : 0);
    }
    cp_async_commit();
  };
  if (!F32) issue_f16(0, 0);

  for (int b = 0; b < nblk; b++) {
    const int kb = b * 128;
    const uint32_t boff = F32 ? 0u : (uint32_t)((b & 1) * 2 * TILE * 2);  // this block's buffer, bytes
    if (!F32) {
      if (b + 1 < nblk) {
        issue_f16(b + 1, (b + 1) & 1);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
    } else {
      __syncthreads();  // the previous block's tiles are consumed
      const float* kc = static_cast<const float*>(a.kc);
      const float* vc = static_cast<const float*>(a.vc);
      for (int i = threadIdx.x; i < 128 * 32; i += kPfThreads) {
        const int r = i >> 5, c4 = i & 31, key = kb + r;
        float4 k4 = make_float4(0.f, 0.f, 0.f, 0.f), v4 = k4;
        if (key < kend) {
          k4 = __ldg(reinterpret_cast<const float4*>(kc + (size_t)key * kvd + kvh * kHeadDim) + c4);
          v4 = __ldg(reinterpret_cast<const float4*>(vc + (size_t)key * kvd + kvh * kHeadDim) + c4);
        }
        __half* kd = Ks + r * kPfPitch + 4 * c4;
        __half* vd = Vs + r * kPfPitch + 4 * c4;
        put4(kd, kd + TILE, k4);
        put4(vd, vd + TILE, v4);
      }
      __syncthreads();
    }
    if (active) {

      // ---- S = q K^T over the block's 128 keys (16 n-tiles of 8 keys)
      float S[16][4];
#pragma unroll
      for (int j = 0; j < 16; j++) S[j][0] = S[j][1] = S[j][2] = S[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {
        uint32_t qh[4], ql[4];
        ldsm_x4(qa_addr + ks * 32, qh[0], qh[1], qh[2], qh[3]);
        if (NQ == 2) ldsm_x4(qa_addr + TILE * 2 + ks * 32, ql[0], ql[1], ql[2], ql[3]);
#pragma unroll
        for (int np = 0; np < 8; np++) {
          const uint32_t ka = kb_addr + boff + (np * 16 * kPfPitch + ks * 16) * 2;
          uint32_t b0, b1, b2, b3;
          ldsm_x4(ka, b0, b1, b2, b3);
          mma16816(S[2 * np], qh, b0, b1);
          mma16816(S[2 * np + 1], qh, b2, b3);
          if (F32) {
            mma16816(S[2 * np], ql, b0, b1);
            mma16816(S[2 * np + 1], ql, b2, b3);
            ldsm_x4(ka + TILE * 2, b0, b1, b2, b3);
            mma16816(S[2 * np], qh, b0, b1);
            mma16816(S[2 * np + 1], qh, b2, b3);
          }
        }
      }
      // ---- scale, causal mask, block max of each of the thread's two rows
      float bm0 = -1e30f, bm1 = -1e30f;
#pragma unroll
      for (int j = 0; j < 16; j++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int key = kb + 8 * j + 2 * tq + (c & 1);
          const bool ok = key < kend && key <= (c < 2 ? abs0 : abs1);
          const float s = ok ? __fmul_rn(S[j][c], scl) : -1e30f;
          S[j][c] = s;
          if (c < 2) bm0 = fmaxf(bm0, s);
          else bm1 = fmaxf(bm1, s);
        }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, o));
        bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, o));
      }
      const float n0 = fmaxf(m0, bm0), n1 = fmaxf(m1, bm1);
      const float corr0 = expf(m0 - n0), corr1 = expf(m1 - n1);
      float bs0 = 0.f, bs1 = 0.f;
#pragma unroll
      for (int j = 0; j < 16; j++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int key = kb + 8 * j + 2 * tq + (c & 1);
          const bool ok = key < kend && key <= (c < 2 ? abs0 : abs1);
          const float p = ok ? expf(S[j][c] - (c < 2 ? n0 : n1)) : 0.f;
          S[j][c] = p;
          if (c < 2) bs0 = __fadd_rn(bs0, p);
          else bs1 = __fadd_rn(bs1, p);
        }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        bs0 = __fadd_rn(bs0, __shfl_xor_sync(0xffffffffu, bs0, o));
        bs1 = __fadd_rn(bs1, __shfl_xor_sync(0xffffffffu, bs1, o));
      }
      l0 = __fadd_rn(__fmul_rn(l0, corr0), bs0);
      l1 = __fadd_rn(__fmul_rn(l1, corr1), bs1);
      m0 = n0;
      m1 = n1;
#pragma unroll
      for (int j = 0; j < 16; j++) {
        O[j][0] = __fmul_rn(O[j][0], corr0);
        O[j][1] = __fmul_rn(O[j][1], corr0);
        O[j][2] = __fmul_rn(O[j][2], corr1);
        O[j][3] = __fmul_rn(O[j][3], corr1);
      }
      // ---- O += P V: P from the S accumulators (A fragments of 16 keys)
#pragma unroll
      for (int kk = 0; kk < 8; kk++) {
        uint32_t ph[4], pl[4];
        split2(S[2 * kk][0], S[2 * kk][1], ph[0], pl[0]);
        split2(S[2 * kk][2], S[2 * kk][3], ph[1], pl[1]);
        split2(S[2 * kk + 1][0], S[2 * kk + 1][1], ph[2], pl[2]);
        split2(S[2 * kk + 1][2], S[2 * kk + 1][3], ph[3], pl[3]);
#pragma unroll
        for (int dn = 0; dn < 8; dn++) {
          const uint32_t va = vb_addr + boff + (kk * 16 * kPfPitch + dn * 16) * 2;
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(va, b0, b1, b2, b3);
          mma16816(O[2 * dn], ph, b0, b1);
          mma16816(O[2 * dn + 1], ph, b2, b3);
          mma16816(O[2 * dn], pl, b0, b1);
          mma16816(O[2 * dn + 1], pl, b2, b3);
          if (F32) {
            ldsm_x4_t(va + TILE * 2, b0, b1, b2, b3);
            mma16816(O[2 * dn], ph, b0, b1);
            mma16816(O[2 * dn + 1], ph, b2, b3);
          }
        }
      }
    }  // active
    if (!F32) __syncthreads();  // this buffer is refilled with block b + 2 next
  }
  if (!active) return;
  const float inv0 = __fdiv_rn(1.f, l0), inv1 = __fdiv_rn(1.f, l1);
  const int ta = t0 + g, tb = ta + 8;
#pragma unroll
  for (int j = 0; j < 16; j++) {
    const int d = 8 * j + 2 * tq;
    if (ta < a.T)
      *reinterpret_cast<float2*>(a.out + (size_t)ta * a.out_stride + h * kHeadDim + d) =
          make_float2(__fmul_rn(O[j][0], inv0), __fmul_rn(O[j][1], inv0));
    if (tb < a.T)
      *reinterpret_cast<float2*>(a.out + (size_t)tb * a.out_stride + h * kHeadDim + d) =
          make_float2(__fmul_rn(O[j][2], inv1), __fmul_rn(O[j][3], inv1));
  }
}

}  // namespace

void prefill_embed(const uint32_t* ids, const uint32_t* emb_w, const float* emb_s, int T, int H, float* hidden,
                   cudaStream_t st) {
  prefill_embed_kernel<<<T, 256, 0, st>>>(ids, emb_w, emb_s, H, hidden);
}

void prefill_rope_append(float* qkv, int T, int qkv_stride, int nh, int nkv, int pos0, const float* cosT,
                         const float* sinT, int kv_f16, void* kc, void* vc, cudaStream_t st) {
  const int threads = 32 * std::min(nh + 2 * nkv, 32);
  if (kv_f16)
    prefill_rope_append_kernel<__half><<<T, threads, 0, st>>>(qkv, qkv_stride, nh, nkv, pos0, cosT, sinT, 1,
                                                              static_cast<__half*>(kc), static_cast<__half*>(vc));
  else
    prefill_rope_append_kernel<float><<<T, threads, 0, st>>>(qkv, qkv_stride, nh, nkv, pos0, cosT, sinT, 0,
                                                             static_cast<float*>(kc), static_cast<float*>(vc));
}

void attn_prefill(const PrefillAttn& a, cudaStream_t st) {
  const int gsz = a.nh / a.nkv, hw = std::min(gsz, 8), nsub = 8 / hw, hc = (gsz + hw - 1) / hw;
  const int qt = 16 * nsub, tiles = (a.T + qt - 1) / qt;
  const dim3 grid(tiles, a.nkv * hc);
  if (a.kv_f16) {
    const int smem = 5 * kPfTileBytes;
    cudaFuncSetAttribute(attn_prefill_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attn_prefill_kernel<__half><<<grid, kPfThreads, smem, st>>>(a, hw, nsub, hc);
  } else {
    const int smem = 6 * kPfTileBytes;
    cudaFuncSetAttribute(attn_prefill_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attn_prefill_kernel<float><<<grid, kPfThreads, smem, st>>>(a, hw, nsub, hc);
  }
}

}  // namespace eg
