// eg_tc.cu -- batched int4 GEMV on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, accumulators in tensor memory), sm_100a.
//
// Y[t][n] = sum_g s[n][g] * dot_g(W4 row n, x_t) for up to 32 token vectors
// x_t (the lanes of a batched decode step, or the positions of a prefill
// chunk) over the same stream-layout int4 matrices as the batch-1 GEMV
// (GEMV4 / GEMV4_ADD / GATE_UP_SILU_GEMV4, kernels.js:884-1072, and the
// prefill GEMM4 / GEMM4_ADD_T, kernels.js:389-473).  The arithmetic is the
// batch-1 one: each 128-wide group's dot product is exact in integers,
// sum_k (q + 8) * D_p[k] per base-256 digit plane p of the token's
// fixed-point activation, and is folded into f32 with the group scale.
//
// MMA shape: A = 128 weight rows (one "octet" of 8 row tiles, or 4 tiles of
// gate + up rows) x 128 k as signed bytes q (odd k as 16 q, the batch-1
// nibble trick, matched by the activation digits), expanded once at load
// into 16 KB int8 images in the MMA's shared-memory layout (q4_tc_to_a8);
// B = the digit planes, N = 4 x tokens columns (token t, plane p at column
// 4t + p); D = 128 TMEM lanes x N s32 columns, one fresh accumulator per
// group (4 instructions of K = 32).  The epilogue warps fold every group
// into f32 registers: per row and token, acc01 += s * (P0 + 256 P1) and
// acc23 += s * (P2 + 256 P3); y = 2^-f acc01 + 2^(16-f) acc23 -- the same
// integers as the batch-1 path's (P - offset correction) with unsigned q + 8.
//
// Work split: the (octet, group) items of the matrix, octet-major, are
// divided evenly among the CTAs (split-K where a CTA boundary falls inside
// an octet).  An octet a single CTA covers is finished by it; a split octet
// is finished by the last of its CTAs to arrive, which sums the partial
// outputs in CTA order (deterministic) before the epilogue.
//
// Warp roles (11 warps): 0-7 epilogue (two warpgroups, one per half of the
// tokens; warp w reads TMEM lanes 32 (w % 4) .., and its row's group scale
// from global memory one group ahead); 8 copies the A images (cp.async.bulk,
// 8 slots, freed when the MMAs that read them complete); 9 issues the MMAs
// (one elected thread) and owns the TMEM allocation; 10 copies the B planes
// (4 slots).  TMEM accumulators: up to 4, freed by the epilogue.
//
// The second half of this file is the whole-prompt (prefill) GEMM for more
// than 32 token rows: kind::f16 over f16 nibble images, described there.
#include <algorithm>

#include "eg_batch.h"
#include "eg_common.cuh"
#include "eg_device.cuh"
#include "eg_stream.cuh"
#include "eg_tc.cuh"

namespace eg {

namespace {

constexpr int kTcThreads = 11 * 32;
constexpr int kTcEpiWarps = 8;                 // warps 0-7
constexpr int kTcProdWarp = 8, kTcMmaWarp = 9, kTcBWarp = 10;
constexpr int kTcA = 8;                        // A image slots (one group each)
constexpr int kTcB = 4;                        // B operand slots (digit planes)
constexpr int kTcABytes = 128 * 128;           // 128 rows x 128 bytes
constexpr int kTcMaxTok = 32;
constexpr int kTcBBytes = 4 * kTcMaxTok * 128; // N x 128 bytes
constexpr uint32_t kTcTmemCols = 256;

struct TcArgs {
  const unsigned char* a8;   // [octet][group][16 KB] int8 A images (q4_tc_to_a8)
  const float* sc;           // [octet][group][128] group scale of each MMA row
  int N, K, R, lanes, tpad;  // lanes: token vectors (<= 32); tpad: lanes rounded up to 4
  const unsigned char* xtc;  // B planes: per group 4 tpad x 128 bytes
  const int* xf;             // [lane] fixed-point exponent
  BatchEpi be;
  float* part;               // [ncta][2][32][128]
  unsigned* counters;        // [octets]
  int* err;
  int pdl;
};

struct TcSmem {
  uint64_t a_full[kTcA], a_empty[kTcA], b_full[kTcB], b_empty[kTcB];
  uint64_t acc_full[4], acc_empty[4];
  uint32_t tmem_base;
  int last;
};

// items * ncta < 2^31 for every matrix here (at most 20,000 items x 296 CTAs).
__host__ __device__ __forceinline__ int item_lo(int items, int ncta, int c) {
  return (int)((unsigned)(items * c) / (unsigned)ncta);
}
__device__ __forceinline__ int cta_of(int items, int ncta, int i) {
  int c = (int)((unsigned)(i * ncta) / (unsigned)items);
  while (c + 1 < ncta && item_lo(items, ncta, c + 1) <= i) c++;
  while (c > 0 && item_lo(items, ncta, c) > i) c--;
  return c;
}

// One run of a CTA: octet o, groups [g0, g1).
struct Seg {
  int o, g0, g1;
};

// The CTA's runs (its share of the (octet, group) items, octet-major) in
// order, the same sequence for every warp role.
struct SegIter {
  int gpr;
  int i, i1;  // next item, end
  __device__ SegIter(int gpr_, int octets) : gpr(gpr_) {
    const int items = octets * gpr;
    i = item_lo(items, gridDim.x, blockIdx.x);
    i1 = item_lo(items, gridDim.x, blockIdx.x + 1);
  }
  __device__ bool next(Seg& sg) {
    if (i >= i1) return false;
    sg.o = i / gpr;
    sg.g0 = i % gpr;
    sg.g1 = min(gpr, sg.g0 + (i1 - i));
    i += sg.g1 - sg.g0;
    return true;
  }
};

// Ring position (slot, phase parity) of a pipeline of n slots.
struct Ring {
  int slot, ph;
  __device__ void adv(int n) {
    if (++slot == n) {
      slot = 0;
      ph ^= 1;
    }
  }
};

// The final epilogue of one row and token (batch_epilogue's arithmetic).
template <class Args>
__device__ __forceinline__ void tc_store(const Args& a, int t, int n, float v, float up) {
  const Epi& E = a.be.e;
  const float* lp = a.be.lora_pre;
  if (a.R == 2) {
    float g = v, u = up;
    if (lp) {
      g = __fadd_rn(g, lp[(size_t)t * a.be.lstride + n]);
      u = __fadd_rn(u, lp[(size_t)t * a.be.lstride + E.N + n]);
    }
    const float sg = __fdiv_rn(g, __fadd_rn(1.f, expf(-g)));
    E.y[(size_t)t * a.be.ystride + n] =
        a.be.silu_f16 ? __half2float(__hmul(__float2half_rn(sg), __float2half_rn(u))) : __fmul_rn(sg, u);
    return;
  }
  if (a.be.add_first && E.mode == EPI_ADD) {  // (y + W x) + LoRA
    float* yp = E.y + (size_t)t * a.be.ystride + n;
    float o = __fadd_rn(__ldcg(yp), v);
    if (E.bias) o = __fadd_rn(o, E.bias[n]);
    if (lp) o = __fadd_rn(o, lp[(size_t)t * a.be.lstride + n]);
    *yp = o;
    return;
  }
  float o = v;
  if (E.bias) o = __fadd_rn(o, E.bias[n]);
  if (lp) o = __fadd_rn(o, lp[(size_t)t * a.be.lstride + n]);
  float* yp = E.y + (size_t)t * a.be.ystride + n;
  *yp = E.mode == EPI_ADD ? __fadd_rn(__ldcg(yp), o) : o;
}

}  // namespace

// A operand bytes of one int4 word (8 nibbles, k = 8w .. 8w + 7): the even
// nibbles as signed bytes q, the odd ones in place as 16 q (the activation
// digits of odd k carry the matching 1/16).  Signed A makes the integer dot
// exactly sum q * D with no offset correction.
__device__ __forceinline__ uint2 a_bytes(uint32_t w) {
  // even: u = nibble, (u ^ 8) + 120 = v + 128 in [120, 135] (no carry
  // between bytes), ^ 0x80 = v as a two's-complement byte
  return make_uint2((((w & 0x0F0F0F0Fu) ^ 0x08080808u) + 0x78787878u) ^ 0x80808080u, w & 0xF0F0F0F0u);
}

template <int TH>  // tokens per epilogue warpgroup (tpad / 2 <= TH)
__global__ void __launch_bounds__(kTcThreads, 1) gemv_q4_tc_kernel(TcArgs a) {
  extern __shared__ __align__(1024) unsigned char tc_dsm[];
  __shared__ TcSmem S;
  unsigned char* abuf = tc_dsm;                               // kTcA x 16 KB
  unsigned char* bbuf = abuf + (size_t)kTcA * kTcABytes;      // kTcB x N x 128
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = a.R, TPO = 8 / R;
  const int gpr = a.K / kGroup, tiles = (a.N + 15) / 16, octets = (tiles + TPO - 1) / TPO;
  const int items = octets * gpr;
  const int ncta = gridDim.x, c = blockIdx.x;
  const int ncol = 4 * a.tpad;
  const int NT = min(4, (int)kTcTmemCols / ncol);  // TMEM accumulator slots
  const uint32_t bbytes = (uint32_t)ncol * 128;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcA; i++) {
      mbar_init(&S.a_full[i], 1);
      mbar_init(&S.a_empty[i], 1);
    }
    for (int i = 0; i < kTcB; i++) {
      mbar_init(&S.b_full[i], 1);
      mbar_init(&S.b_empty[i], 1);
    }
    for (int i = 0; i < 4; i++) {
      mbar_init(&S.acc_full[i], 1);
      mbar_init(&S.acc_empty[i], kTcEpiWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kTcMmaWarp) tmem_alloc(&S.tmem_base, kTcTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;
  bool dead = false;

  if (warp == kTcProdWarp) {
    // ---------------------------------------------------- A images
    // the weights depend on no earlier kernel: no griddepcontrol.wait here
    if (a.pdl && lane == 0) pdl_launch_dependents();
    SegIter it(gpr, octets);
    Seg sg;
    Ring ra{0, 0};
    int n = 0;
    while (it.next(sg))
      for (int g = sg.g0; g < sg.g1; g++, n++) {
        if (!dead && !tc_wait(&S.a_empty[ra.slot], ra.ph ^ 1, a.err)) dead = true;
        if (lane == 0) {
          mbar_expect_tx(&S.a_full[ra.slot], kTcABytes);
          bulk_g2s(abuf + (size_t)ra.slot * kTcABytes, a.a8 + ((size_t)sg.o * gpr + g) * kTcABytes, kTcABytes,
                   &S.a_full[ra.slot]);
        }
        __syncwarp();
        ra.adv(kTcA);
      }
    for (int j = 0; j < kTcA && j < n; j++) {  // never leave with a copy in flight
      if (ra.slot == 0) {
        ra.slot = kTcA - 1;
        ra.ph ^= 1;
      } else {
        ra.slot--;
      }
      if (!tc_wait_bounded(&S.a_full[ra.slot], ra.ph)) break;
    }
  } else if (warp == kTcBWarp) {
    // ---------------------------------------------------- B planes
    if (a.pdl) pdl_wait();
    Ring rb{0, 0};
    int nb = 0;
    SegIter it(gpr, octets);
    Seg sg;
    while (it.next(sg))
      for (int g = sg.g0; g < sg.g1; g++, nb++) {
        if (!dead && !tc_wait(&S.b_empty[rb.slot], rb.ph ^ 1, a.err)) dead = true;
        if (lane == 0) {
          mbar_expect_tx(&S.b_full[rb.slot], bbytes);
          bulk_g2s(bbuf + (size_t)rb.slot * kTcBBytes, a.xtc + (size_t)g * bbytes, bbytes, &S.b_full[rb.slot]);
        }
        __syncwarp();
        rb.adv(kTcB);
      }
    for (int j = 0; j < kTcB && j < nb; j++) {  // copies in flight have landed
      if (rb.slot == 0) {
        rb.slot = kTcB - 1;
        rb.ph ^= 1;
      } else {
        rb.slot--;
      }
      tc_wait_bounded(&S.b_full[rb.slot], rb.ph);
    }
  } else if (warp == kTcMmaWarp) {
    // ---------------------------------------------------- MMA issue
    const uint32_t idesc = idesc_i8(128, ncol) | (1u << 7);  // A signed
    Ring ra{0, 0}, rb{0, 0}, rt{0, 0};
    int nm = 0;
    SegIter it(gpr, octets);
    Seg sg;
    while (it.next(sg))
      for (int g = sg.g0; g < sg.g1; g++, nm++) {
        if (!dead && !tc_wait(&S.a_full[ra.slot], ra.ph, a.err)) dead = true;
        if (!dead && !tc_wait(&S.b_full[rb.slot], rb.ph, a.err)) dead = true;
        if (!dead && !tc_wait(&S.acc_empty[rt.slot], rt.ph ^ 1, a.err)) dead = true;
        tc_fence_after();
        if (lane == 0) {
          const unsigned char* A = abuf + (size_t)ra.slot * kTcABytes;
          const unsigned char* B = bbuf + (size_t)rb.slot * kTcBBytes;
          const uint32_t d = tmem + (uint32_t)(rt.slot * ncol);
#pragma unroll
          for (int j = 0; j < 4; j++)  // K = 32 bytes = 2 core matrices per instruction
            mma_i8(d, smem_desc(A + j * 2 * 2048, 2048, 128),
                   smem_desc(B + (size_t)j * 2 * (ncol / 8) * 128, (ncol / 8) * 128, 128), idesc,
                   j > 0);
          mma_commit(&S.acc_full[rt.slot]);
          mma_commit(&S.a_empty[ra.slot]);
          mma_commit(&S.b_empty[rb.slot]);
        }
        __syncwarp();
        ra.adv(kTcA);
        rb.adv(kTcB);
        rt.adv(NT);
      }
    // the MMAs this warp issued have finished before TMEM is freed
    for (int j = 0; j < NT && j < nm; j++) {
      if (rt.slot == 0) {
        rt.slot = NT - 1;
        rt.ph ^= 1;
      } else {
        rt.slot--;
      }
      tc_wait_bounded(&S.acc_full[rt.slot], rt.ph);
    }
  } else if (warp < kTcEpiWarps) {
    // ---------------------------------------------------- epilogue
    if (a.pdl) pdl_wait();
    const int sub = warp & 3, wg = warp >> 2;
    const int m = 32 * sub + lane;  // MMA row = TMEM lane
    const int th = a.tpad / 2, tb = wg * th;  // this warpgroup's tokens [tb, tb + th)
    const int ti = R == 1 ? m >> 4 : m >> 5, r = R == 1 ? 0 : (m >> 4) & 1, row = m & 15;
    float acc01[TH], acc23[TH];
#pragma unroll
    for (int j = 0; j < TH; j++) acc01[j] = acc23[j] = 0.f;
    const int first_o = item_lo(items, ncta, c) / gpr;
    Ring rt{0, 0};
    SegIter it(gpr, octets);
    Seg sg;
    while (it.next(sg)) {
      const float* srow = a.sc + (size_t)sg.o * gpr * 128 + m;  // this row's scale of group g at g * 128
      float s_next = __ldg(srow + (size_t)sg.g0 * 128);
      for (int g = sg.g0; g < sg.g1; g++) {
        const float s_m = s_next;
        if (g + 1 < sg.g1) s_next = __ldg(srow + (size_t)(g + 1) * 128);  // one group ahead
        const int qt = rt.slot;
        if (!dead && !tc_wait(&S.acc_full[qt], rt.ph, a.err)) dead = true;
        rt.adv(NT);
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(32 * sub) << 16) + (uint32_t)(qt * ncol + 4 * tb);
        // 8 tokens (32 columns) per TMEM load
#pragma unroll
        for (int h8 = 0; h8 < (TH + 7) / 8; h8++) {
          if (8 * h8 >= th) break;
          uint32_t v[32];
          tmem_ld32(taddr + 32 * h8, v);
          tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 8; jj++) {
            const int j = 8 * h8 + jj;
            if (j >= th) break;
            const int p01 = (int)v[4 * jj] + 256 * (int)v[4 * jj + 1];
            const int p23 = (int)v[4 * jj + 2] + 256 * (int)v[4 * jj + 3];
            acc01[j] = fmaf(s_m, (float)p01, acc01[j]);
            acc23[j] = fmaf(s_m, (float)p23, acc23[j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.acc_empty[qt]);
      }
      // ---- run done: final or partial output of octet sg.o
      const int o_ = sg.o;
      float y[TH];
#pragma unroll
      for (int j = 0; j < TH; j++) {
        const int t = tb + j;
        const int f = (j < th && t < a.lanes) ? __ldcg(a.xf + t) : 0;
        y[j] = __fadd_rn(__fmul_rn(acc01[j], __int_as_float((127 - f) << 23)),
                         __fmul_rn(acc23[j], __int_as_float((143 - f) << 23)));
        acc01[j] = acc23[j] = 0.f;
      }
      bool fin;
      {  // an octet split across CTAs is finished by the last to arrive
        const int c_lo = cta_of(items, ncta, o_ * gpr);
        const int c_hi = cta_of(items, ncta, o_ * gpr + gpr - 1);
        fin = c_lo == c_hi;
        if (!fin) {
          // partial: every thread stores, the warpgroups meet, ONE thread
          // fences and counts the arrival (a fence per thread serialises)
          float* pp = a.part + ((size_t)c * 2 + (o_ == first_o ? 0 : 1)) * kTcMaxTok * 128;
#pragma unroll
          for (int j = 0; j < TH; j++)
            if (j < th) pp[(size_t)(tb + j) * 128 + m] = y[j];
          __syncwarp();
          asm volatile("bar.sync 2, %0;" ::"n"(kTcEpiWarps * 32) : "memory");
          __syncwarp();
          if (warp == 0 && lane == 0) {
            __threadfence();
            const bool last = atomicAdd(a.counters + o_, 1u) == (unsigned)(c_hi - c_lo);
            if (last) {
              __threadfence();
              a.counters[o_] = 0u;  // for the next launch
            }
            S.last = last;
          }
          __syncwarp();
          asm volatile("bar.sync 2, %0;" ::"n"(kTcEpiWarps * 32) : "memory");
          fin = S.last != 0;
          if (fin) {  // sum the partials in CTA order, four CTAs' loads in flight at a time
#pragma unroll
            for (int j = 0; j < TH; j++) y[j] = 0.f;
            for (int cc = c_lo; cc <= c_hi; cc += 4) {
              float pv[4][TH];
#pragma unroll
              for (int u = 0; u < 4; u++) {
                const int c2 = cc + u;
                const float* qp = nullptr;
                if (c2 <= c_hi) {
                  const int cfirst = item_lo(items, ncta, c2) / gpr;
                  qp = a.part + ((size_t)c2 * 2 + (o_ == cfirst ? 0 : 1)) * kTcMaxTok * 128;
                }
#pragma unroll
                for (int j = 0; j < TH; j++)
                  pv[u][j] = (qp && j < th) ? __ldcg(qp + (size_t)(tb + j) * 128 + m) : 0.f;
              }
#pragma unroll
              for (int u = 0; u < 4; u++)
#pragma unroll
                for (int j = 0; j < TH; j++)
                  if (cc + u <= c_hi) y[j] = __fadd_rn(y[j], pv[u][j]);
            }
          }
          asm volatile("bar.sync 2, %0;" ::"n"(kTcEpiWarps * 32) : "memory");  // S.last reuse
        }
      }
      if (!fin) continue;
      const int n = 16 * (o_ * TPO + ti) + row;
#pragma unroll
      for (int j = 0; j < TH; j++) {
        const float up = __shfl_down_sync(0xffffffffu, y[j], 16);  // R = 2: the up row
        const int t = tb + j;
        if (j >= th || t >= a.lanes || n >= a.N) continue;
        if (R == 2 && r == 1) continue;
        tc_store(a, t, n, y[j], up);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kTcMmaWarp) tmem_free(tmem, kTcTmemCols);
}

// int8 A images from the tc layout: block og = (octet, group) of 128 rows x
// 128 k as signed bytes (even nibbles q, odd nibbles in place as 16 q) in the
// MMA's canonical K-major layout.  Word w of MMA row m's fragment-order
// block holds k = 8w .. 8w + 7: k-chunk w / 2, half w & 1.
__global__ void q4_tc_to_a8_kernel(const unsigned char* __restrict__ wc, int R, unsigned char* __restrict__ a8,
                                   float* __restrict__ sc) {
  const int blk = q4_block_bytes(R), TPO = 8 / R;
  const size_t og = blockIdx.x;
  const unsigned char* st = wc + og * TPO * blk;
  unsigned char* A = a8 + og * kTcABytes;
  const int ct = threadIdx.x;
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int pc = ct + 256 * j;
    const int pl = pc & 31, h = (pc >> 5) & 1, rest = pc >> 6;
    const int ti = R == 1 ? rest : rest >> 1, r = R == 1 ? 0 : rest & 1;
    const int m = R == 1 ? 16 * ti + 8 * h + (pl >> 2) : 32 * ti + 16 * r + 8 * h + (pl >> 2);
    const int t = pl & 3;
    const uint4 v = *reinterpret_cast<const uint4*>(st + ti * blk + r * 1024 + h * 512 + pl * 16);
    unsigned char* rowp = A + (m >> 3) * 128 + (m & 7) * 16 + (t & 1) * 8;
    const int kc = t >> 1;
    *reinterpret_cast<uint2*>(rowp + (kc + 0) * 2048) = a_bytes(v.x);
    *reinterpret_cast<uint2*>(rowp + (kc + 2) * 2048) = a_bytes(v.y);
    *reinterpret_cast<uint2*>(rowp + (kc + 4) * 2048) = a_bytes(v.z);
    *reinterpret_cast<uint2*>(rowp + (kc + 6) * 2048) = a_bytes(v.w);
  }
  if (ct < 128) {  // the group scale of each MMA row
    const int sti = R == 1 ? ct >> 4 : ct >> 5, sr = R == 1 ? 0 : (ct >> 4) & 1, srow = ct & 15;
    sc[og * 128 + ct] =
        *reinterpret_cast<const float*>(st + sti * blk + R * 1024 + 4 * (sr * 16 + 2 * (srow & 7) + (srow >> 3)));
  }
}

// The tc layout: the stream-layout blocks regrouped octet-major, group-next,
// tile-minor ([octet][group][tile of the octet][block]), so that a stage
// (an octet's run of groups) is one contiguous range; tiles past the matrix
// in the last octet are zero blocks.
size_t q4_tc_bytes(int N, int K, int R) {
  const int tiles = (N + 15) / 16, TPO = 8 / R, octets = (tiles + TPO - 1) / TPO;
  return (size_t)octets * TPO * (K / kGroup) * q4_block_bytes(R);
}

__global__ void q4_stream_to_tc_kernel(const uint4* __restrict__ ws, int tiles, int gpr, int TPO,
                                       int blk16, uint4* __restrict__ out, long long n16) {
  for (long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x; u < n16;
       u += (long long)gridDim.x * blockDim.x) {
    const long long b = u / blk16;  // output block: (octet, group, tile in octet)
    const int w = (int)(u % blk16);
    const int i = (int)(b % TPO);
    const long long og = b / TPO;
    const int g = (int)(og % gpr);
    const int tile = (int)(og / gpr) * TPO + i;
    out[u] = tile < tiles ? ws[((long long)tile * gpr + g) * blk16 + w] : make_uint4(0, 0, 0, 0);
  }
}

void q4_stream_to_tc(const unsigned char* ws, int N, int K, int R, unsigned char* out, cudaStream_t st) {
  const int tiles = (N + 15) / 16, TPO = 8 / R, blk16 = q4_block_bytes(R) / 16;
  const long long n16 = (long long)q4_tc_bytes(N, K, R) / 16;
  q4_stream_to_tc_kernel<<<(unsigned)std::min<long long>((n16 + 255) / 256, 148 * 16), 256, 0, st>>>(
      reinterpret_cast<const uint4*>(ws), tiles, K / kGroup, TPO, blk16, reinterpret_cast<uint4*>(out), n16);
}

size_t gemv_q4_tc_part_bytes() { return (size_t)2 * 148 * 2 * kTcMaxTok * 128 * sizeof(float); }
int gemv_q4_tc_max_octets() { return 4096; }

size_t q4_a8_bytes(int N, int K, int R) {
  const int tiles = (N + 15) / 16, TPO = 8 / R, octets = (tiles + TPO - 1) / TPO;
  return (size_t)octets * (K / kGroup) * kTcABytes;
}

size_t q4_row_scale_bytes(int N, int K, int R) { return q4_a8_bytes(N, K, R) / kTcABytes * 128 * sizeof(float); }

void q4_tc_to_a8(const unsigned char* wc, int N, int K, int R, unsigned char* a8, float* sc, cudaStream_t st) {
  q4_tc_to_a8_kernel<<<(unsigned)(q4_a8_bytes(N, K, R) / kTcABytes), 256, 0, st>>>(wc, R, a8, sc);
}

void gemv_q4_tc(const unsigned char* a8, const float* sc, int N, int K, int R, int lanes, const BatchPlanes& xp,
                const BatchEpi& be, float* part, unsigned* counters, int* err, cudaStream_t st, bool pdl) {
  TcArgs a = {};
  a.a8 = a8;
  a.sc = sc;
  a.N = N;
  a.K = K;
  a.R = R;
  a.lanes = lanes;
  a.tpad = xp.tc_tpad;
  a.xtc = static_cast<const unsigned char*>(xp.xtc);
  a.xf = xp.xf;
  a.be = be;
  a.part = part;
  a.counters = counters;
  a.err = err;
  a.pdl = pdl;
  const int gpr = K / kGroup, tiles = (N + 15) / 16, octets = (tiles + 8 / R - 1) / (8 / R);
  const int items = octets * gpr;
  // every SM takes a share of at least 4 groups: a narrow matrix (16 octets
  // for N = 2048) splits each octet over many CTAs, whose partials the last
  // to arrive sums (a fence, an atomic and its partial reads per split octet)
  const int ncta = std::max(1, std::min(sm_count(), items / 4));
  const size_t smem = (size_t)kTcA * kTcABytes + (size_t)kTcB * kTcBBytes;
  void (*kern)(TcArgs) = a.tpad <= 16 ? gemv_q4_tc_kernel<8> : gemv_q4_tc_kernel<16>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ncta);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, a);
}

// ======================================================================
// Whole-prompt GEMM (prefill passes of more than 32 positions)
// ======================================================================
// Many token rows make the MMA's N large, and then the per-group fold of the
// integer path (four digit-plane columns per token, each converted and
// scaled) costs more issue slots than the MMAs.  So the whole-prompt GEMM
// runs kind::f16 with f32 accumulation: A = the 128 x 128 nibble values q of
// an (octet, group) as f16 (exact), expanded once at load into 32 KB images
// in the MMA's shared-memory layout; B = each token's x' = x * 2^f as f16
// hi + lo, STACKED ALONG K (k 0..127 hi, 128..255 lo) against the same A
// twice, so the tensor core adds the two halves and each token needs ONE
// f32 accumulator column.  The products q * hi, q * lo are exact in f32; the
// sum is the f32 accumulation of the tensor core (the reference's GEMM4
// sums f32 products too).  Per group: 16 MMAs of M = 128, N = 128 tokens,
// K = 16; the epilogue folds acc += s * D per token and group, and
// y = 2^-f acc.
//
// Warp roles (19 warps): 0-15 epilogue (warp w reads TMEM lanes 32 (w % 4)
// .. and tokens 32 (w / 4) .. of the tile, and its row's group scales from
// global memory one group ahead); 16 copies A images; 17 issues the MMAs and
// owns TMEM; 18 copies B tiles.  Each CTA walks whole (octet, token tile)
// pairs, octet-major, so CTAs running at once share an octet's images in L2.
namespace {

constexpr int kPgTok = 128;                  // tokens per B tile (MMA N)
constexpr int kPgThreads = 19 * 32;
constexpr int kPgEpiWarps = 16;
constexpr int kPgAWarp = 16, kPgMmaWarp = 17, kPgBWarp = 18;
constexpr int kPgA = 2, kPgB = 2;            // ring slots
constexpr int kPgABytes = 128 * 128 * 2;     // 32 KB: 128 rows x 128 k, f16
constexpr int kPgBBytes = kPgTok * 256 * 2;  // 64 KB: 128 tokens x (128 hi + 128 lo), f16
constexpr uint32_t kPgTmemCols = 2 * kPgTok;  // two accumulators

struct PgArgs {
  const unsigned char* a16;  // [octet][group][32 KB] A images (q4_tc_to_a16)
  const float* s16;          // [octet][group][128] group scale of each MMA row
  int N, K, R, lanes;
  const unsigned char* xh;   // [token tile][group][64 KB] B tiles
  const int* xf;
  BatchEpi be;
  int* err;
};

struct PgSmem {
  uint64_t a_full[kPgA], a_empty[kPgA], b_full[kPgB], b_empty[kPgB];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
};

// Instruction descriptor of tcgen05.mma kind::f16: D f32, A and B f16,
// both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t taddr, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(taddr),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}

__global__ void __launch_bounds__(kPgThreads, 1) gemm_q4_prefill_kernel(PgArgs a) {
  extern __shared__ __align__(1024) unsigned char pg_dsm[];
  __shared__ PgSmem S;
  unsigned char* abuf = pg_dsm;                            // kPgA x 32 KB
  unsigned char* bbuf = abuf + (size_t)kPgA * kPgABytes;   // kPgB x 64 KB
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = a.R, TPO = 8 / R;
  const int gpr = a.K / kGroup, tiles = (a.N + 15) / 16, octets = (tiles + TPO - 1) / TPO;
  const int ntau = (a.lanes + kPgTok - 1) / kPgTok, npairs = octets * ntau;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPgA; i++) {
      mbar_init(&S.a_full[i], 1);
      mbar_init(&S.a_empty[i], 1);
    }
    for (int i = 0; i < kPgB; i++) {
      mbar_init(&S.b_full[i], 1);
      mbar_init(&S.b_empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&S.acc_full[i], 1);
      mbar_init(&S.acc_empty[i], kPgEpiWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kPgMmaWarp) tmem_alloc(&S.tmem_base, kPgTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;
  bool dead = false;

  if (warp == kPgAWarp) {
    // ---------------------------------------------------- A images
    Ring ra{0, 0};
    int n = 0;
    for (int pr = blockIdx.x; pr < npairs; pr += gridDim.x) {
      const int o = pr / ntau;
      for (int g = 0; g < gpr; g++, n++) {
        if (!dead && !tc_wait(&S.a_empty[ra.slot], ra.ph ^ 1, a.err)) dead = true;
        if (lane == 0) {
          mbar_expect_tx(&S.a_full[ra.slot], kPgABytes);
          bulk_g2s(abuf + (size_t)ra.slot * kPgABytes, a.a16 + ((size_t)o * gpr + g) * kPgABytes, kPgABytes,
                   &S.a_full[ra.slot]);
        }
        __syncwarp();
        ra.adv(kPgA);
      }
    }
    for (int j = 0; j < kPgA && j < n; j++) {  // copies in flight have landed
      if (ra.slot == 0) {
        ra.slot = kPgA - 1;
        ra.ph ^= 1;
      } else {
        ra.slot--;
      }
      tc_wait_bounded(&S.a_full[ra.slot], ra.ph);
    }
  } else if (warp == kPgBWarp) {
    // ---------------------------------------------------- B tiles
    Ring rb{0, 0};
    int n = 0;
    for (int pr = blockIdx.x; pr < npairs; pr += gridDim.x) {
      const int tau = pr % ntau;
      for (int g = 0; g < gpr; g++, n++) {
        if (!dead && !tc_wait(&S.b_empty[rb.slot], rb.ph ^ 1, a.err)) dead = true;
        if (lane == 0) {
          mbar_expect_tx(&S.b_full[rb.slot], kPgBBytes);
          bulk_g2s(bbuf + (size_t)rb.slot * kPgBBytes, a.xh + ((size_t)tau * gpr + g) * kPgBBytes, kPgBBytes,
                   &S.b_full[rb.slot]);
        }
        __syncwarp();
        rb.adv(kPgB);
      }
    }
    for (int j = 0; j < kPgB && j < n; j++) {
      if (rb.slot == 0) {
        rb.slot = kPgB - 1;
        rb.ph ^= 1;
      } else {
        rb.slot--;
      }
      tc_wait_bounded(&S.b_full[rb.slot], rb.ph);
    }
  } else if (warp == kPgMmaWarp) {
    // ---------------------------------------------------- MMA issue
    const uint32_t idesc = idesc_f16(128, kPgTok);
    Ring ra{0, 0}, rb{0, 0}, rt{0, 0};
    int n = 0;
    for (int pr = blockIdx.x; pr < npairs; pr += gridDim.x)
      for (int g = 0; g < gpr; g++, n++) {
        if (!dead && !tc_wait(&S.a_full[ra.slot], ra.ph, a.err)) dead = true;
        if (!dead && !tc_wait(&S.b_full[rb.slot], rb.ph, a.err)) dead = true;
        if (!dead && !tc_wait(&S.acc_empty[rt.slot], rt.ph ^ 1, a.err)) dead = true;
        tc_fence_after();
        if (lane == 0) {
          const unsigned char* A = abuf + (size_t)ra.slot * kPgABytes;
          const unsigned char* B = bbuf + (size_t)rb.slot * kPgBBytes;
          const uint32_t d = tmem + (uint32_t)(rt.slot * kPgTok);
          // 8 k-steps of 16 over the hi half of B, then the same A against the lo half
#pragma unroll
          for (int j = 0; j < 16; j++)
            mma_f16(d, smem_desc(A + (j & 7) * 2 * 2048, 2048, 128), smem_desc(B + j * 2 * 2048, 2048, 128),
                    idesc, j > 0);
          mma_commit(&S.acc_full[rt.slot]);
          mma_commit(&S.a_empty[ra.slot]);
          mma_commit(&S.b_empty[rb.slot]);
        }
        __syncwarp();
        ra.adv(kPgA);
        rb.adv(kPgB);
        rt.adv(2);
      }
    for (int j = 0; j < 2 && j < n; j++) {  // the MMAs have finished before TMEM is freed
      if (rt.slot == 0) {
        rt.slot = 1;
        rt.ph ^= 1;
      } else {
        rt.slot--;
      }
      tc_wait_bounded(&S.acc_full[rt.slot], rt.ph);
    }
  } else if (warp < kPgEpiWarps) {
    // ---------------------------------------------------- epilogue
    const int sub = warp & 3, tb = 32 * (warp >> 2);  // TMEM lanes 32 sub.., tokens tb .. tb + 31
    const int m = 32 * sub + lane;
    const int ti = R == 1 ? m >> 4 : m >> 5, r = R == 1 ? 0 : (m >> 4) & 1, row = m & 15;
    Ring rt{0, 0};
    for (int pr = blockIdx.x; pr < npairs; pr += gridDim.x) {
      const int o = pr / ntau, t0 = kPgTok * (pr % ntau) + tb;
      const float* srow = a.s16 + (size_t)o * gpr * 128 + m;  // this row's scale of group g at g * 128
      float acc[32];
#pragma unroll
      for (int j = 0; j < 32; j++) acc[j] = 0.f;
      float s_next = __ldg(srow);
      for (int g = 0; g < gpr; g++) {
        const float s_m = s_next;
        if (g + 1 < gpr) s_next = __ldg(srow + (size_t)(g + 1) * 128);  // one group ahead
        const int qt = rt.slot;
        if (!dead && !tc_wait(&S.acc_full[qt], rt.ph, a.err)) dead = true;
        rt.adv(2);
        tc_fence_after();
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(32 * sub) << 16) + (uint32_t)(qt * kPgTok + tb), v);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.acc_empty[qt]);
#pragma unroll
        for (int j = 0; j < 32; j++) acc[j] = fmaf(s_m, __uint_as_float(v[j]), acc[j]);
      }
      const int n = 16 * (o * TPO + ti) + row;
#pragma unroll
      for (int j = 0; j < 32; j++) {
        const int t = t0 + j;
        const int f = t < a.lanes ? __ldcg(a.xf + t) : 0;
        const float y = __fmul_rn(acc[j], __int_as_float((127 - f) << 23));  // 2^-f, exact
        const float up = __shfl_down_sync(0xffffffffu, y, 16);  // R = 2: the up row
        if (t >= a.lanes || n >= a.N || (R == 2 && r == 1)) continue;
        tc_store(a, t, n, y, up);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kPgMmaWarp) tmem_free(tmem, kPgTmemCols);
}

// A images from the tc layout: block og = (octet, group) of 128 rows x 128 k
// as f16 nibble values, element (m, k) at (k / 8) * 2 KB + (m / 8) * 128 +
// (m % 8) * 16 + (k % 8) * 2 (K-major 8 x 16-byte core matrices).  Word w of MMA row m's fragment-order block
// holds k = 8w .. 8w + 7 (the mapping gemv_q4_tc's converter warps use).
__global__ void q4_tc_to_a16_kernel(const unsigned char* __restrict__ wc, int R, unsigned char* __restrict__ a16) {
  const int blk = q4_block_bytes(R), TPO = 8 / R;
  const size_t og = blockIdx.x;
  const unsigned char* st = wc + og * TPO * blk;
  unsigned char* A = a16 + og * kPgABytes;
  const int ct = threadIdx.x;
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int pc = ct + 256 * j;
    const int pl = pc & 31, h = (pc >> 5) & 1, rest = pc >> 6;
    const int ti = R == 1 ? rest : rest >> 1, r = R == 1 ? 0 : rest & 1;
    const int m = R == 1 ? 16 * ti + 8 * h + (pl >> 2) : 32 * ti + 16 * r + 8 * h + (pl >> 2);
    const int t = pl & 3;
    const uint4 v = *reinterpret_cast<const uint4*>(st + ti * blk + r * 1024 + h * 512 + pl * 16);
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int w = 4 * i + t;  // word index: k = 8w .. 8w + 7
      uint32_t hv[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int q0 = (int)(words[i] << (28 - 8 * e)) >> 28, q1 = (int)(words[i] << (24 - 8 * e)) >> 28;
        const __half2 hh = __floats2half2_rn((float)q0, (float)q1);
        hv[e] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      *reinterpret_cast<uint4*>(A + w * 2048 + (m >> 3) * 128 + (m & 7) * 16) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    }
  }
}

}  // namespace

size_t q4_a16_bytes(int N, int K, int R) {
  const int tiles = (N + 15) / 16, TPO = 8 / R, octets = (tiles + TPO - 1) / TPO;
  return (size_t)octets * (K / kGroup) * kPgABytes;
}
void q4_tc_to_a16(const unsigned char* wc, int N, int K, int R, unsigned char* a16, cudaStream_t st) {
  const unsigned blocks = (unsigned)(q4_a16_bytes(N, K, R) / kPgABytes);
  q4_tc_to_a16_kernel<<<blocks, 256, 0, st>>>(wc, R, a16);
}

void gemm_q4_prefill(const unsigned char* a16, const float* s16, int N, int K, int R, int lanes,
                     const BatchPlanes& xp, const BatchEpi& be, int* err, cudaStream_t st) {
  PgArgs a = {};
  a.a16 = a16;
  a.s16 = s16;
  a.N = N;
  a.K = K;
  a.R = R;
  a.lanes = lanes;
  a.xh = static_cast<const unsigned char*>(xp.xh);
  a.xf = xp.xf;
  a.be = be;
  a.err = err;
  const int tiles = (N + 15) / 16, octets = (tiles + 8 / R - 1) / (8 / R);
  const int npairs = octets * ((lanes + kPgTok - 1) / kPgTok);
  const int smem = kPgA * kPgABytes + kPgB * kPgBBytes;
  cudaFuncSetAttribute(gemm_q4_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  gemm_q4_prefill_kernel<<<std::min(sm_count(), npairs), kPgThreads, smem, st>>>(a);
}

}  // namespace eg
