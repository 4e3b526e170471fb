// eg_batch.cu -- multi-sequence batched decode kernels (sm_100a).
//
// A batch step runs the single-sequence decode step (runtime.js:1466-1571)
// for up to 16 sequences ("lanes") at once.  The weights are the same
// stream-layout matrices as the batch-1 path and every tile crosses HBM once
// per step; the integer-MMA arithmetic is the batch-1 arithmetic with more B
// columns in use:
//   * a staging kernel (one CTA per lane) puts each lane's GEMV input through
//     the batch-1 activation prologue (RMSNorm, fixed point, four base-256
//     digit planes + group corrections) into global memory;
//   * the batched GEMV keeps the producer / consumer / epilogue warp roles;
//     its 16 consumer warps are 4 k-slices x 4 lane quarters: warp (ks, vq)
//     takes the blocks g = ks (mod 4) of each tile and, per block, two
//     m16n8k32 n-tiles = lanes 4vq .. 4vq+3 x 4 digit planes, so all eight
//     MMA columns carry data (the batch-1 kernel uses four);
//   * the epilogue warp sums the four k-slices per (lane, row) and runs the
//     batch-1 epilogue (bias / residual / SiLU / LoRA) on each lane's output.
#include <math.h>

#include <algorithm>

#include "eg_batch.h"
#include "eg_common.cuh"
#include "eg_device.cuh"
#include "eg_stream.cuh"

namespace eg {

constexpr int kBW = 16;                    // consumer warps
constexpr int kBThreads = kBW * 32 + 64;   // + producer + epilogue
constexpr int kStageThreads = 512;         // staging CTA (one per lane)
constexpr int kBBarBytes = 256;
constexpr int kBRingBudget = 150 * 1024;

// Every batch kernel is launched with programmatic dependent launch when
// `pdl`: it reads its predecessors' outputs only after griddepcontrol.wait
// (the GEMV's weight stream, which depends on nothing, starts before it).
template <typename Kern, typename... Args>
static void blaunch(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
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

__device__ __forceinline__ XSrc lane_src(const BatchSrc& b, int v) {
  XSrc s = b.x;
  if (s.x) s.x += (size_t)v * b.stride;
  if (s.hidden_out) s.hidden_out += (size_t)v * b.stride;
  if (s.mode == X_EMBED_RMS) {
    const int slot = b.seq.lane_slot[v];
    s.pos = b.seq.pos + slot;
    // chunked prefill: lane v embeds the token of position pos + v
    s.ids = b.seq.ids + (size_t)slot * b.seq.slot_ctx + (b.seq.chunk ? v : 0);
    s.use_fixed_id = 0;
  }
  return s;
}

// ----------------------------------------------------------- staging
// LoRA A rows folded into the staging (lane v's d at d + v * dstride).
struct LoraFold {
  const LoraMod* mods;
  int nmods;
  float* d;
  int dstride;
};

template <int MAXU, bool NORM>
__global__ void __launch_bounds__(kStageThreads) batch_stage_q4_kernel(BatchSrc b, int K,
                                                                        BatchPlanes xp, LoraFold lf, int pdl) {
  __shared__ float sred[32];
  __shared__ float lsm[kStageLoraRows * (kStageThreads / 32 + 1)];
  const int v = blockIdx.y;
  // the lane's slot (X_EMBED_RMS) was set before the step began
  const XSrc s = lane_src(b, v);
  uint2* xb = reinterpret_cast<uint2*>(xp.xb) + (size_t)v * xp.gpr_max * 64;
  StageLora sl = {lf.mods, lf.nmods, lf.d + (size_t)v * lf.dstride, lsm};
  stage_xd<MAXU, NORM, kStageThreads>(s, K, xb, xp.xcor + (size_t)v * 2 * xp.gpr_max, xp.xf + v,
                                      sred, pdl, static_cast<unsigned char*>(xp.xtc), 4 * xp.tc_tpad, 4 * v,
                                      xp.xh ? static_cast<unsigned char*>(xp.xh) + (size_t)(v / 128) * (K / kGroup) * 65536
                                            : nullptr,
                                      v % 128, lf.mods ? &sl : nullptr);
  if (pdl) pdl_launch_dependents();
}

bool batch_stage_q4(const BatchSrc& s, int K, int lanes, const BatchPlanes& xp, cudaStream_t st, bool pdl,
                    const LoraMod* mods, int nmods, int max_rank, float* d, int dstride) {
  const int u = (K / 8 + kStageThreads - 1) / kStageThreads;
  const dim3 grid(1, lanes);
  const bool norm = s.x.mode != X_PLAIN;
  const bool fold = mods && nmods * max_rank <= kStageLoraRows;
  const LoraFold lf = {fold ? mods : nullptr, nmods, d, dstride};
  if (u <= 1) {
    if (norm) blaunch(batch_stage_q4_kernel<1, true>, grid, dim3(kStageThreads), 0, st, pdl, s, K, xp, lf, (int)pdl);
    else blaunch(batch_stage_q4_kernel<1, false>, grid, dim3(kStageThreads), 0, st, pdl, s, K, xp, lf, (int)pdl);
  } else if (u <= 3) {
    if (norm) blaunch(batch_stage_q4_kernel<3, true>, grid, dim3(kStageThreads), 0, st, pdl, s, K, xp, lf, (int)pdl);
    else blaunch(batch_stage_q4_kernel<3, false>, grid, dim3(kStageThreads), 0, st, pdl, s, K, xp, lf, (int)pdl);
  } else {
    if (norm) blaunch(batch_stage_q4_kernel<6, true>, grid, dim3(kStageThreads), 0, st, pdl, s, K, xp, lf, (int)pdl);
    else blaunch(batch_stage_q4_kernel<6, false>, grid, dim3(kStageThreads), 0, st, pdl, s, K, xp, lf, (int)pdl);
  }
  return fold;
}

template <int MAXU, bool NORM>
__global__ void __launch_bounds__(kStageThreads) batch_stage_q8_kernel(BatchSrc b, int K,
                                                                        BatchPlanes xp, int pdl) {
  __shared__ float sred[32];
  const int v = blockIdx.y;
  const XSrc s = lane_src(b, v);
  const int Kp = (K + kGroup - 1) / kGroup * kGroup;
  uint32_t* xb = reinterpret_cast<uint32_t*>(xp.xb) + (size_t)v * xp.gpr_max * 128;
  stage_xd8<MAXU, NORM, kStageThreads>(s, K, Kp, xb, xp.xmul + (size_t)v * 2 * xp.gpr_max, sred,
                                       pdl);
  if (pdl) pdl_launch_dependents();
}

void batch_stage_q8(const BatchSrc& s, int K, int lanes, const BatchPlanes& xp, cudaStream_t st,
                    bool pdl) {
  const int Kp4 = (K + kGroup - 1) / kGroup * kGroup / 4;
  const int u = (Kp4 + kStageThreads - 1) / kStageThreads;
  const dim3 grid(1, lanes);
  const bool norm = s.x.mode != X_PLAIN;
  if (u <= 1) {
    if (norm) blaunch(batch_stage_q8_kernel<1, true>, grid, dim3(kStageThreads), 0, st, pdl, s, K, xp, (int)pdl);
    else blaunch(batch_stage_q8_kernel<1, false>, grid, dim3(kStageThreads), 0, st, pdl, s, K, xp, (int)pdl);
  } else {
    if (norm) blaunch(batch_stage_q8_kernel<6, true>, grid, dim3(kStageThreads), 0, st, pdl, s, K, xp, (int)pdl);
    else blaunch(batch_stage_q8_kernel<6, false>, grid, dim3(kStageThreads), 0, st, pdl, s, K, xp, (int)pdl);
  }
}

// ----------------------------------------------------------- batched GEMVs
template <int R>
struct BRed {
  float v[2][4][kBatchMax][R][16];  // [buffer][k-slice][lane][r][row]
  float l[2][kBatchMax][R][16];     // LoRA B terms computed at hand-off (lora_pre null)
};

struct GBArgs {
  const unsigned char* ws;  // stream layout
  const float* s;           // int8: row scales
  int N, K, lanes;
  BatchPlanes xp;
  BatchEpi be;              // int4
  float* y;                 // int8: logits [lanes][ystride]
  int ystride;
  int* err;
  int stages, stage_bytes, cap;
  int pdl;
};

__device__ __forceinline__ void batch_barriers(uint64_t* full, uint64_t* empty,
                                               uint64_t* tile_full, uint64_t* tile_free,
                                               int stages) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kBW);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tile_full[i], kBW);
      mbar_init(&tile_free[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
}

// LoRA B term of row n of lane vector v (lora_b_batch's value: the module
// split of epilogue_row, or gate (half 0) / up (half 1) for SiLU).
__device__ __forceinline__ float batch_lora(const BatchEpi& be, int v, int n, int half) {
  Epi e = be.e;
  e.lora_d += (size_t)v * be.dstride;
  if (e.mode == EPI_SILU) return lora_dot(e, half, n, e.N);
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
  return lora_dot(e, m, nm, Nm);
}

// Consumer hand-off of one tile: lane (gq, t) holds, per n-tile nt and
// weight half r, rows gq and gq + 8 of lane vector 4vq + 2nt + (t >> 1),
// column pair t & 1 (already scaled); the pair sum goes to red.
template <int R>
__device__ __forceinline__ void batch_handoff(BRed<R>& red, uint64_t* tile_full,
                                              uint64_t* tile_free, int tj, float (&acc)[2][R][2],
                                              const float (&scl)[2], int ks, int vq, bool& dead,
                                              int* err, const BatchEpi* lf = nullptr, int n0 = 0,
                                              int lanes = 0) {
  const int lane = threadIdx.x & 31, gq = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; nt++)
#pragma unroll
    for (int r = 0; r < R; r++) {
      acc[nt][r][0] *= scl[nt];
      acc[nt][r][1] *= scl[nt];
      acc[nt][r][0] += __shfl_xor_sync(0xffffffffu, acc[nt][r][0], 1);
      acc[nt][r][1] += __shfl_xor_sync(0xffffffffu, acc[nt][r][1], 1);
    }
  const int b = tj & 1;
  if (!dead && !mbar_wait(&tile_free[b], ((tj >> 1) & 1) ^ 1, err)) dead = true;
  if (lf) {  // LoRA B: the 4 warps of lane quad vq share its 4 x R x 16 terms
    for (int w = lane + 32 * ks; w < 4 * R * 16; w += 128) {
      const int vi = w / (R * 16), r = (w / 16) % R, row = w % 16;
      const int v = vq * 4 + vi, n = n0 + row;
      red.l[b][v][r][row] = (v < lanes && n < lf->e.N) ? batch_lora(*lf, v, n, r) : 0.f;
    }
  }
  if ((t & 1) == 0) {
#pragma unroll
    for (int nt = 0; nt < 2; nt++) {
      const int vo = vq * 4 + nt * 2 + (t >> 1);
#pragma unroll
      for (int r = 0; r < R; r++) {
        red.v[b][ks][vo][r][gq] = acc[nt][r][0];
        red.v[b][ks][vo][r][gq + 8] = acc[nt][r][1];
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < 2; nt++)
#pragma unroll
    for (int r = 0; r < R; r++) acc[nt][r][0] = acc[nt][r][1] = 0.f;
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&tile_full[b]);
}

// Walk this warp's blocks (g = ks mod 4 of every tile) through the ring,
// calling body(bp, g) per block and hand(tile) after each tile.
template <typename Body, typename Hand>
__device__ __forceinline__ void batch_walk(const unsigned char* ring, uint64_t* full,
                                           uint64_t* empty, int stages, int stage_bytes, int cap,
                                           int ntiles, int gpr, int blk, int ks, bool& dead,
                                           int* err, Body body, Hand hand) {
  const int lane = threadIdx.x & 31;
  const int nitems = ntiles * gpr;
  const int nchunks = (nitems + cap - 1) / cap;
  if (nchunks == 0) return;
  RingPos rp = {0, 0};
  int chunk = 0, chunk_lo = 0;
  if (!dead && !mbar_wait(&full[rp.st], rp.ph, err)) dead = true;
  const unsigned char* stage = ring + (size_t)rp.st * stage_bytes;
  int i = ks;
  for (int j = 0; j < ntiles; j++) {
    const int tile_end = (j + 1) * gpr;
    for (; i < tile_end; i += 4) {
      while (i >= chunk_lo + cap) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[rp.st]);
        ring_advance(rp, stages);
        chunk++;
        chunk_lo += cap;
        stage = ring + (size_t)rp.st * stage_bytes;
        if (!dead && !mbar_wait(&full[rp.st], rp.ph, err)) dead = true;
      }
      body(stage + (size_t)(i - chunk_lo) * blk, i - j * gpr);
    }
    hand(j);
  }
  for (; chunk < nchunks; chunk++) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[rp.st]);
    ring_advance(rp, stages);
    if (chunk + 1 < nchunks && !dead && !mbar_wait(&full[rp.st], rp.ph, err)) dead = true;
  }
}

// Epilogue of one row n for every lane (the single-lane epilogue_row with
// LoRA added from lora_pre): all loads are issued before any store.
// R == 1: this lane holds lane vectors hi + 2i; R == 2: lanes 0-15 hold the
// gate rows and 16-31 the up rows of every lane vector.
template <int R>
__device__ __forceinline__ void batch_epilogue(const BatchEpi& be, int lanes, int n, int hi,
                                               const float (&val)[R == 2 ? kBatchMax : kBatchMax / 2],
                                               const float* ls = nullptr) {
  // ls (optional): this row's LoRA B terms from the hand-off, term (v, r) at ls[(v * R + r) * 16]
  const Epi& E = be.e;
  const bool ok_n = n < E.N;
  const float* lp = be.lora_pre;
  if (R == 2) {  // GATE_UP_SILU: y = silu(g) * u
    float up[kBatchMax], lg[kBatchMax], lu[kBatchMax];
#pragma unroll
    for (int i = 0; i < kBatchMax; i++) {
      up[i] = __shfl_down_sync(0xffffffffu, val[i], 16);
      const bool ok = hi == 0 && ok_n && i < lanes && lp;
      lg[i] = ok ? lp[(size_t)i * be.lstride + n] : ls ? ls[(i * 2) * 16] : 0.f;
      lu[i] = ok ? lp[(size_t)i * be.lstride + E.N + n] : ls ? ls[(i * 2 + 1) * 16] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kBatchMax; i++) {
      if (hi != 0 || !ok_n || i >= lanes) continue;
      float g = val[i], u = up[i];
      if (lp || ls) {
        g = __fadd_rn(g, lg[i]);
        u = __fadd_rn(u, lu[i]);
      }
      E.y[(size_t)i * be.ystride + n] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
    }
    return;
  }
  constexpr int NV = kBatchMax / 2;
  const float bn = (E.bias && ok_n) ? E.bias[n] : 0.f;
  float res[NV], lo[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int v = hi + 2 * i;
    const bool ok = ok_n && v < lanes;
    res[i] = (ok && E.mode == EPI_ADD) ? __ldcg(E.y + (size_t)v * be.ystride + n) : 0.f;
    lo[i] = (ok && lp) ? lp[(size_t)v * be.lstride + n] : (ok && ls) ? ls[v * 16] : 0.f;
  }
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int v = hi + 2 * i;
    if (!ok_n || v >= lanes) continue;
    float o = val[i];
    if (E.bias) o = __fadd_rn(o, bn);
    if (lp || ls) o = __fadd_rn(o, lo[i]);
    E.y[(size_t)v * be.ystride + n] = E.mode == EPI_ADD ? __fadd_rn(res[i], o) : o;
  }
}

template <int R, bool Q8>
__global__ void __launch_bounds__(kBThreads, 1) gemv_batch_kernel(GBArgs p) {
  extern __shared__ __align__(128) unsigned char gb_smem[];
  __shared__ BRed<R> red;
  uint64_t* full = reinterpret_cast<uint64_t*>(gb_smem);
  uint64_t* empty = full + p.stages;
  uint64_t* tile_full = empty + p.stages;
  uint64_t* tile_free = tile_full + 2;
  unsigned char* ring = gb_smem + kBBarBytes;
  const int gpr = (p.K + kGroup - 1) / kGroup;
  const int blk = Q8 ? kQ8Block : q4_block_bytes(R);
  const int tiles = (p.N + 15) / 16;
  const int t_lo = (int)((long long)tiles * blockIdx.x / gridDim.x);
  const int t_hi = (int)((long long)tiles * (blockIdx.x + 1) / gridDim.x);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  batch_barriers(full, empty, tile_full, tile_free, p.stages);

  if (warp == kBW) {  // producer
    RingPos rp = {0, 0};
    int issued = 0;
    ring_produce(ring, full, empty, p.stages, p.stage_bytes, p.ws + (size_t)t_lo * gpr * blk,
                 (t_hi - t_lo) * gpr, p.cap, blk, rp, issued, p.err, lane);
    ring_drain(full, p.stages, rp, issued);
    return;
  }

  if (warp == kBW + 1) {  // epilogue: sum the k-slices, per lane vector and row
    if (p.pdl) pdl_wait();  // residuals / LoRA terms come from earlier kernels
    const int row = lane & 15, hi = lane >> 4;
    int tj = 0;
    for (int tile = t_lo; tile < t_hi; tile++, tj++) {
      const int b = tj & 1;
      if (!mbar_wait(&tile_full[b], (tj >> 1) & 1, p.err)) return;
      // R == 2: lanes 0-15 gate rows, 16-31 up rows of every lane vector;
      // R == 1: lanes 0-15 even vectors, 16-31 odd vectors
      constexpr int NV = R == 2 ? kBatchMax : kBatchMax / 2;
      float val[NV];
#pragma unroll
      for (int i = 0; i < NV; i++) {
        const int v = R == 2 ? i : hi + 2 * i;
        const int r = R == 2 ? hi : 0;
        val[i] = ((red.v[b][0][v][r][row] + red.v[b][1][v][r][row]) + red.v[b][2][v][r][row]) +
                 red.v[b][3][v][r][row];
      }
      const bool lfold = !Q8 && p.be.e.mods && !p.be.lora_pre;  // LoRA B terms in red.l
      if (!lfold) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&tile_free[b]);
      }
      const int n = tile * 16 + row;
      if (Q8) {
#pragma unroll
        for (int i = 0; i < NV; i++) {
          const int v = hi + 2 * i;
          // GEMV (kernels.js:20-59): the row sum first, the row scale last
          if (v < p.lanes && n < p.N) p.y[(size_t)v * p.ystride + n] = __fmul_rn(val[i], p.s[n]);
        }
      } else {
        batch_epilogue<R>(p.be, p.lanes, n, hi, val, lfold ? &red.l[b][0][0][row] : nullptr);
      }
      if (lfold) {  // red.l[b] read: the buffer is free
        __syncwarp();
        if (lane == 0) mbar_arrive(&tile_free[b]);
      }
    }
    return;
  }

  // consumers: the staged activations come from the previous kernel
  if (p.pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
  const int ks = warp & 3, vq = warp >> 2;
  const int gq = lane >> 2, t = lane & 3;
  const uint4* xcol[2];
  const int* cor[2];
  const float* mul[2];
  float scl[2];
#pragma unroll
  for (int nt = 0; nt < 2; nt++) {
    const int vb = vq * 4 + nt * 2 + (gq >> 2);  // B column gq: lane vb, plane gq & 3
    const int vo = vq * 4 + nt * 2 + (t >> 1);   // C columns 2t, 2t+1: lane vo, pair t & 1
    xcol[nt] = reinterpret_cast<const uint4*>(p.xp.xb) + (size_t)vb * p.xp.gpr_max * 32 +
               ((gq & 3) * 4 + t) * 2;
    if (Q8) {
      cor[nt] = nullptr;
      mul[nt] = p.xp.xmul + (size_t)vo * 2 * p.xp.gpr_max + (t & 1);
      scl[nt] = 1.f;
    } else {
      mul[nt] = nullptr;
      cor[nt] = p.xp.xcor + (size_t)vo * 2 * p.xp.gpr_max + (t & 1);
      const int f = __ldg(p.xp.xf + vo);
      scl[nt] = __int_as_float(((t & 1) ? 143 - f : 127 - f) << 23);  // 2^-f / 2^(16-f)
    }
  }
  float acc[2][R][2];
#pragma unroll
  for (int nt = 0; nt < 2; nt++)
#pragma unroll
    for (int r = 0; r < R; r++) acc[nt][r][0] = acc[nt][r][1] = 0.f;
  bool dead = false;
  int tj = 0;
  auto body = [&](const unsigned char* bp, int g) {
    if (Q8) {
      const uint4 A0 = *reinterpret_cast<const uint4*>(bp + lane * 16);
      const uint4 A1 = *reinterpret_cast<const uint4*>(bp + 512 + lane * 16);
      const uint4 B0 = *reinterpret_cast<const uint4*>(bp + 1024 + lane * 16);
      const uint4 B1 = *reinterpret_cast<const uint4*>(bp + 1536 + lane * 16);
#pragma unroll
      for (int nt = 0; nt < 2; nt++) {
        const uint4 X0 = __ldg(xcol[nt] + g * 32), X1 = __ldg(xcol[nt] + g * 32 + 1);
        const float m = __ldg(mul[nt] + 2 * g);
        int cc[4] = {0, 0, 0, 0};
        imma16832_ss(cc, A0.x, B0.x, A0.y, B0.y, X0.x, X0.y);
        imma16832_ss(cc, A0.z, B0.z, A0.w, B0.w, X0.z, X0.w);
        imma16832_ss(cc, A1.x, B1.x, A1.y, B1.y, X1.x, X1.y);
        imma16832_ss(cc, A1.z, B1.z, A1.w, B1.w, X1.z, X1.w);
        acc[nt][0][0] = fmaf(m, (float)(cc[0] + 256 * cc[1]), acc[nt][0][0]);
        acc[nt][0][1] = fmaf(m, (float)(cc[2] + 256 * cc[3]), acc[nt][0][1]);
      }
    } else {
      uint32_t al[R][4], bl[R][4], ah[R][4], bh[R][4];
      float2 s2[R];
      const float2* sc = reinterpret_cast<const float2*>(bp + R * 1024);  // (row gq, row gq+8)
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint4 A = *reinterpret_cast<const uint4*>(bp + r * 1024 + lane * 16);
        const uint4 B = *reinterpret_cast<const uint4*>(bp + r * 1024 + 512 + lane * 16);
        const uint32_t aw[4] = {A.x, A.y, A.z, A.w}, bw[4] = {B.x, B.y, B.z, B.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          al[r][q] = nib_lo_u8(aw[q]);
          bl[r][q] = nib_lo_u8(bw[q]);
          ah[r][q] = nib_hi16_u8(aw[q]);
          bh[r][q] = nib_hi16_u8(bw[q]);
        }
        s2[r] = sc[8 * r + gq];
      }
#pragma unroll
      for (int nt = 0; nt < 2; nt++) {
        const uint4 X0 = __ldg(xcol[nt] + g * 32), X1 = __ldg(xcol[nt] + g * 32 + 1);
        const int cr = __ldg(cor[nt] + 2 * g);
#pragma unroll
        for (int r = 0; r < R; r++) {
          int cc[4] = {0, 0, 0, 0};
          imma16832(cc, al[r][0], bl[r][0], ah[r][0], bh[r][0], X0.x, X0.y);
          imma16832(cc, al[r][1], bl[r][1], ah[r][1], bh[r][1], X0.z, X0.w);
          imma16832(cc, al[r][2], bl[r][2], ah[r][2], bh[r][2], X1.x, X1.y);
          imma16832(cc, al[r][3], bl[r][3], ah[r][3], bh[r][3], X1.z, X1.w);
          acc[nt][r][0] = fmaf(s2[r].x, (float)(cc[0] + 256 * cc[1] - cr), acc[nt][r][0]);
          acc[nt][r][1] = fmaf(s2[r].y, (float)(cc[2] + 256 * cc[3] - cr), acc[nt][r][1]);
        }
      }
    }
  };
  const bool lfold = !Q8 && p.be.e.mods && !p.be.lora_pre;
  auto hand = [&](int j) {
    batch_handoff<R>(red, tile_full, tile_free, tj, acc, scl, ks, vq, dead, p.err, lfold ? &p.be : nullptr,
                     (t_lo + j) * 16, p.lanes);
    tj++;
  };
  batch_walk(ring, full, empty, p.stages, p.stage_bytes, p.cap, t_hi - t_lo, gpr, blk, ks, dead,
             p.err, body, hand);
}

template <int R, bool Q8>
static void gemv_batch_go(GBArgs a, cudaStream_t st, bool pdl) {
  const int blk = Q8 ? kQ8Block : q4_block_bytes(R);
  a.cap = Q8 ? 16 : 32 / R;
  a.stage_bytes = a.cap * blk;
  a.stages = std::max(2, std::min(8, (kBRingBudget - kBBarBytes) / a.stage_bytes));
  const int smem = kBBarBytes + a.stages * a.stage_bytes;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int P = std::min(sms, (a.N + 15) / 16);
  a.pdl = pdl ? 1 : 0;
  auto k = gemv_batch_kernel<R, Q8>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  blaunch(k, dim3(P), dim3(kBThreads), (size_t)smem, st, pdl, a);
}

void gemv_q4_batch(const unsigned char* ws, int N, int K, int lanes, const BatchPlanes& xp,
                   const BatchEpi& be, int* err, cudaStream_t st, bool pdl) {
  GBArgs a = {};
  a.ws = ws;
  a.N = N;
  a.K = K;
  a.lanes = lanes;
  a.xp = xp;
  a.be = be;
  a.err = err;
  if (be.e.mode == EPI_SILU)
    gemv_batch_go<2, false>(a, st, pdl);
  else
    gemv_batch_go<1, false>(a, st, pdl);
}

void gemv_q8_batch(const unsigned char* ws, const float* s, int N, int K, int lanes,
                   const BatchPlanes& xp, float* y, int ystride, int* err, cudaStream_t st,
                   bool pdl) {
  GBArgs a = {};
  a.ws = ws;
  a.s = s;
  a.N = N;
  a.K = K;
  a.lanes = lanes;
  a.xp = xp;
  a.y = y;
  a.ystride = ystride;
  a.err = err;
  gemv_batch_go<1, true>(a, st, pdl);
}

// ----------------------------------------------------------- attention
template <typename KVT>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_batch_kernel(AttnArgs a0, AttnBatch b,
                                                                      int pdl) {
  __shared__ AttnSmem sm;
  const int v = blockIdx.z;
  const int slot = b.seq.lane_slot[v];
  AttnArgs a = a0;
  a.qkv = a0.qkv + (size_t)v * b.qkv_stride;
  if (b.page_table) {
    a.pages = b.page_table + (size_t)slot * b.max_pages;
  } else {
    a.kc = reinterpret_cast<char*>(a0.kc) + (size_t)slot * b.kv_slot_bytes;
    a.vc = reinterpret_cast<char*>(a0.vc) + (size_t)slot * b.kv_slot_bytes;
  }
  a.pos = b.seq.pos + slot;
  a.pm = a0.pm + (size_t)v * b.part_stride;
  a.pz = a0.pz + (size_t)v * b.part_stride;
  a.po = a0.po + (size_t)v * b.part_stride * kHeadDim;
  a.out = a0.out + (size_t)v * b.out_stride;
  a.counters = a0.counters + (size_t)v * 64;
  if (b.seq.chunk) {
    a.pos_off = v;
    a.appended = 1;
  }
  attn_run<KVT>(a, blockIdx.x, gridDim.x, pdl, sm);
}

// One warp per (lane, KV head): RoPE(k) and v of position pos + lane into
// the cache (rope_lane4 / kv_cvt, as the attention item appends them).
template <typename KVT>
__global__ void kv_append_batch_kernel(AttnArgs a0, AttnBatch b) {
  const int v = blockIdx.x, lane = threadIdx.x & 31;
  const int slot = b.seq.lane_slot[v];
  const int pos = b.seq.pos[slot] + v;
  const int hd = kHeadDim, kvd = a0.nkv * hd;
  const uint32_t* pages = b.page_table ? b.page_table + (size_t)slot * b.max_pages : nullptr;
  char* kb = reinterpret_cast<char*>(a0.kc) + (b.page_table ? 0 : (size_t)slot * b.kv_slot_bytes);
  char* vb = reinterpret_cast<char*>(a0.vc) + (b.page_table ? 0 : (size_t)slot * b.kv_slot_bytes);
  const float* qkv = a0.qkv + (size_t)v * b.qkv_stride;
  const size_t row = kv_row(pages, pos);
  float cj[4], sj[4];
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const int j = (4 * lane + c) & (hd / 2 - 1);
    cj[c] = __ldg(a0.cosT + (size_t)pos * hd + j);
    sj[c] = __ldg(a0.sinT + (size_t)pos * hd + j);
  }
  for (int kvh = threadIdx.x >> 5; kvh < a0.nkv; kvh += blockDim.x >> 5) {
    const float4 kx = rope_lane4(
        __ldcg(reinterpret_cast<const float4*>(qkv + a0.nh * hd + kvh * hd + 4 * lane)), cj, sj,
        a0.kv_f16, false);
    const float4 vr =
        __ldcg(reinterpret_cast<const float4*>(qkv + a0.nh * hd + kvd + kvh * hd + 4 * lane));
    KVT* kw = reinterpret_cast<KVT*>(kb) + row * kvd + kvh * hd + 4 * lane;
    KVT* vw = reinterpret_cast<KVT*>(vb) + row * kvd + kvh * hd + 4 * lane;
    kw[0] = kv_cvt<KVT>(kx.x); kw[1] = kv_cvt<KVT>(kx.y); kw[2] = kv_cvt<KVT>(kx.z); kw[3] = kv_cvt<KVT>(kx.w);
    vw[0] = kv_cvt<KVT>(vr.x); vw[1] = kv_cvt<KVT>(vr.y); vw[2] = kv_cvt<KVT>(vr.z); vw[3] = kv_cvt<KVT>(vr.w);
  }
}

void kv_append_batch(const AttnArgs& a, const AttnBatch& b, int lanes, cudaStream_t st) {
  if (a.kv_f16)
    kv_append_batch_kernel<__half><<<lanes, 32 * std::min(a.nkv, 32), 0, st>>>(a, b);
  else
    kv_append_batch_kernel<float><<<lanes, 32 * std::min(a.nkv, 32), 0, st>>>(a, b);
}

void attn_batch(const AttnArgs& a, const AttnBatch& b, int lanes, cudaStream_t st, bool pdl) {
  const dim3 grid(attn_ctas(a, lanes), 1, lanes);
  if (a.kv_f16)
    blaunch(attn_batch_kernel<__half>, grid, dim3(kAttnWarps * 32), 0, st, pdl, a, b, (int)pdl);
  else
    blaunch(attn_batch_kernel<float>, grid, dim3(kAttnWarps * 32), 0, st, pdl, a, b, (int)pdl);
}

// ----------------------------------------------------------- LoRA A
__global__ void lora_a_batch_kernel(BatchSrc b, int K, const LoraMod* mods, float* d, int dstride,
                                    int pdl) {
  __shared__ float sred[32];
  if (pdl) pdl_wait();
  const int m = blockIdx.y, r = blockIdx.x, v = blockIdx.z;
  const LoraMod md = mods[m];
  if (r >= md.rank || !md.A) return;
  XSrc s = lane_src(b, v);
  s.hidden_out = nullptr;
  XCtx c;
  setup_x(s, K, c, sred);
  float acc = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x)
    acc = __fadd_rn(acc, __fmul_rn(xval(c, k), md.A[(size_t)r * K + k]));
  acc = block_sum(acc, sred);
  if (threadIdx.x == 0) d[(size_t)v * dstride + m * kMaxRank + r] = acc;
}

void lora_a_batch(const BatchSrc& s, int K, const LoraMod* mods, int nmods, int max_rank, float* d,
                  int dstride, int lanes, cudaStream_t st, bool pdl) {
  if (max_rank <= 0) return;
  blaunch(lora_a_batch_kernel, dim3(max_rank, nmods, lanes), dim3(kCtaThreads), 0, st, pdl, s, K,
          mods, d, dstride, (int)pdl);
}

__global__ void lora_b_batch_kernel(BatchEpi be, int rows, float* out, int pdl) {
  if (pdl) pdl_wait();
  const int v = blockIdx.y;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= rows) return;
  Epi e = be.e;
  e.lora_d += (size_t)v * be.dstride;
  float L;
  if (e.mode == EPI_SILU) {
    L = n < e.N ? lora_dot(e, 0, n, e.N) : lora_dot(e, 1, n - e.N, e.N);
  } else {  // the module split of epilogue_row
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
    L = lora_dot(e, m, nm, Nm);
  }
  out[(size_t)v * be.lstride + n] = L;
}

void lora_b_batch(const BatchEpi& be, int rows, int lanes, float* out, cudaStream_t st, bool pdl) {
  blaunch(lora_b_batch_kernel, dim3((rows + 255) / 256, lanes), dim3(256), 0, st, pdl, be, rows, out,
          (int)pdl);
}

// ----------------------------------------------------------- step end
__global__ void batch_advance_kernel(SeqTable seq, const uint32_t* choice, int lanes,
                                     uint32_t* out, int* step_ctr) {
  const int v = threadIdx.x;
  const int step = *step_ctr;
  if (seq.chunk) {  // chunked prefill: the slot moves on by the chunk
    if (v == 0) seq.pos[seq.lane_slot[0]] += lanes;
    return;
  }
  if (v < lanes) {
    const int s = seq.lane_slot[v];
    const int p = seq.pos[s];
    uint32_t* ids = seq.ids + (size_t)s * seq.slot_ctx;
    if (p + 1 >= seq.len[s]) {  // past the known ids: append this step's token
      const uint32_t c = choice[v];
      ids[p + 1] = c < seq.vocab ? c : 0u;  // the next step embeds this id
      seq.len[s] = p + 2;
    }
    out[(size_t)step * lanes + v] = ids[p + 1];
    seq.pos[s] = p + 1;
  }
  __syncthreads();
  if (v == 0) *step_ctr = step + 1;
}

void batch_advance(SeqTable seq, const uint32_t* choice, int lanes, uint32_t* out, int* step_ctr,
                   cudaStream_t st) {
  batch_advance_kernel<<<1, 32, 0, st>>>(seq, choice, lanes, out, step_ctr);
}

}  // namespace eg
