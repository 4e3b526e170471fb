// eg_fused.cu -- persistent decode: n tokens of runtime.js:1466-1571 (plus
// EMBED_BUF in front and ARGMAX behind) in ONE cooperative launch.
//
// Grid = one CTA per SM, the warp roles of the streaming GEMVs
// (eg_stream.cuh): warps 0-15 consume, warp 16 produces, warp 17 runs the
// epilogues.  A token is a fixed sequence of phases -- per layer QKV, ATTN,
// O, GATE_UP, DOWN, then the LM head -- separated by grid barriers; every
// GEMV phase gives each CTA a contiguous range of the matrix's 16-row tiles.
//
// The producer walks the CTA's weight runs of the whole launch (every phase
// of every token) in order and streams them through one shared-memory ring,
// one cp.async.bulk per stage.  The weights do not depend on activations, so
// it never waits for a grid barrier: HBM keeps streaming the next phases'
// weights while the consumers wait at a barrier, stage activations or run
// attention.  At the end of a GEMV phase the epilogue warp, once its last
// tile's outputs are written, arrives at the grid barrier itself with one
// release reduction (red.release.gpu, no separate fence); consumer thread 0
// polls it (ld.acquire.gpu).  Activations written before a barrier are read after it
// with ld.global.cg, so no stale L1 line is seen inside the launch.  After
// the LM head every CTA reduces the CTAs' argmax candidates itself, so the
// next token's embedding needs no further barrier.  Every wait is bounded:
// on timeout the waiter records an error word, the others see it and leave,
// and the host reports EG_ERR_DEVICE.
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>

#include "eg_fused.h"
#include "eg_stream.cuh"

namespace eg {

constexpr int kFusedWarps = 16;  // consumer warps (attention items need 512 threads)
constexpr int kFusedThreads = kFusedWarps * 32 + 64;
constexpr int kFStageBytes = 34816;  // 32 int4 blocks, 16 gate/up blocks, 17 int8 blocks
constexpr int kFMaxStages = 6;
constexpr int kFBarBytes = 256;      // ring + tile mbarriers
constexpr unsigned long long kBarrierTimeoutNs = 2000000000ull;  // 2 s

enum { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4 };

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool lm_runs(const FusedArgs& a, int tok) {
  return a.lm_every || tok == a.n_tokens - 1;
}

__device__ __forceinline__ void tile_range(int tiles, int& t_lo, int& t_hi) {
  t_lo = (int)((long long)tiles * blockIdx.x / gridDim.x);
  t_hi = (int)((long long)tiles * (blockIdx.x + 1) / gridDim.x);
}

// One GEMV phase of this CTA: the matrix, its tile range and ring geometry.
struct Run {
  const unsigned char* src;  // first block of the CTA's range
  int t_lo, t_hi, gpr, blk, cap;
};

__device__ __forceinline__ Run run_of(const FusedArgs& a, const FusedLayer& l, int ph) {
  Run r;
  int N, K, R = 1;
  const unsigned char* w;
  switch (ph) {
    case PH_QKV: w = l.qkv; N = a.QD + 2 * a.KVD; K = a.H; break;
    case PH_O: w = l.o; N = a.H; K = a.QD; break;
    case PH_GU: w = l.gu; N = a.I; K = a.H; R = 2; break;
    default: w = l.d; N = a.H; K = a.I; break;
  }
  tile_range((N + 15) / 16, r.t_lo, r.t_hi);
  r.gpr = K / kGroup;
  r.blk = q4_block_bytes(R);
  r.cap = kFStageBytes / r.blk;
  r.src = w + (size_t)r.t_lo * r.gpr * r.blk;
  return r;
}

__device__ __forceinline__ Run run_lm(const FusedArgs& a) {
  Run r;
  tile_range((a.V + 15) / 16, r.t_lo, r.t_hi);
  r.gpr = (a.H + kGroup - 1) / kGroup;
  r.blk = kQ8Block;
  r.cap = kFStageBytes / kQ8Block;
  r.src = a.lm + (size_t)r.t_lo * r.gpr * kQ8Block;
  return r;
}

// ---------------------------------------------------------------- barrier
// Monotonic arrival counter: the k-th barrier completes when the counter
// reaches k * gridDim.x, one arrival per CTA and phase.  Called by all
// consumer threads; in a GEMV phase (`epi`) the CTA's epilogue warp has
// arrived (epi_arrive), otherwise thread 0 arrives; thread 0 polls, then
// publishes the passed phase count for the epilogue warp.  Returns false,
// uniformly, when the launch is being abandoned.
__device__ bool phase_barrier(const FusedArgs& a, unsigned& epoch, volatile int* passed, bool epi,
                              int* s_ok, int prof_ph) {
  constexpr int NT = kFusedWarps * 32;
  bar_sync_n<NT>();
  if (threadIdx.x == 0) {
    int ok = 1;
    if (a.prof && prof_ph >= 0 && !epi) atomicMax(a.prof + 2 * prof_ph + 1, gtime());
    epoch += 1;
    const unsigned target = epoch * gridDim.x;
    // GEMV phases: this CTA's epilogue warp arrived after writing its
    // outputs; other phases (attention): thread 0 arrives for the consumers,
    // whose writes the bar.sync above ordered before this release
    if (!epi) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
    const unsigned long long t0 = gtime();
    for (long long spins = 0; ok; spins++) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.bar) : "memory");
      if (v >= target) break;
      if ((spins & 255) == 255) {
        if (err_set(a.err)) {
          ok = 0;
        } else if (gtime() - t0 > kBarrierTimeoutNs) {
          atomicExch(a.err, 1);
          ok = 0;
        }
      }
    }
    if (err_set(a.err)) ok = 0;
    *s_ok = ok;
    *passed = (int)epoch;  // the epilogue warp may arrive for the next phase
  }
  bar_sync_n<NT>();
  return *s_ok != 0;
}

// The epilogue warp's grid-barrier arrival for launch phase q (0-based),
// once its outputs of the phase are written: a release reduction by lane 0
// after __syncwarp covers the whole warp's stores (no separate fence).  It
// waits until the barrier of phase q - 1 has passed in this CTA, so a CTA
// with no tiles in phase q cannot arrive before the others finished q - 1.
__device__ __forceinline__ bool epi_arrive(const FusedArgs& a, volatile int* passed, int q,
                                           int prof_ph) {
  __syncwarp();
  bool ok = true;
  if ((threadIdx.x & 31) == 0) {
    const unsigned long long t0 = gtime();
    for (long long spins = 0; *passed < q; spins++)
      if ((spins & 255) == 255 && (err_set(a.err) || gtime() - t0 > kBarrierTimeoutNs)) {
        atomicExch(a.err, 1);
        ok = false;
        break;
      }
    if (a.prof && prof_ph >= 0) atomicMax(a.prof + 2 * prof_ph + 1, gtime());
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
  }
  return __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
}

// ---------------------------------------------------------------- the kernel
// 18 warps: the register file is allocated to them in 4-warp units (20
// warps' worth), so a thread gets at most 96 registers.
template <typename KVT>
__global__ void __maxnreg__(96) fused_decode_kernel(FusedArgs a, int xbytes, int kFStages) {
  constexpr int NT = kFusedWarps * 32;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float sred[32];
  __shared__ TileRed<kFusedWarps, 1> red1;
  __shared__ TileRed<kFusedWarps, 2> red2;
  __shared__ AttnSmem asm_;
  __shared__ int bar_passed;  // launch phases whose grid barrier this CTA passed
  __shared__ int s_ok;
  __shared__ uint32_t s_id;
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm);
  uint64_t* empty = full + kFStages;
  uint64_t* tile_full = empty + kFStages;
  uint64_t* tile_free = tile_full + 2;
  unsigned char* xreg = dsm + kFBarBytes;  // activation digit planes
  unsigned char* ring = xreg + xbytes;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int L = a.layers_n;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kFStages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kFusedWarps);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tile_full[i], kFusedWarps);
      mbar_init(&tile_free[i], 1);
    }
    bar_passed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  RingPos rp = {0, 0};
  int tj = 0;
  const int phs[4] = {PH_QKV, PH_O, PH_GU, PH_DOWN};

  if (warp == kFusedWarps) {  // ---------------------------------------- producer
    int issued = 0;
    bool ok = true;
    for (int tok = 0; tok < a.n_tokens && ok; tok++) {
      for (int li = 0; li < L && ok; li++)
        for (int k = 0; k < 4 && ok; k++) {
          const Run r = run_of(a, a.layers[li], phs[k]);
          ok = ring_produce(ring, full, empty, kFStages, kFStageBytes, r.src,
                            (r.t_hi - r.t_lo) * r.gpr, r.cap, r.blk, rp, issued, a.err, lane);
        }
      if (ok && lm_runs(a, tok)) {
        const Run r = run_lm(a);
        ok = ring_produce(ring, full, empty, kFStages, kFStageBytes, r.src,
                          (r.t_hi - r.t_lo) * r.gpr, r.cap, r.blk, rp, issued, a.err, lane);
      }
    }
    ring_drain(full, kFStages, rp, issued);
    return;
  }

  if (warp == kFusedWarps + 1) {  // ------------------------------------ epilogue
    int q0 = 0;  // launch phase index of this token's first phase
    for (int tok = 0; tok < a.n_tokens; tok++) {
      for (int li = 0; li < L; li++) {
        const FusedLayer& l = a.layers[li];
        for (int k = 0; k < 4; k++) {
          const int ph = phs[k];
          const Run r = run_of(a, l, ph);
          Epi e = {};
          bool ok;
          if (ph == PH_GU) {
            e.mode = EPI_SILU;
            e.y = a.tmp;
            e.N = a.I;
            ok = epilogue_q4_run<kFusedWarps, 2>(e, r.t_lo, r.t_hi, red2, tile_full, tile_free, tj, false, a.err);
          } else {
            if (ph == PH_QKV) {  // q/k/v rows + bias
              e.mode = EPI_STORE;
              e.y = a.qkv;
              e.bias = l.qkv_b;
              e.N = a.QD + 2 * a.KVD;
            } else {  // GEMV4_ADD: hidden += W x (runtime.js:1531, :1566)
              e.mode = EPI_ADD;
              e.y = a.hidden;
              e.N = a.H;
            }
            e.split1 = e.split2 = e.N;
            ok = epilogue_q4_run<kFusedWarps, 1>(e, r.t_lo, r.t_hi, red1, tile_full, tile_free, tj, false, a.err);
          }
          if (!ok) return;
          const int q = q0 + 5 * li + ph;
          if (!epi_arrive(a, &bar_passed, q, tok == 0 ? 5 * li + ph : -1)) return;
        }
      }
      if (lm_runs(a, tok)) {
        const Run r = run_lm(a);
        float bv = -1e30f;
        uint32_t bi = 0xffffffffu;
        if (!epilogue_q8_run<kFusedWarps>(a.emb_s, a.logits, a.V, r.t_lo, r.t_hi, red1, tile_full, tile_free, tj,
                             bv, bi, a.err))
          return;
        if (lane == 0) {
          a.cand_v[blockIdx.x] = bv;
          a.cand_i[blockIdx.x] = bi;
        }
        if (!epi_arrive(a, &bar_passed, q0 + 5 * L, tok == 0 ? 5 * L : -1)) return;
      }
      q0 += 5 * L + (lm_runs(a, tok) ? 1 : 0);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  unsigned epoch = 0;
  bool dead = false;
  uint2* xb = reinterpret_cast<uint2*>(xreg);
  // the first input token is ids[start_pos]; later ones come from the
  // previous LM head (greedy) or from ids[] (prefill)
  bool have_id = false;
  uint32_t next_id = 0;
  for (int tok = 0; tok < a.n_tokens; tok++) {
    const int pos = a.start_pos + tok;
    for (int li = 0; li < L; li++) {
      const FusedLayer& l = a.layers[li];
      const int pb = tok == 0 ? li * 5 : -1000;  // profile index base (token 0)
      const bool prof0 = a.prof && tok == 0 && blockIdx.x == 0 && threadIdx.x == 0;
      // ---- QKV: (embed +) RMSNorm prologue, q/k/v rows + bias
      if (prof0) a.prof[2 * pb] = gtime();
      {
        const Run r = run_of(a, l, PH_QKV);
        const int gpr = a.H / kGroup;
        int* xcor = reinterpret_cast<int*>(xb + (size_t)gpr * 64);
        int* xf = xcor + 2 * gpr;
        XSrc x = {};
        x.mode = li == 0 ? X_EMBED_RMS : X_RMS;
        x.x = a.hidden;
        x.norm_g = l.in_norm;
        x.eps = a.eps;
        x.f16 = a.f16;
        x.emb_w = a.emb_w;
        x.emb_s = a.emb_s;
        x.ids = a.ids;
        x.fixed_pos = pos;
        x.use_fixed_id = have_id ? 1 : 0;
        x.fixed_id = next_id;
        x.hidden_out = a.hidden;
        if (r.t_lo < r.t_hi) {
          stage_xd<1, true, NT>(x, a.H, xb, xcor, xf, sred, 0);
          consume_q4_run<kFusedWarps, 1>(ring, full, empty, kFStages, kFStageBytes, r.cap, r.t_lo, r.t_hi, r.gpr,
                            xb, xcor, xf, red1, tile_full, tile_free, rp, tj, dead, a.err);
        }
      }
      if (!phase_barrier(a, epoch, &bar_passed, true, &s_ok, tok == 0 ? pb : -1)) return;
      // ---- attention: RoPE, KV append, split partials, merge
      if (prof0) a.prof[2 * (pb + 1)] = gtime();
      {
        AttnArgs at = {};
        at.qkv = a.qkv;
        at.kc = l.kc;
        at.vc = l.vc;
        at.cosT = a.cosT;
        at.sinT = a.sinT;
        at.pos = nullptr;
        at.fixed_pos = pos;
        at.nh = a.nh;
        at.nkv = a.nkv;
        at.max_splits = a.max_splits;
        at.ctx_bound = pos + 1;
        at.kv_f16 = a.f16;
        at.chunk = a.attn_chunk;
        at.pm = a.pm;
        at.pz = a.pz;
        at.po = a.po;
        at.out = a.attn;
        at.counters = a.attn_counters;
        attn_run<KVT, false>(at, blockIdx.x, gridDim.x, 0, asm_);
      }
      if (!phase_barrier(a, epoch, &bar_passed, false, &s_ok, tok == 0 ? pb + 1 : -1)) return;
      // ---- O projection + residual
      if (prof0) a.prof[2 * (pb + 2)] = gtime();
      {
        const Run r = run_of(a, l, PH_O);
        const int gpr = a.QD / kGroup;
        int* xcor = reinterpret_cast<int*>(xb + (size_t)gpr * 64);
        int* xf = xcor + 2 * gpr;
        XSrc x = {};
        x.mode = X_PLAIN;
        x.x = a.attn;
        if (r.t_lo < r.t_hi) {
          stage_xd<1, false, NT>(x, a.QD, xb, xcor, xf, sred, 0);
          consume_q4_run<kFusedWarps, 1>(ring, full, empty, kFStages, kFStageBytes, r.cap, r.t_lo, r.t_hi, r.gpr,
                            xb, xcor, xf, red1, tile_full, tile_free, rp, tj, dead, a.err);
        }
      }
      if (!phase_barrier(a, epoch, &bar_passed, true, &s_ok, tok == 0 ? pb + 2 : -1)) return;
      // ---- gate/up + SiLU
      if (prof0) a.prof[2 * (pb + 3)] = gtime();
      {
        const Run r = run_of(a, l, PH_GU);
        const int gpr = a.H / kGroup;
        int* xcor = reinterpret_cast<int*>(xb + (size_t)gpr * 64);
        int* xf = xcor + 2 * gpr;
        XSrc x = {};
        x.mode = X_RMS;
        x.x = a.hidden;
        x.norm_g = l.post_norm;
        x.eps = a.eps;
        x.f16 = a.f16;
        if (r.t_lo < r.t_hi) {
          stage_xd<1, true, NT>(x, a.H, xb, xcor, xf, sred, 0);
          consume_q4_run<kFusedWarps, 2>(ring, full, empty, kFStages, kFStageBytes, r.cap, r.t_lo, r.t_hi, r.gpr,
                            xb, xcor, xf, red2, tile_full, tile_free, rp, tj, dead, a.err);
        }
      }
      if (!phase_barrier(a, epoch, &bar_passed, true, &s_ok, tok == 0 ? pb + 3 : -1)) return;
      // ---- down projection + residual
      if (prof0) a.prof[2 * (pb + 4)] = gtime();
      {
        const Run r = run_of(a, l, PH_DOWN);
        const int gpr = a.I / kGroup;
        int* xcor = reinterpret_cast<int*>(xb + (size_t)gpr * 64);
        int* xf = xcor + 2 * gpr;
        XSrc x = {};
        x.mode = X_PLAIN;
        x.x = a.tmp;
        if (r.t_lo < r.t_hi) {
          stage_xd<3, false, NT>(x, a.I, xb, xcor, xf, sred, 0);
          consume_q4_run<kFusedWarps, 1>(ring, full, empty, kFStages, kFStageBytes, r.cap, r.t_lo, r.t_hi, r.gpr,
                            xb, xcor, xf, red1, tile_full, tile_free, rp, tj, dead, a.err);
        }
      }
      if (!phase_barrier(a, epoch, &bar_passed, true, &s_ok, tok == 0 ? pb + 4 : -1)) return;
    }
    // ---- LM head (int8) + argmax + token advance
    if (!lm_runs(a, tok)) {
      have_id = false;  // the next input is ids[pos + 1] (prefill)
      continue;
    }
    const int pl = 5 * L;
    if (a.prof && tok == 0 && blockIdx.x == 0 && threadIdx.x == 0) a.prof[2 * pl] = gtime();
    {
      const Run r = run_lm(a);
      uint32_t* xb8 = reinterpret_cast<uint32_t*>(xreg);
      float* xm8 = reinterpret_cast<float*>(xb8 + (size_t)r.gpr * 128);
      XSrc x = {};
      x.mode = X_RMS;
      x.x = a.hidden;
      x.norm_g = a.final_norm;
      x.eps = a.eps;
      x.f16 = a.f16;
      if (r.t_lo < r.t_hi) {
        stage_xd8<1, true, NT>(x, a.H, r.gpr * kGroup, xb8, xm8, sred, 0);
        consume_q8_run<kFusedWarps>(ring, full, empty, kFStages, kFStageBytes, r.cap, r.t_lo, r.t_hi, r.gpr, xb8,
                       xm8, red1, tile_full, tile_free, rp, tj, dead, a.err);
      }
    }
    if (!phase_barrier(a, epoch, &bar_passed, true, &s_ok, tok == 0 ? pl : -1)) return;
    if (a.greedy) {
      // every CTA merges the candidates (ARGMAX, kernels.js:771-784); ties
      // to the lower index
      if (warp == 0) {
        float v = -1e30f;
        uint32_t id = 0xffffffffu;
        for (int b = lane; b < (int)gridDim.x; b += 32) {
          const float cv = __ldcg(a.cand_v + b);
          const uint32_t ci = __ldcg(a.cand_i + b);
          if (beats(cv, ci, v, id)) {
            v = cv;
            id = ci;
          }
        }
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
          s_id = id;
          if (blockIdx.x == 0) {
            *a.amax = id;
            a.ids[pos + 1] = id;
            a.out_ids[tok] = id;
          }
        }
      }
      bar_sync_n<NT>();
      next_id = s_id;
      have_id = true;
      // the candidates are rewritten by the next LM head only after many more
      // grid barriers, so every CTA has read them by then
    } else {
      have_id = false;
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) a.state_pos[0] = a.start_pos + a.n_tokens;
}

// Activation region: the largest staged vector (int4 digit planes of H, QD
// or I; int8 digit planes of H).
static int fused_stages() {
  const char* v = getenv("EG_FUSED_STAGES");  // tuning only
  const int n = v ? atoi(v) : 4;
  return std::max(2, std::min(kFMaxStages, n));
}

static int fused_xbytes(const FusedArgs& a) {
  const int q4 = std::max(std::max(a.H, a.QD), a.I) / kGroup * (512 + 16);
  const int q8 = (a.H + kGroup - 1) / kGroup * (512 + 8);
  return (std::max(q4, q8) + 127) & ~127;
}

int fused_smem_bytes(const FusedArgs& a) {
  return kFBarBytes + fused_xbytes(a) + fused_stages() * kFStageBytes;
}

cudaError_t fused_decode(const FusedArgs& a, cudaStream_t st) {
  const int smem = fused_smem_bytes(a);
  const int xbytes = fused_xbytes(a);
  const int stages = fused_stages();
  void (*k)(FusedArgs, int, int) = a.f16 ? fused_decode_kernel<__half> : fused_decode_kernel<float>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kFusedThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) {
    cudaFuncAttributes fa = {};
    cudaFuncGetAttributes(&fa, k);
    fprintf(stderr,
            "fused_decode: no CTA fits an SM: %d regs/thread x %d threads, %zu B static + %d B "
            "dynamic shared (max dynamic %d), %zu B local\n",
            fa.numRegs, kFusedThreads, fa.sharedSizeBytes, smem, fa.maxDynamicSharedSizeBytes,
            fa.localSizeBytes);
    return cudaErrorCooperativeLaunchTooLarge;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count());
  cfg.blockDim = dim3(kFusedThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, a, xbytes, stages);
}

}  // namespace eg
