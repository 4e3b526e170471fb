// eg_kernels.cu -- sm_100a kernels for the Emberglass batch-1 decode path.
//
// GEMVs (int4 layers and the int8 LM head): the weights are repacked once,
// at finalize, from the reference's packed rows (quantize.js:28-111) into a
// "stream" layout of 16-row x 128-k blocks stored as tensor-core A
// fragments, tile-major, so that any contiguous run of blocks is one
// contiguous byte range.  One persistent-style CTA per SM streams its run of
// blocks through a shared-memory ring with one cp.async.bulk per stage (a
// producer warp), 16 consumer warps multiply them with the integer tensor
// path (m16n8k32 u8.s8 for int4, s8.s8 for int8) against the activation held
// as four base-256 digit planes of a per-group fixed-point value (exact
// integer dots per 128-wide group, scaled in f32), and an epilogue warp
// applies the scale / residual / bias / SiLU / LoRA / argmax epilogue.
//
// Attention: one CTA per (query head, split of <= 256 keys) with the K/V rows
// in registers (ATTN_PARTIAL/ATTN_COMBINE, kernels.js:258-388), RoPE
// (ROPE_QK, kernels.js:205-257) and the KV append (runtime.js:1509-1514)
// fused in.
#include <float.h>
#include <math.h>

#include <stdlib.h>

#include <algorithm>

#include "eg_common.cuh"
#include "eg_device.cuh"
#include "eg_batch.h"
#include "eg_kernels.h"
#include "eg_stream.cuh"

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
// Streaming int4 GEMV (GEMV4 / GEMV4_ADD / QKV / GATE_UP_SILU_GEMV4,
// kernels.js:884-1072) over the stream layout (q4_to_stream)
// ======================================================================
// One CTA per SM: warps 0-15 consume, warp 16 produces, warp 17 runs the
// epilogues (eg_stream.cuh).  The tiles are split into contiguous ranges,
// one per CTA; every tile is finished inside one CTA, so the epilogue needs
// no cross-CTA combine (a memory fence under a saturated memory system costs
// microseconds).  Shared memory: barriers | activation digit planes | ring.
struct G4Args {
  const unsigned char* ws;  // stream layout
  const unsigned char* pf;  // optional L2 prefetch (GemvWork)
  size_t pf_bytes;
  int N, K;
  XSrc x;
  Epi e;
  int* err;
  int stages, stage_bytes, cap, xs_off, ring_off;
  int pdl;
};

// Barrier block at the start of the dynamic shared memory: 2 * stages ring
// mbarriers + 2 tile_full + 2 tile_free (stages <= 8).
constexpr int kBarBytes = 256;

// 16 consumer warps + producer + epilogue.  (8 consumer warps in ~105 KB, so
// that the next kernel's CTA fits beside this one under PDL, measured slower:
// the overlap gained less than the halved consumer group lost.)
constexpr int kOpWarps = 16;
constexpr int kOpThreads = kOpWarps * 32 + 64;

__device__ __forceinline__ void init_ring_barriers(uint64_t* full, uint64_t* empty,
                                                   uint64_t* tile_full, uint64_t* tile_free,
                                                   int stages) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kOpWarps);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tile_full[i], kOpWarps);
      mbar_init(&tile_free[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
}

template <int R, int MAXU, bool NORM>
__global__ void __launch_bounds__(kOpThreads, 1) gemv_q4_kernel(G4Args p) {
  constexpr int NT = kOpWarps * 32;
  extern __shared__ __align__(128) unsigned char g4_smem[];
  __shared__ float sred[32];
  __shared__ TileRed<kOpWarps, R> red;
  uint64_t* full = reinterpret_cast<uint64_t*>(g4_smem);
  uint64_t* empty = full + p.stages;
  uint64_t* tile_full = empty + p.stages;
  uint64_t* tile_free = tile_full + 2;
  const int gpr = p.K / kGroup;
  uint2* xb = reinterpret_cast<uint2*>(g4_smem + p.xs_off);  // [gpr][4][4][4]
  int* xcor = reinterpret_cast<int*>(xb + (size_t)gpr * 64);   // [gpr][2]
  int* xf = xcor + 2 * gpr;
  unsigned char* ring = g4_smem + p.ring_off;
  const int tiles = (p.N + 15) / 16;
  const int t_lo = (int)((long long)tiles * blockIdx.x / gridDim.x);
  const int t_hi = (int)((long long)tiles * (blockIdx.x + 1) / gridDim.x);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  init_ring_barriers(full, empty, tile_full, tile_free, p.stages);
  RingPos rp = {0, 0};
  int tj = 0;
  if (warp == kOpWarps) {  // producer: the weights need no wait
    int issued = 0;
    ring_produce(ring, full, empty, p.stages, p.stage_bytes,
                 p.ws + (size_t)t_lo * gpr * q4_block_bytes(R), (t_hi - t_lo) * gpr, p.cap,
                 q4_block_bytes(R), rp, issued, p.err, lane, p.pf, p.pf_bytes);
    ring_drain(full, p.stages, rp, issued);
    return;
  }
  if (warp == kOpWarps + 1) {  // epilogue: residuals come from earlier kernels
    if (p.pdl) pdl_wait();
    epilogue_q4_run<kOpWarps, R>(p.e, t_lo, t_hi, red, tile_full, tile_free, tj, true, p.err);
    return;
  }
  stage_xd<MAXU, NORM, NT>(p.x, p.K, xb, xcor, xf, sred, p.pdl);
  // the next kernel may start once this one's predecessors are complete (the
  // attention kernel relies on that to read the position early)
  if (p.pdl) pdl_launch_dependents();
  bool dead = false;
  consume_q4_run<kOpWarps, R>(ring, full, empty, p.stages, p.stage_bytes, p.cap, t_lo, t_hi, gpr, xb, xcor,
                    xf, red, tile_full, tile_free, rp, tj, dead, p.err);
}

// Shared-memory plan of one launch (bytes): barriers, x digit planes + group
// words, then the ring; ~150 KB so an attention CTA fits beside it under PDL.
struct G4Plan {
  int stages, stage_bytes, cap, xs_off, ring_off, smem;
};
static G4Plan g4_plan(int R, int K) {
  G4Plan q;
  const int gpr = K / kGroup;
  q.cap = 32 / R;  // blocks per stage: 34 KB
  q.stage_bytes = q.cap * q4_block_bytes(R);
  q.xs_off = kBarBytes;
  q.ring_off = (q.xs_off + gpr * (512 + 16) + 127) & ~127;
  const int budget = 150 * 1024;
  q.stages = std::max(2, std::min(8, (budget - q.ring_off) / q.stage_bytes));
  q.smem = q.ring_off + q.stages * q.stage_bytes;
  return q;
}

int gemv_q4_ctas() { return sm_count(); }

template <int R, int MAXU, bool NORM>
static void gemv_q4_go(const G4Args& a0, const G4Plan& q, cudaStream_t st, bool pdl) {
  G4Args a = a0;
  a.stages = q.stages;
  a.stage_bytes = q.stage_bytes;
  a.cap = q.cap;
  a.xs_off = q.xs_off;
  a.ring_off = q.ring_off;
  a.pdl = pdl ? 1 : 0;
  const int P = std::min(gemv_q4_ctas(), (a.N + 15) / 16);
  auto k = gemv_q4_kernel<R, MAXU, NORM>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, q.smem);
  launch(k, dim3(P), dim3(kOpThreads), (size_t)q.smem, st, pdl, a);
}

template <int R>
static void gemv_q4_r(const G4Args& a, cudaStream_t st, bool pdl) {
  const G4Plan q = g4_plan(R, a.K);
  const int u = (a.K / 8 + kOpWarps * 32 - 1) / (kOpWarps * 32);  // units per thread
  // MAXU >= u: every unit of the vector is staged (K <= 12288)
  if (a.x.mode != X_PLAIN) {  // RMSNorm holds the whole vector in registers
    if (u <= 1) gemv_q4_go<R, 1, true>(a, q, st, pdl);
    else if (u <= 3) gemv_q4_go<R, 3, true>(a, q, st, pdl);
    else gemv_q4_go<R, 6, true>(a, q, st, pdl);
  } else if (u <= 1) {
    gemv_q4_go<R, 1, false>(a, q, st, pdl);
  } else if (u <= 3) {
    gemv_q4_go<R, 3, false>(a, q, st, pdl);
  } else {
    gemv_q4_go<R, 6, false>(a, q, st, pdl);
  }
}

void gemv_q4(const unsigned char* ws, int N, int K, const XSrc& x, const Epi& e, cudaStream_t st,
             bool pdl, const GemvWork& wk) {
  G4Args a = {};
  a.ws = ws;
  a.N = N;
  a.K = K;
  a.x = x;
  a.e = e;
  a.err = wk.err;
  a.pf = wk.pf;
  a.pf_bytes = wk.pf_bytes;
  if (e.mode == EPI_SILU)
    gemv_q4_r<2>(a, st, pdl);
  else
    gemv_q4_r<1>(a, st, pdl);
}

size_t q4_stream_bytes(int N, int K, int R) {
  return (size_t)((N + 15) / 16) * (K / kGroup) * q4_block_bytes(R);
}

// One thread per 16-byte fragment word of the stream layout; rows past N
// are zero.  Threads past the fragment words copy the scales instead.
__global__ void q4_to_stream_kernel(const uint32_t* __restrict__ w, const float* __restrict__ s,
                                    int N, int K, int R, unsigned char* __restrict__ out) {
  const int gpr = K / kGroup, tiles = (N + 15) / 16;
  const long long nfrag = (long long)tiles * gpr * R * 64;  // 16-byte words
  const long long nsc = (long long)tiles * gpr * R * 16;
  const long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (u < nfrag) {
    const int lane = (int)(u & 31), h = (int)((u >> 5) & 1);
    const long long q = u >> 6;  // (block, r)
    const int r = (int)(q % R);
    const long long b = q / R;
    const int G = (int)(b % gpr), tile = (int)(b / gpr);
    const int rt = tile * 16 + 8 * h + (lane >> 2);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (rt < N) {
      const size_t row = (size_t)rt + (size_t)r * N;
      // words t, 4+t, 8+t, 12+t of the group (the integer-MMA k order)
      const uint32_t* src = w + row * (K / 8) + 16 * G + (lane & 3);
      v = make_uint4(src[0], src[4], src[8], src[12]);
    }
    *reinterpret_cast<uint4*>(out + b * q4_block_bytes(R) + r * 1024 + h * 512 + lane * 16) = v;
  } else if (u < nfrag + nsc) {
    const long long v = u - nfrag;
    const int i = (int)(v & 15);
    const long long q = v >> 4;
    const int r = (int)(q % R);
    const long long b = q / R;
    const int G = (int)(b % gpr), tile = (int)(b / gpr);
    const int rt = tile * 16 + i;
    const float sv = rt < N ? s[((size_t)rt + (size_t)r * N) * gpr + G] : 0.f;
    // (row i, row i + 8) pairs: one 8-byte load per consumer lane
    reinterpret_cast<float*>(out + b * q4_block_bytes(R) + R * 1024)[r * 16 + (i & 7) * 2 + (i >> 3)] = sv;
  }
}

void q4_to_stream(const uint32_t* w, const float* s, int N, int K, int R, unsigned char* out,
                  cudaStream_t st) {
  const long long n = (long long)((N + 15) / 16) * (K / kGroup) * R * 80;
  q4_to_stream_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, s, N, K, R, out);
}

// ======================================================================
// int8 GEMV (tied LM head, GEMV kernels.js:20-59) + fused argmax tail
// ======================================================================
// Stream layout of an int8 matrix (q8_to_stream): blocks of 16 rows x 128 k
// (2 KB), tile-major, group-minor; inside a block [row half h][k half k2]
// [lane (gq, t)][16 bytes] = row 8h + gq, words 16 k2 + t + {0, 4, 8, 12} of
// the group, i.e. the m16n8k32 s8 A fragments of MMAs 2 k2 and 2 k2 + 1 with
// no unpacking.  The row scales stay a plain f32 array (applied after the
// row sum, as the reference does).
size_t q8_stream_bytes(int N, int K) {
  return (size_t)((N + 15) / 16) * ((K + kGroup - 1) / kGroup) * kQ8Block;
}

__global__ void q8_to_stream_kernel(const uint32_t* __restrict__ w, int N, int K,
                                    unsigned char* __restrict__ out) {
  const int gpr = (K + kGroup - 1) / kGroup, K4 = K / 4, tiles = (N + 15) / 16;
  const long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // 16-byte word
  if (u >= (long long)tiles * gpr * (kQ8Block / 16)) return;
  const int lane = (int)(u & 31), k2 = (int)((u >> 5) & 1), h = (int)((u >> 6) & 1);
  const long long b = u >> 7;
  const int G = (int)(b % gpr), tile = (int)(b / gpr);
  const int row = tile * 16 + 8 * h + (lane >> 2);
  uint32_t v[4] = {0u, 0u, 0u, 0u};
  if (row < N)
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int word = G * 32 + 16 * k2 + (lane & 3) + 4 * j;
      if (word < K4) v[j] = w[(size_t)row * K4 + word];
    }
  *reinterpret_cast<uint4*>(out + b * kQ8Block + h * 1024 + k2 * 512 + lane * 16) =
      make_uint4(v[0], v[1], v[2], v[3]);
}

void q8_to_stream(const uint32_t* w, int N, int K, unsigned char* out, cudaStream_t st) {
  const long long n = (long long)((N + 15) / 16) * ((K + kGroup - 1) / kGroup) * (kQ8Block / 16);
  q8_to_stream_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, N, K, out);
}

struct Q8Args {
  const unsigned char* ws;  // stream layout
  const float* s;           // row scales
  int N, K;
  XSrc x;
  float* y;
  StepTail tail;
  int has_tail;
  int* err;
  int stages, stage_bytes, cap, xs_off, ring_off;
  int pdl;
};

// Same warp roles as gemv_q4_kernel.  With a tail, the CTAs' argmax
// candidates are merged by the last CTA to finish, which also advances the
// decode position (ARGMAX kernels.js:771-784, then decodeBatch's copy of
// s.amax into the id buffer, runtime.js:1783-1785).
template <int MAXU, bool NORM>
__global__ void __launch_bounds__(kOpThreads, 1) gemv_q8_kernel(Q8Args p) {
  constexpr int NT = kOpWarps * 32;
  extern __shared__ __align__(128) unsigned char g4_smem[];
  __shared__ float sred[32];
  __shared__ TileRed<kOpWarps, 1> red;
  uint64_t* full = reinterpret_cast<uint64_t*>(g4_smem);
  uint64_t* empty = full + p.stages;
  uint64_t* tile_full = empty + p.stages;
  uint64_t* tile_free = tile_full + 2;
  const int gpr = (p.K + kGroup - 1) / kGroup;
  uint32_t* xb = reinterpret_cast<uint32_t*>(g4_smem + p.xs_off);  // [gpr][4][4][4][2]
  float* xmul = reinterpret_cast<float*>(xb + (size_t)gpr * 128);  // [gpr][2]
  unsigned char* ring = g4_smem + p.ring_off;
  const int tiles = (p.N + 15) / 16;
  const int P = gridDim.x, c = blockIdx.x;
  const int t_lo = (int)((long long)tiles * c / P), t_hi = (int)((long long)tiles * (c + 1) / P);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  init_ring_barriers(full, empty, tile_full, tile_free, p.stages);
  RingPos rp = {0, 0};
  int tj = 0;
  if (warp == kOpWarps) {  // producer
    int issued = 0;
    ring_produce(ring, full, empty, p.stages, p.stage_bytes, p.ws + (size_t)t_lo * gpr * kQ8Block,
                 (t_hi - t_lo) * gpr, p.cap, kQ8Block, rp, issued, p.err, lane);
    ring_drain(full, p.stages, rp, issued);
    return;
  }
  if (warp == kOpWarps + 1) {  // epilogue
    float bv = -1e30f;
    uint32_t bi = 0xffffffffu;
    if (!epilogue_q8_run<kOpWarps>(p.s, p.y, p.N, t_lo, t_hi, red, tile_full, tile_free, tj, bv, bi, p.err))
      return;
    if (!p.has_tail) return;
    const StepTail& tl = p.tail;
    unsigned prev = 0;
    if (lane == 0) {
      tl.cand_v[c] = bv;
      tl.cand_i[c] = bi;
      __threadfence();
      prev = atomicAdd(tl.counter, 1u);
    }
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != (unsigned)P - 1) return;
    __threadfence();
    float v = -1e30f;
    uint32_t id = 0xffffffffu;
    for (int b = lane; b < P; b += 32) {
      const float cv = __ldcg(tl.cand_v + b);
      const uint32_t ci = __ldcg(tl.cand_i + b);
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
    if (lane == 0 && !tl.advance) {  // shard mode: the best of this row range
      *tl.amax = id + tl.id0;
      *tl.best_v = v;
      *tl.counter = 0u;
    } else if (lane == 0) {
      const int ps = *tl.pos;
      if (tl.greedy) {
        *tl.amax = id;
        tl.ids[ps + 1] = id;
        const int k = *tl.out_idx;
        tl.out_ids[k] = id;
        *tl.out_idx = k + 1;
      }
      *tl.pos = ps + 1;
      *tl.counter = 0u;
    }
    return;
  }
  stage_xd8<MAXU, NORM, NT>(p.x, p.K, gpr * kGroup, xb, xmul, sred, p.pdl);
  if (p.pdl) pdl_launch_dependents();
  bool dead = false;
  consume_q8_run<kOpWarps>(ring, full, empty, p.stages, p.stage_bytes, p.cap, t_lo, t_hi, gpr, xb, xmul, red,
                 tile_full, tile_free, rp, tj, dead, p.err);
}

template <int MAXU, bool NORM>
static void gemv_q8_go(const Q8Args& a0, cudaStream_t st, bool pdl) {
  Q8Args a = a0;
  const int gpr = (a.K + kGroup - 1) / kGroup;
  a.cap = 16;  // 32 KB stages
  a.stage_bytes = a.cap * kQ8Block;
  a.xs_off = kBarBytes;
  a.ring_off = (a.xs_off + gpr * (512 + 8) + 127) & ~127;
  const int budget = 150 * 1024;
  a.stages = std::max(2, std::min(8, (budget - a.ring_off) / a.stage_bytes));
  const int smem = a.ring_off + a.stages * a.stage_bytes;
  a.pdl = pdl ? 1 : 0;
  const int P = std::min(sm_count(), (a.N + 15) / 16);
  auto k = gemv_q8_kernel<MAXU, NORM>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  launch(k, dim3(P), dim3(kOpThreads), (size_t)smem, st, pdl, a);
}

void gemv_q8(const unsigned char* ws, const float* s, int N, int K, const XSrc& x, float* y,
             const StepTail* tail, cudaStream_t st, bool pdl, const GemvWork& wk) {
  Q8Args a = {};
  a.ws = ws;
  a.s = s;
  a.N = N;
  a.K = K;
  a.x = x;
  a.y = y;
  if (tail) a.tail = *tail;
  a.has_tail = tail ? 1 : 0;
  a.err = wk.err;
  const int u = (K / 4 + kOpWarps * 32 - 1) / (kOpWarps * 32);  // units of 4 per thread
  if (x.mode != X_PLAIN) {
    if (u <= 1) gemv_q8_go<1, true>(a, st, pdl);
    else gemv_q8_go<6, true>(a, st, pdl);
  } else {
    if (u <= 1) gemv_q8_go<1, false>(a, st, pdl);
    else gemv_q8_go<6, false>(a, st, pdl);
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
// Decode attention (attn_run, eg_stream.cuh): a 1-D grid of CTAs that take
// the (KV head, head subset, chunk) items of the current context
// ======================================================================
static_assert(kAttnDefaultChunk == kAttnKeys, "one default chunk");
int attn_max_splits(int max_ctx) { return std::max(64, (max_ctx + 15) / 16); }

// CTAs of one attention launch: enough for one item per query head and
// chunk at ctx_bound, at most one per SM (512 threads x 111-128 registers).
int attn_ctas(const AttnArgs& a, int lanes) {
  const int keys = a.chunk > 0 ? a.chunk : kAttnKeys;
  const int chunks = std::min(a.max_splits, (a.ctx_bound + keys - 1) / keys);
  const int cap = std::max(1, sm_count() / std::max(1, lanes));
  return std::max(1, std::min(cap, a.nh * chunks));
}

template <typename KVT>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_head_kernel(AttnArgs a, int pdl) {
  __shared__ AttnSmem sm;
  attn_run<KVT, false>(a, blockIdx.x, gridDim.x, pdl, sm);
}

// Long contexts: one tensor-core item per (KV head, chunk).
__global__ void __launch_bounds__(kAttnWarps * 32) attn_long_kernel(AttnArgs a, int pdl) {
  __shared__ AttnSmem sm;
  attn_run_mma<__half>(a, blockIdx.x, gridDim.x, pdl, sm);
}

bool attn_long(const AttnArgs& a, int pos) {
  const int keys = a.chunk > 0 ? a.chunk : kAttnKeys;
  return a.kv_f16 && a.nh / a.nkv <= kAmHeads && (pos + keys) / keys >= kAmMinSplits;
}

void attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl, bool long_ctx) {
  if (long_ctx && a.kv_f16 && a.nh / a.nkv <= kAmHeads) {
    const int keys = a.chunk > 0 ? a.chunk : kAttnKeys;
    const int chunks = std::min(a.max_splits, (a.ctx_bound + keys - 1) / keys);
    const dim3 grid(std::max(1, std::min(sm_count(), a.nkv * chunks)));
    launch(attn_long_kernel, grid, dim3(kAttnWarps * 32), 0, st, pdl, a, (int)pdl);
    return;
  }
  const dim3 grid(attn_ctas(a, 1));
  if (a.kv_f16)
    launch(attn_head_kernel<__half>, grid, dim3(kAttnWarps * 32), 0, st, pdl, a, (int)pdl);
  else
    launch(attn_head_kernel<float>, grid, dim3(kAttnWarps * 32), 0, st, pdl, a, (int)pdl);
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
int topk_cand_blocks(int n) { return std::max(1, std::min(kCandMax, (n + 1023) / 1024)); }

// Stage 1: per-block argmax candidates.  Stage 2 (one block) merges them.
// Lanes of a batch: stage 1 blockIdx.y, stage 2 blockIdx.x (logits [lane][n]).
__global__ void argmax_stage1(const float* logits, int n, float* cv, uint32_t* ci) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  logits += (size_t)blockIdx.y * n;
  cv += (size_t)blockIdx.y * gridDim.x;
  ci += (size_t)blockIdx.y * gridDim.x;
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
  cv += (size_t)blockIdx.x * nc;
  ci += (size_t)blockIdx.x * nc;
  out += blockIdx.x;
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
  logits += (size_t)blockIdx.y * n;
  cv += (size_t)blockIdx.y * gridDim.x * k;
  ci += (size_t)blockIdx.y * gridDim.x * k;
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
  cv_in += (size_t)blockIdx.x * nc;
  ci_in += (size_t)blockIdx.x * nc;
  ids += (size_t)blockIdx.x * k;
  vals += (size_t)blockIdx.x * k;
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
static int topk_blocks(int n) {
  int nb = topk_cand_blocks(n);
  while ((long long)nb * 256 * kTopkPer < n) nb++;
  return std::min(nb, kCandMax);
}
void topk(const float* logits, int n, int k, uint32_t* ids, float* vals, float* cand_v,
          uint32_t* cand_i, cudaStream_t st) {
  topk_batch(logits, n, k, 1, ids, vals, cand_v, cand_i, st);
}
int topk_batch_cand(int n, int k) { return topk_blocks(n) * k; }
void topk_batch(const float* logits, int n, int k, int lanes, uint32_t* ids, float* vals,
                float* cand_v, uint32_t* cand_i, cudaStream_t st) {
  const int nb = topk_blocks(n);
  topk_stage1<<<dim3(nb, lanes), 256, 0, st>>>(logits, n, k, cand_v, cand_i);
  const int nc = nb * k;
  cudaFuncSetAttribute(topk_stage2, cudaFuncAttributeMaxDynamicSharedMemorySize, nc * 8);
  topk_stage2<<<lanes, 256, (size_t)nc * 8, st>>>(cand_v, cand_i, nc, k, ids, vals);
}
void argmax_batch(const float* logits, int n, int lanes, uint32_t* out, float* cand_v,
                  uint32_t* cand_i, cudaStream_t st) {
  const int nb = topk_cand_blocks(n);
  argmax_stage1<<<dim3(nb, lanes), 256, 0, st>>>(logits, n, cand_v, cand_i);
  argmax_stage2<<<lanes, 256, 0, st>>>(cand_v, cand_i, nb, out);
}

// SAMPLE_TOPK restated literally: 64 slots, exp without max subtraction,
// pairwise tree sum, Hillis-Steele inclusive prefix, first j with r <= P_j.
// Batch lanes: blockIdx.x, with r = r_all[*step_ctr * kBatchMax + lane].
__global__ void sample_topk_kernel(const uint32_t* ids, const float* vals, int k, float temp, float r,
                                   uint32_t* out, uint32_t* out2, const float* r_all,
                                   const int* step_ctr) {
  __shared__ float s[64], red[64];
  const int tid = threadIdx.x;
  if (r_all) {
    r = r_all[(size_t)*step_ctr * kBatchMax + blockIdx.x];
    ids += (size_t)blockIdx.x * k;
    vals += (size_t)blockIdx.x * k;
    out += blockIdx.x;
  }
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
  sample_topk_kernel<<<1, 64, 0, st>>>(ids, vals, k, temp, r, out, out2, nullptr, nullptr);
}
void sample_batch(const uint32_t* ids, const float* vals, int k, float temp, const float* r,
                  const int* step_ctr, int lanes, uint32_t* out, cudaStream_t st) {
  sample_topk_kernel<<<lanes, 64, 0, st>>>(ids, vals, k, temp, 0.f, out, nullptr, r, step_ctr);
}

}  // namespace eg
