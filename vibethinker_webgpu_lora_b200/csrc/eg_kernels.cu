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

// ----------------------------------------------------------------------
// Streaming int4 GEMV over the "stream" layout (q4_to_stream): the matrix
// as blocks (tile, group) -- 16 rows x 128 k of packed nibbles (for
// [gate;up] a tile is the gate tile plus its up tile), stored in MMA
// fragment order and followed by the block's 16 (32) group scales -- laid
// out tile-major, group-minor.  The tiles are split into gridDim.x
// contiguous ranges, one per CTA, and any contiguous run of blocks is one
// contiguous byte range: warp 8 moves each ring stage (<= 16 KB of nibbles)
// with a single cp.async.bulk.  The weights do not depend on the previous
// kernel, so those copies start before griddepcontrol.wait.  Warps 0-7 build
// the activation fragments (stage_xg), then turn each stage into m16n8k16
// MMAs; each warp's 16-byte fragment loads cover 512 contiguous bytes (no
// bank conflicts).  Every tile is finished inside one CTA, so the epilogue
// needs no cross-CTA combine (a memory fence under a saturated memory
// system costs microseconds).
struct G4Args {
  const unsigned char* ws;  // stream layout
  int N, K;
  XSrc x;
  Epi e;
  int* err;
  int stages, stage_bytes, cap, xs_off, ring_off;
  int pdl;
};

// Block of the stream layout: R * (1024 bytes of nibbles + 64 bytes of scales).
__host__ __device__ constexpr int q4_block_bytes(int R) { return R * 1088; }


#ifdef EG_G4_TRACE  // timeline probe (clock64 per CTA), never in library builds
__device__ long long g4_trace[512][64];
#define G4T(slot)                                                     \
  do {                                                                \
    if (lane == 0 && (slot) < 64) g4_trace[blockIdx.x][(slot)] = clock64(); \
  } while (0)
#else
#define G4T(slot) \
  do {            \
  } while (0)
#endif

constexpr int kG4Warps = 16;                   // consumer warps per CTA (one CTA per SM)
constexpr int kG4Threads = kG4Warps * 32 + 64;  // + producer warp + epilogue warp

// Producer warp of a streaming GEMV: copy `nitems` blocks of `blk` bytes
// from src0 into the ring, `cap` blocks (one cp.async.bulk) per stage, each
// stage reused once all consumer warps released it.
__device__ __forceinline__ void ring_produce(unsigned char* ring, uint64_t* full, uint64_t* empty,
                                             int stages, int stage_bytes,
                                             const unsigned char* src0, int nitems, int cap,
                                             int blk, int* err, int lane) {
  const int nchunks = (nitems + cap - 1) / cap;
  int st = 0, ph = 0, n = 0;
  for (; n < nchunks; n++) {
    if (!mbar_wait(&empty[st], ph ^ 1, err)) break;
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)(min(cap, nitems - n * cap) * blk);
      mbar_expect_tx(&full[st], bytes);
      bulk_g2s(ring + (size_t)st * stage_bytes, src0 + (size_t)n * cap * blk, bytes, &full[st]);
    }
    __syncwarp();
    if (++st == stages) {
      st = 0;
      ph ^= 1;
    }
  }
  // every issued copy has landed before the CTA may exit (bounded even after
  // an error elsewhere)
  for (int k = n > stages ? n - stages : 0; k < n; k++)
    if (!mbar_wait_bounded(&full[k % stages], (k / stages) & 1)) break;
}

// One CTA per SM.  Warps 0-15 consume, warp 16 produces, warp 17 runs the
// epilogues.  The CTA's tiles form a contiguous run of blocks (items) in the
// stream layout; the producer copies it in stages of p.cap items (one
// cp.async.bulk each) into a ring.  Consumer warp w takes items w, w + 16,
// w + 32, ... (so for K = 2048 every warp holds one group of every tile),
// keeps one running sum per row pair across stages, and at the end of each
// tile leaves its partial row sums in red[buf] for the epilogue warp.  Every
// consumer waits on every stage and releases it, items or not, so the ring
// protocol needs no per-warp bookkeeping.
template <int R, int MAXU, bool NORM>
__global__ void __launch_bounds__(kG4Threads, 1) gemv_q4_kernel(G4Args p) {
  constexpr int CW = kG4Warps, NT = CW * 32;
  extern __shared__ __align__(128) unsigned char g4_smem[];
  __shared__ float sred[32];
  __shared__ float red[2][CW][R][16];  // double buffered tile hand-off
  uint64_t* full = reinterpret_cast<uint64_t*>(g4_smem);
  uint64_t* empty = full + p.stages;
  uint64_t* tile_full = empty + p.stages;  // [2]
  uint64_t* tile_free = tile_full + 2;     // [2]
  const int gpr = p.K / kGroup;
  uint2* xb = reinterpret_cast<uint2*>(g4_smem + p.xs_off);  // [gpr][4][4][4]
  int* xcor = reinterpret_cast<int*>(xb + (size_t)gpr * 64);  // [gpr][2]
  float* xmul = reinterpret_cast<float*>(xcor + 2 * gpr);     // [gpr][2]
  unsigned char* ring = g4_smem + p.ring_off;
  const int tiles = (p.N + 15) / 16;
  const int P = gridDim.x, c = blockIdx.x;
  const int t_lo = (int)((long long)tiles * c / P), t_hi = (int)((long long)tiles * (c + 1) / P);
  const int nitems = (t_hi - t_lo) * gpr;
  const int cap = p.cap;
  const int nchunks = (nitems + cap - 1) / cap;
  const int blk = q4_block_bytes(R);
  const unsigned char* src0 = p.ws + (size_t)t_lo * gpr * blk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CW);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tile_full[i], CW);
      mbar_init(&tile_free[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == 0) G4T(0);

  if (warp == CW) {  // --------------------------------------------- producer
    ring_produce(ring, full, empty, p.stages, p.stage_bytes, src0, nitems, cap, blk, p.err, lane);
    return;
  }

  if (warp == CW + 1) {  // ------------------------------------------- epilogue
    if (p.pdl) pdl_wait();  // residuals are written by earlier kernels
    const bool lora = p.e.mods != nullptr;
    float pre = 0.f;
    if (lane < 16 && !lora) pre = epi_pre(p.e, t_lo * 16 + lane);
    for (int tile = t_lo, j = 0; tile < t_hi; tile++, j++) {
      const int b = j & 1;
      if (!mbar_wait(&tile_full[b], (j >> 1) & 1, p.err)) break;
      float v = 0.f;
      if (lane < 16 * R)
        for (int ww = 0; ww < CW; ww++) v += red[b][ww][lane >> 4][lane & 15];
      __syncwarp();
      if (lane == 0) mbar_arrive(&tile_free[b]);
      const float up = __shfl_down_sync(0xffffffffu, v, 16);
      if (lane < 16) {
        const int row = tile * 16 + lane;
        if (lora)
          epilogue_row(p.e, row, v, R == 2 ? up : 0.f);
        else
          epilogue_row_pre(p.e, row, v, R == 2 ? up : 0.f, pre);
        if (!lora && tile + 1 < t_hi) pre = epi_pre(p.e, row + 16);
      }
    }
    return;
  }

  // ------------------------------------------------------------- consumers
  stage_xd<MAXU, NORM, NT>(p.x, p.K, xb, xcor, xmul, sred, p.pdl);
  // the next kernel may start once this one's predecessors are complete
  // (the attention kernel relies on that to read the position early)
  if (p.pdl) pdl_launch_dependents();
  if (warp == 0) G4T(1);
  const int gq = lane >> 2, t = lane & 3;
  const bool bl = gq < 4;  // lanes holding a digit plane (B columns 0-3)
  float acc[R][2];
#pragma unroll
  for (int r = 0; r < R; r++) acc[r][0] = acc[r][1] = 0.f;
  // after a failed wait the CTA runs on without waiting and its results are
  // void; the host sees the error word
  bool dead = false;
  int st = 0, ph = 0, chunk = 0, chunk_lo = 0;
  if (nchunks > 0 && !mbar_wait(&full[0], 0, p.err)) dead = true;
  const unsigned char* stage = ring;
  int i = warp;  // item index within the CTA's run
  for (int tile = t_lo, j = 0; tile < t_hi; tile++, j++) {
    const int tile_end = (j + 1) * gpr;
    for (; i < tile_end; i += 16) {
      while (i >= chunk_lo + cap) {  // next stage
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if (++st == p.stages) {
          st = 0;
          ph ^= 1;
        }
        chunk++;
        chunk_lo += cap;
        stage = ring + (size_t)st * p.stage_bytes;
        if (!dead && !mbar_wait(&full[st], ph, p.err)) dead = true;
        if (warp == 0) G4T(2 + chunk);
      }
      const int g = i - j * gpr;
      const unsigned char* bp = stage + (size_t)(i - chunk_lo) * blk;
      // B: digit plane gq of this group's 4 k32 blocks (zero for gq >= 4)
      uint4 X0 = make_uint4(0, 0, 0, 0), X1 = make_uint4(0, 0, 0, 0);
      if (bl) {
        const uint4* xp = reinterpret_cast<const uint4*>(xb + ((g * 4 + gq) * 4 + t) * 4);
        X0 = xp[0];
        X1 = xp[1];
      }
      uint4 A[R], B[R];
#pragma unroll
      for (int r = 0; r < R; r++) {
        // words t, 4+t, 8+t, 12+t of rows gq (A) and gq+8 (B)
        A[r] = *reinterpret_cast<const uint4*>(bp + r * 1024 + lane * 16);
        B[r] = *reinterpret_cast<const uint4*>(bp + r * 1024 + 512 + lane * 16);
      }
      int cc[R][4];
#pragma unroll
      for (int r = 0; r < R; r++) {
        cc[r][0] = cc[r][1] = cc[r][2] = cc[r][3] = 0;
        imma16832(cc[r], nib_lo_u8(A[r].x), nib_lo_u8(B[r].x), nib_hi_u8(A[r].x), nib_hi_u8(B[r].x), X0.x, X0.y);
        imma16832(cc[r], nib_lo_u8(A[r].y), nib_lo_u8(B[r].y), nib_hi_u8(A[r].y), nib_hi_u8(B[r].y), X0.z, X0.w);
        imma16832(cc[r], nib_lo_u8(A[r].z), nib_lo_u8(B[r].z), nib_hi_u8(A[r].z), nib_hi_u8(B[r].z), X1.x, X1.y);
        imma16832(cc[r], nib_lo_u8(A[r].w), nib_lo_u8(B[r].w), nib_hi_u8(A[r].w), nib_hi_u8(B[r].w), X1.z, X1.w);
      }
      if (t < 2) {  // columns 2t, 2t+1 = digit planes 2t, 2t+1
        const int cor = xcor[2 * g + t];
        const float mul = xmul[2 * g + t];
        const float* sc = reinterpret_cast<const float*>(bp + R * 1024);
#pragma unroll
        for (int r = 0; r < R; r++) {
          const float sa = sc[16 * r + gq] * mul, sb = sc[16 * r + gq + 8] * mul;
          acc[r][0] = fmaf(sa, (float)(cc[r][0] + 256 * cc[r][1] - cor), acc[r][0]);
          acc[r][1] = fmaf(sb, (float)(cc[r][2] + 256 * cc[r][3] - cor), acc[r][1]);
        }
      }
    }
    // ---- tile complete for this warp: hand its partial rows to the epilogue
#pragma unroll
    for (int r = 0; r < R; r++) {
      acc[r][0] += __shfl_xor_sync(0xffffffffu, acc[r][0], 1);
      acc[r][1] += __shfl_xor_sync(0xffffffffu, acc[r][1], 1);
    }
    const int b = j & 1;
    if (!dead && !mbar_wait(&tile_free[b], ((j >> 1) & 1) ^ 1, p.err)) dead = true;
    if (t == 0) {
#pragma unroll
      for (int r = 0; r < R; r++) {
        red[b][warp][r][gq] = acc[r][0];
        red[b][warp][r][gq + 8] = acc[r][1];
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++) acc[r][0] = acc[r][1] = 0.f;
    __syncwarp();
    if (lane == 0) mbar_arrive(&tile_full[b]);
    if (warp == 0) G4T(48 + min(j, 13));
  }
  // release the current stage and wait/release any later ones this warp had
  // no items in, so every stage sees all CW arrivals
  for (; chunk < nchunks; chunk++) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (++st == p.stages) {
      st = 0;
      ph ^= 1;
    }
    if (chunk + 1 < nchunks && !dead && !mbar_wait(&full[st], ph, p.err)) dead = true;
  }
  if (warp == 0) G4T(63);
}


// Shared-memory plan of one launch (bytes): barriers, x fragments + group
// multipliers, then the ring of stages of `cap` items.
struct G4Plan {
  int stages, stage_bytes, cap, xs_off, ring_off, smem;
};
static G4Plan g4_plan(int R, int K) {
  G4Plan q;
  const int gpr = K / kGroup;
  q.cap = (getenv("EG_G4_CAP") ? atoi(getenv("EG_G4_CAP")) : 32) / R;  // items per stage: 35 KB
  q.stage_bytes = q.cap * q4_block_bytes(R);
  q.xs_off = 256;  // barriers: 2 * stages + 4 mbarriers (stages <= 8)
  const int xbytes = gpr * (512 + 16);
  q.ring_off = (q.xs_off + xbytes + 127) & ~127;
  // leave room for the attention kernel's CTA (67 KB) beside this one under PDL
  const int budget = (getenv("EG_G4_SMEM") ? atoi(getenv("EG_G4_SMEM")) : 150) * 1024;
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
  launch(k, dim3(P), dim3(kG4Threads), (size_t)q.smem, st, pdl, a);
}

template <int R>
static void gemv_q4_r(const G4Args& a, cudaStream_t st, bool pdl) {
  const G4Plan q = g4_plan(R, a.K);
  const int u = (a.K / 8 + kG4Warps * 32 - 1) / (kG4Warps * 32);  // units per thread
  if (a.x.mode != X_PLAIN) {  // RMSNorm holds the whole vector in registers
    if (u <= 1) gemv_q4_go<R, 1, true>(a, q, st, pdl);
    else gemv_q4_go<R, 3, true>(a, q, st, pdl);
  } else if (u <= 1) {
    gemv_q4_go<R, 1, false>(a, q, st, pdl);
  } else {
    gemv_q4_go<R, 3, false>(a, q, st, pdl);  // K <= 12288
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
  if (e.mode == EPI_SILU)
    gemv_q4_r<2>(a, st, pdl);
  else
    gemv_q4_r<1>(a, st, pdl);
}

size_t q4_stream_bytes(int N, int K, int R) {
  return (size_t)((N + 15) / 16) * (K / kGroup) * q4_block_bytes(R);
}

// One thread per 16-byte fragment word of the stream layout; rows past N
// are zero.  Threads with u >= the fragment count copy the scales instead.
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
    reinterpret_cast<float*>(out + b * q4_block_bytes(R) + R * 1024)[r * 16 + i] = sv;
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
constexpr int kQ8Block = 2048;

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

// Same warp roles as gemv_q4_kernel.  The epilogue warp writes
// y[n] = (row sum) * s[n] and keeps the best (value, index); with a tail, the
// CTAs' candidates are merged by the last CTA to finish, which also advances
// the decode position (ARGMAX kernels.js:771-784, then decodeBatch's copy of
// s.amax into the id buffer, runtime.js:1783-1785).
template <int MAXU, bool NORM>
__global__ void __launch_bounds__(kG4Threads, 1) gemv_q8_kernel(Q8Args p) {
  constexpr int CW = kG4Warps, NT = CW * 32;
  extern __shared__ __align__(128) unsigned char g4_smem[];
  __shared__ float sred[32];
  __shared__ float red[2][CW][16];
  uint64_t* full = reinterpret_cast<uint64_t*>(g4_smem);
  uint64_t* empty = full + p.stages;
  uint64_t* tile_full = empty + p.stages;  // [2]
  uint64_t* tile_free = tile_full + 2;     // [2]
  const int gpr = (p.K + kGroup - 1) / kGroup;
  uint32_t* xb = reinterpret_cast<uint32_t*>(g4_smem + p.xs_off);  // [gpr][4][4][4][2]
  float* xmul = reinterpret_cast<float*>(xb + (size_t)gpr * 128);  // [gpr][2]
  unsigned char* ring = g4_smem + p.ring_off;
  const int tiles = (p.N + 15) / 16;
  const int P = gridDim.x, c = blockIdx.x;
  const int t_lo = (int)((long long)tiles * c / P), t_hi = (int)((long long)tiles * (c + 1) / P);
  const int nitems = (t_hi - t_lo) * gpr;
  const int cap = p.cap;
  const int nchunks = (nitems + cap - 1) / cap;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CW);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tile_full[i], CW);
      mbar_init(&tile_free[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == CW) {  // --------------------------------------------- producer
    ring_produce(ring, full, empty, p.stages, p.stage_bytes, p.ws + (size_t)t_lo * gpr * kQ8Block,
                 nitems, cap, kQ8Block, p.err, lane);
    return;
  }

  if (warp == CW + 1) {  // ------------------------------------------- epilogue
    float sc = lane < 16 && t_lo * 16 + lane < p.N ? __ldg(p.s + t_lo * 16 + lane) : 0.f;
    float bv = -1e30f;
    uint32_t bi = 0xffffffffu;
    for (int tile = t_lo, j = 0; tile < t_hi; tile++, j++) {
      const int b = j & 1;
      if (!mbar_wait(&tile_full[b], (j >> 1) & 1, p.err)) break;
      float v = 0.f;
      if (lane < 16)
        for (int ww = 0; ww < CW; ww++) v += red[b][ww][lane];
      __syncwarp();
      if (lane == 0) mbar_arrive(&tile_free[b]);
      const int n = tile * 16 + lane;
      if (lane < 16 && n < p.N) {
        const float o = __fmul_rn(v, sc);  // sum first, scale last
        p.y[n] = o;
        if (beats(o, (uint32_t)n, bv, bi)) {
          bv = o;
          bi = (uint32_t)n;
        }
        sc = n + 16 < p.N && tile + 1 < t_hi ? __ldg(p.s + n + 16) : 0.f;
      }
    }
    if (!p.has_tail) return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (beats(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
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
    if (lane == 0) {
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

  // ------------------------------------------------------------- consumers
  stage_xd8<MAXU, NORM, NT>(p.x, p.K, gpr * kGroup, xb, xmul, sred, p.pdl);
  if (p.pdl) pdl_launch_dependents();
  const int gq = lane >> 2, t = lane & 3;
  const bool bl = gq < 4;  // lanes holding a digit plane (B columns 0-3)
  float acc0 = 0.f, acc1 = 0.f;
  bool dead = false;
  int st = 0, ph = 0, chunk = 0, chunk_lo = 0;
  if (nchunks > 0 && !mbar_wait(&full[0], 0, p.err)) dead = true;
  const unsigned char* stage = ring;
  int i = warp;
  for (int tile = t_lo, j = 0; tile < t_hi; tile++, j++) {
    const int tile_end = (j + 1) * gpr;
    for (; i < tile_end; i += 16) {
      while (i >= chunk_lo + cap) {  // next stage
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if (++st == p.stages) {
          st = 0;
          ph ^= 1;
        }
        chunk++;
        chunk_lo += cap;
        stage = ring + (size_t)st * p.stage_bytes;
        if (!dead && !mbar_wait(&full[st], ph, p.err)) dead = true;
      }
      const int g = i - j * gpr;
      const unsigned char* bp = stage + (size_t)(i - chunk_lo) * kQ8Block;
      uint4 X0 = make_uint4(0, 0, 0, 0), X1 = make_uint4(0, 0, 0, 0);
      if (bl) {
        const uint4* xp = reinterpret_cast<const uint4*>(xb + ((g * 4 + gq) * 4 + t) * 8);
        X0 = xp[0];
        X1 = xp[1];
      }
      const uint4 A0 = *reinterpret_cast<const uint4*>(bp + lane * 16);
      const uint4 A1 = *reinterpret_cast<const uint4*>(bp + 512 + lane * 16);
      const uint4 B0 = *reinterpret_cast<const uint4*>(bp + 1024 + lane * 16);
      const uint4 B1 = *reinterpret_cast<const uint4*>(bp + 1536 + lane * 16);
      int cc[4] = {0, 0, 0, 0};
      imma16832_ss(cc, A0.x, B0.x, A0.y, B0.y, X0.x, X0.y);
      imma16832_ss(cc, A0.z, B0.z, A0.w, B0.w, X0.z, X0.w);
      imma16832_ss(cc, A1.x, B1.x, A1.y, B1.y, X1.x, X1.y);
      imma16832_ss(cc, A1.z, B1.z, A1.w, B1.w, X1.z, X1.w);
      if (t < 2) {  // columns 2t, 2t+1 = digit planes 2t, 2t+1
        const float mul = xmul[2 * g + t];
        acc0 = fmaf(mul, (float)(cc[0] + 256 * cc[1]), acc0);
        acc1 = fmaf(mul, (float)(cc[2] + 256 * cc[3]), acc1);
      }
    }
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    const int b = j & 1;
    if (!dead && !mbar_wait(&tile_free[b], ((j >> 1) & 1) ^ 1, p.err)) dead = true;
    if (t == 0) {
      red[b][warp][gq] = acc0;
      red[b][warp][gq + 8] = acc1;
    }
    acc0 = acc1 = 0.f;
    __syncwarp();
    if (lane == 0) mbar_arrive(&tile_full[b]);
  }
  // release the current stage and wait/release the later ones (see gemv_q4_kernel)
  for (; chunk < nchunks; chunk++) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (++st == p.stages) {
      st = 0;
      ph ^= 1;
    }
    if (chunk + 1 < nchunks && !dead && !mbar_wait(&full[st], ph, p.err)) dead = true;
  }
}

template <int MAXU, bool NORM>
static void gemv_q8_go(const Q8Args& a0, cudaStream_t st, bool pdl) {
  Q8Args a = a0;
  const int gpr = (a.K + kGroup - 1) / kGroup;
  a.cap = 16;  // 32 KB stages
  a.stage_bytes = a.cap * kQ8Block;
  a.xs_off = 256;
  a.ring_off = (a.xs_off + gpr * (512 + 8) + 127) & ~127;
  const int budget = 150 * 1024;
  a.stages = std::max(2, std::min(8, (budget - a.ring_off) / a.stage_bytes));
  const int smem = a.ring_off + a.stages * a.stage_bytes;
  a.pdl = pdl ? 1 : 0;
  const int P = std::min(sm_count(), (a.N + 15) / 16);
  auto k = gemv_q8_kernel<MAXU, NORM>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  launch(k, dim3(P), dim3(kG4Threads), (size_t)smem, st, pdl, a);
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
  const int u = (K / 4 + kG4Warps * 32 - 1) / (kG4Warps * 32);  // units of 4 per thread
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
// Attention: RoPE + KV append + split-K partials, then combine
// ======================================================================
int attn_max_splits(int max_ctx) { return std::max(64, (max_ctx + 15) / 16); }

// ----------------------------------------------------------------------
// Decode attention, one CTA per (query head, split of <= kAttnKeys keys).
// Each of the 16 warps takes keys t0 + w, t0 + w + 16, ...; a lane holds 4
// of the 128 dims.  All K and V rows of the warp are requested before
// griddepcontrol.wait (the cache rows t != pos were written by earlier
// steps), so the kernel pays one memory latency for them.  Each warp forms a
// partial (m, z, sum e^(s-m) v) over its keys (ATTN_PARTIAL, kernels.js:
// 258-345), the 16 warp partials are merged in shared memory with the
// ATTN_COMBINE formula (kernels.js:346-388, f16 rounding of the partial
// outputs in the f16 variant), and for contexts longer than one split the
// CTA partials are merged once more by the last CTA of the head.  The new
// k (RoPE) / v row of position pos is formed in registers; the first query
// head of each KV group appends it to the cache (runtime.js:1509-1514).
constexpr int kAttnWarps = 16;
constexpr int kAttnKeys = 256;                   // keys per split (16 per warp)
constexpr int kAttnKpw = kAttnKeys / kAttnWarps;

// A value as the cache stores it (rounded to the cache type).
template <typename KVT>
__device__ __forceinline__ float kv_round(float v);
template <>
__device__ __forceinline__ float kv_round<float>(float v) { return v; }
template <>
__device__ __forceinline__ float kv_round<__half>(float v) { return round_h(v); }

template <typename KVT>
struct KvRow;  // 4 consecutive cache values of one lane
template <>
struct KvRow<__half> {
  uint2 u;
  __device__ __forceinline__ void load(const __half* p) { u = __ldcg(reinterpret_cast<const uint2*>(p)); }
  __device__ __forceinline__ float4 get() const {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  __device__ __forceinline__ void set(float4 v) {  // values already f16-exact
    const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
  }
};
template <>
struct KvRow<float> {
  float4 f;
  __device__ __forceinline__ void load(const float* p) { f = __ldcg(reinterpret_cast<const float4*>(p)); }
  __device__ __forceinline__ float4 get() const { return f; }
  __device__ __forceinline__ void set(float4 v) { f = v; }
};

template <typename KVT>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_head_kernel(AttnArgs a, int pdl) {
  __shared__ float wm[kAttnWarps], wz[kAttnWarps];
  __shared__ __align__(16) float wo[kAttnWarps][kHeadDim];
  __shared__ bool last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, split = blockIdx.x;
  const int G = a.nh / a.nkv, kvh = h / G, hd = kHeadDim, half = hd / 2;
  const int kvd = a.nkv * hd;
  const int f16 = a.kv_f16;
  // The position and the cached rows t != pos were written before the
  // producing GEMV started (it triggers this launch only after its own
  // griddepcontrol.wait).
  const int pos = a.pos ? __ldcg(a.pos) : a.fixed_pos;
  const int ctx = pos + 1;
  const int keys = a.chunk > 0 ? a.chunk : kAttnKeys;
  const int nsplit = (ctx + keys - 1) / keys;
  if (split >= nsplit) return;
  const int t0 = split * keys, t1 = min(t0 + keys, ctx);
  const KVT* kc = reinterpret_cast<const KVT*>(a.kc) + kvh * hd + 4 * lane;
  const KVT* vc = reinterpret_cast<const KVT*>(a.vc) + kvh * hd + 4 * lane;
  KvRow<KVT> K[kAttnKpw], V[kAttnKpw];
#pragma unroll
  for (int i = 0; i < kAttnKpw; i++) {
    const int t = t0 + warp + kAttnWarps * i;
    if (t < t1 && t != pos) {
      K[i].load(kc + (size_t)t * kvd);
      V[i].load(vc + (size_t)t * kvd);
    }
  }
  if (pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
  // q (ROPE_QK, f16 round in the f16 variant): lane holds dims 4l..4l+3; the
  // RoPE partner of dim j < 64 is j + 64, held by lane l ^ 16
  const float* cs = a.cosT + (size_t)pos * hd;
  const float* sn = a.sinT + (size_t)pos * hd;
  auto rope4 = [&](float4 x) {
    float4 o = x;
    float* e = reinterpret_cast<float*>(&o);
    const float* xi = reinterpret_cast<const float*>(&x);
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const float other = __shfl_xor_sync(0xffffffffu, xi[c], 16);
      const int d = 4 * lane + c, j = d & (half - 1);
      float lo = lane < 16 ? xi[c] : other, hi = lane < 16 ? other : xi[c];
      rope_pair(lo, hi, cs[j], sn[j], f16);
      if (f16) round_h2(lo, hi);
      e[c] = lane < 16 ? lo : hi;
    }
    return o;
  };
  const float4 q4 = rope4(__ldcg(reinterpret_cast<const float4*>(a.qkv + h * hd + 4 * lane)));
  if (pos >= t0 && pos < t1) {  // the new row: k = RoPE(k), v (f16-rounded in the f16 cache)
    const float* kn = a.qkv + a.nh * hd + kvh * hd;
    const float* vn = a.qkv + a.nh * hd + kvd + kvh * hd;
    float4 kr = __ldcg(reinterpret_cast<const float4*>(kn + 4 * lane));
    float4 vr = __ldcg(reinterpret_cast<const float4*>(vn + 4 * lane));
    // the cache keeps RoPE(k) rounded once to its type; scores use that value
    float4 kx;
    {
      float* e = reinterpret_cast<float*>(&kx);
      const float* xi = reinterpret_cast<const float*>(&kr);
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const float other = __shfl_xor_sync(0xffffffffu, xi[c], 16);
        const int d = 4 * lane + c, j = d & (half - 1);
        float lo = lane < 16 ? xi[c] : other, hi = lane < 16 ? other : xi[c];
        rope_pair(lo, hi, cs[j], sn[j], f16);
        e[c] = lane < 16 ? lo : hi;
      }
    }
    KvRow<KVT> kn4, vn4;
    kn4.set(make_float4(kv_round<KVT>(kx.x), kv_round<KVT>(kx.y), kv_round<KVT>(kx.z), kv_round<KVT>(kx.w)));
    vn4.set(make_float4(kv_round<KVT>(vr.x), kv_round<KVT>(vr.y), kv_round<KVT>(vr.z), kv_round<KVT>(vr.w)));
    const int i = (pos - t0) / kAttnWarps, w = (pos - t0) % kAttnWarps;
    if (warp == w) {
#pragma unroll
      for (int ii = 0; ii < kAttnKpw; ii++)
        if (ii == i) {
          K[ii] = kn4;
          V[ii] = vn4;
        }
    }
    if (h % G == 0 && warp == 0) {  // one query head per KV group appends
      KVT* kw = reinterpret_cast<KVT*>(a.kc) + (size_t)pos * kvd + kvh * hd + 4 * lane;
      KVT* vw = reinterpret_cast<KVT*>(a.vc) + (size_t)pos * kvd + kvh * hd + 4 * lane;
      kw[0] = kv_cvt<KVT>(kx.x); kw[1] = kv_cvt<KVT>(kx.y); kw[2] = kv_cvt<KVT>(kx.z); kw[3] = kv_cvt<KVT>(kx.w);
      vw[0] = kv_cvt<KVT>(vr.x); vw[1] = kv_cvt<KVT>(vr.y); vw[2] = kv_cvt<KVT>(vr.z); vw[3] = kv_cvt<KVT>(vr.w);
    }
  }
  // scores of this warp's keys: key i's score ends up in lane i
  const float scale = 1.0f / sqrtf((float)hd);
  float s_mine = -1e30f;
  float m = -1e30f;
#pragma unroll
  for (int i = 0; i < kAttnKpw; i++) {
    const int t = t0 + warp + kAttnWarps * i;
    if (t >= t1) break;
    const float4 k4 = K[i].get();
    float p = __fmul_rn(q4.x, k4.x);
    p = __fadd_rn(p, __fmul_rn(q4.y, k4.y));
    p = __fadd_rn(p, __fmul_rn(q4.z, k4.z));
    p = __fadd_rn(p, __fmul_rn(q4.w, k4.w));
    const float sv = __fmul_rn(warp_sum(p), scale);
    if (lane == i) s_mine = sv;
    m = fmaxf(m, sv);
  }
  const int nk = t1 - t0 > warp ? (t1 - t0 - warp + kAttnWarps - 1) / kAttnWarps : 0;
  const float ev_mine = lane < nk ? expf(s_mine - m) : 0.f;
  const float z = warp_sum(ev_mine);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kAttnKpw; i++) {
    if (i >= nk) break;
    const float ev = __shfl_sync(0xffffffffu, ev_mine, i);
    const float4 v4 = V[i].get();
    acc.x = __fadd_rn(acc.x, __fmul_rn(ev, v4.x));
    acc.y = __fadd_rn(acc.y, __fmul_rn(ev, v4.y));
    acc.z = __fadd_rn(acc.z, __fmul_rn(ev, v4.z));
    acc.w = __fadd_rn(acc.w, __fmul_rn(ev, v4.w));
  }
  if (f16) {  // ATTN_COMBINE_F16 reads the partial outputs through f16
    round_h2(acc.x, acc.y);
    round_h2(acc.z, acc.w);
  }
  if (lane == 0) {
    wm[warp] = nk ? m : -1e30f;
    wz[warp] = z;
  }
  *reinterpret_cast<float4*>(&wo[warp][4 * lane]) = acc;
  __syncthreads();
  // ---- merge the warp partials: warp 0, lane l holds dims 4l..4l+3
  if (warp == 0) {
    float M = -1e30f;
    for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, wm[w]);
    float Z = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int w = 0; w < kAttnWarps; w++) {
      if (wz[w] == 0.f) continue;
      const float wgt = expf(wm[w] - M);
      Z = __fadd_rn(Z, __fmul_rn(wz[w], wgt));
      const float4 p = *reinterpret_cast<const float4*>(&wo[w][4 * lane]);
      o.x = __fadd_rn(o.x, __fmul_rn(wgt, p.x));
      o.y = __fadd_rn(o.y, __fmul_rn(wgt, p.y));
      o.z = __fadd_rn(o.z, __fmul_rn(wgt, p.z));
      o.w = __fadd_rn(o.w, __fmul_rn(wgt, p.w));
    }
    if (nsplit == 1) {
      const float invZ = 1.0f / Z;
      *reinterpret_cast<float4*>(a.out + h * hd + 4 * lane) =
          make_float4(__fmul_rn(o.x, invZ), __fmul_rn(o.y, invZ), __fmul_rn(o.z, invZ), __fmul_rn(o.w, invZ));
    } else {
      if (f16) {
        round_h2(o.x, o.y);
        round_h2(o.z, o.w);
      }
      *reinterpret_cast<float4*>(a.po + ((size_t)h * a.max_splits + split) * hd + 4 * lane) = o;
      if (lane == 0) {
        a.pm[h * a.max_splits + split] = M;
        a.pz[h * a.max_splits + split] = Z;
      }
    }
  }
  if (nsplit == 1) return;
  // ---- several splits: the last CTA of the head merges them
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(a.counters + h, 1u) == (unsigned)nsplit - 1;
  __syncthreads();
  if (!last || warp != 0) return;
  __threadfence();
  const float* pm = a.pm + h * a.max_splits;
  const float* pz = a.pz + h * a.max_splits;
  float M = -1e30f;
  for (int s2 = 0; s2 < nsplit; s2++) M = fmaxf(M, __ldcg(pm + s2));
  float Z = 0.f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s2 = 0; s2 < nsplit; s2++) {
    const float wgt = expf(__ldcg(pm + s2) - M);
    Z = __fadd_rn(Z, __fmul_rn(__ldcg(pz + s2), wgt));
    const float4 p = __ldcg(reinterpret_cast<const float4*>(a.po + ((size_t)h * a.max_splits + s2) * hd + 4 * lane));
    o.x = __fadd_rn(o.x, __fmul_rn(wgt, p.x));
    o.y = __fadd_rn(o.y, __fmul_rn(wgt, p.y));
    o.z = __fadd_rn(o.z, __fmul_rn(wgt, p.z));
    o.w = __fadd_rn(o.w, __fmul_rn(wgt, p.w));
  }
  const float invZ = 1.0f / Z;
  *reinterpret_cast<float4*>(a.out + h * hd + 4 * lane) =
      make_float4(__fmul_rn(o.x, invZ), __fmul_rn(o.y, invZ), __fmul_rn(o.z, invZ), __fmul_rn(o.w, invZ));
  if (lane == 0) a.counters[h] = 0u;  // ready for the next launch
}


void attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl) {
  // splits of kAttnKeys keys (a fixed chunk, when given, for tests of the
  // multi-split merge); the partial slots (max_splits per head) cover them
  const int keys = a.chunk > 0 ? a.chunk : kAttnKeys;
  dim3 grid(std::min(a.max_splits, (a.ctx_bound + keys - 1) / keys), a.nh);
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
