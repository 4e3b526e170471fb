// eg_fused.cu -- persistent fused decode: K tokens of runtime.js:1466-1571
// (plus EMBED_BUF in front and ARGMAX behind) in ONE cooperative launch.
//
// Grid = one CTA per SM.  A token is a fixed sequence of phases -- per layer
// QKV, ATTN, O, GATE_UP, DOWN, then the LM head -- each split statically over
// the CTAs (16-row tiles of each matrix, (split, kv-head) attention items) and
// separated by a grid barrier.
//
// Inside a CTA, warp 8 is a producer: it walks the CTA's weight slices of the
// whole launch (every layer, every token) in consumption order and streams
// them with cp.async.bulk into a 4-stage shared-memory ring (32 KB per stage
// = 32 row segments of <= 1 KB), signalling an mbarrier per stage.  The
// weights do not depend on activations, so the producer never waits for a
// grid barrier: HBM keeps streaming the next phase's weights while the 8
// consumer warps wait, compute attention, or run epilogues.  Consumers turn
// the nibbles/bytes of each stage into m16n8k16 fragments (eg_common.cuh) and
// release the stage.
//
// Cross-CTA data (hidden, q/k/v, attention output, SiLU output, KV rows, token
// ids) is written before a grid barrier and read after it with ld.global.cg,
// so no stale L1 line is observed inside the launch.  Every wait (grid
// barrier, mbarrier) is bounded: on timeout the waiter records an error word,
// the other waits see it and give up, and the host reports EG_ERR_DEVICE.
#include <algorithm>

#include "eg_device.cuh"
#include "eg_fused.h"

namespace eg {

constexpr int kConsumerWarps = 8;                // == kCtaThreads / 32
constexpr int kFusedThreads = kCtaThreads + 32;  // + producer warp
constexpr int kStages = 4;
constexpr int kSegBytes = 1024;
constexpr int kSegs = 32;
constexpr int kScaleSeg = 96;                   // per-segment room for its row's group scales
constexpr int kStageBytes = kSegs * (kSegBytes + kScaleSeg);  // 32 KB weights + 3 KB scales
constexpr int kChunkK = 2048;                   // int4 k-values per 1 KB row segment

// ---------------------------------------------------------------- waits
// Monotonic arrival counter over the consumer groups of all CTAs: the k-th
// barrier completes when the counter reaches k * gridDim.x.  Returns false
// (uniformly for the consumer group) when the launch is being abandoned.
__device__ __forceinline__ bool grid_barrier(unsigned* bar, int* err, unsigned& epoch) {
  __shared__ int s_ok;
  cta_sync();
  if (threadIdx.x == 0) {
    epoch += 1;
    const unsigned target = epoch * gridDim.x;
    __threadfence();
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
    int ok = 1;
    for (long long spins = 0;; spins++) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
      if (v >= target) break;
      if ((spins & 255) == 0 && err_set(err)) {
        ok = 0;
        break;
      }
      if (spins > kSpinLimit) {
        atomicExch(err, 1);
        ok = 0;
        break;
      }
    }
    s_ok = ok && !err_set(err);
  }
  cta_sync();
  return s_ok != 0;
}

__device__ __forceinline__ void tile_range(int tiles, int& t0, int& t1) {
  t0 = (int)((long long)tiles * blockIdx.x / gridDim.x);
  t1 = (int)((long long)tiles * (blockIdx.x + 1) / gridDim.x);
}

// ---------------------------------------------------------------- units
// A "unit" fills one ring stage.  int4 phases: two 16-row slots (tiles a and
// a+1; gate/up: the gate tile and its up tile) x one 2048-wide k chunk;
// segment 16*slot + r holds row r's bytes of that chunk.  LM head (int8): one
// 16-row tile, segment 2r + h = row r's bytes [1024h, 1024h + 1024).
enum { P_QKV = 0, P_O = 1, P_GU = 2, P_DOWN = 3, P_LM = 4 };

struct Geo {
  const uint32_t* w;
  const float* s;
  int N, K;    // rows of one matrix half (gate/up: I), reduction length
  int t0, t1;  // this CTA's tiles
  int pair;    // 1: slots are tiles a, a+1; 0: gate/up halves (or LM)
  int nk;      // k chunks per slot pair
};

__device__ __forceinline__ Geo geo(const FusedArgs& a, const FusedLayer& l, int kind) {
  Geo g = {};
  switch (kind) {
    case P_QKV: g.w = l.qkv_w; g.s = l.qkv_s; g.N = a.QD + 2 * a.KVD; g.K = a.H; g.pair = 1; break;
    case P_O: g.w = l.o_w; g.s = l.o_s; g.N = a.H; g.K = a.QD; g.pair = 1; break;
    case P_GU: g.w = l.gu_w; g.s = l.gu_s; g.N = a.I; g.K = a.H; g.pair = 0; break;
    case P_DOWN: g.w = l.d_w; g.s = l.d_s; g.N = a.H; g.K = a.I; g.pair = 1; break;
    default: g.w = a.emb_w; g.s = a.emb_s; g.N = a.V; g.K = a.H; g.pair = 0; break;
  }
  tile_range((g.N + 15) / 16, g.t0, g.t1);
  g.nk = kind == P_LM ? 1 : (g.K + kChunkK - 1) / kChunkK;
  return g;
}

__device__ __forceinline__ int units_of(const Geo& g, int kind) {
  const int tiles = g.t1 - g.t0;
  if (kind == P_LM) return tiles;
  return (g.pair ? (tiles + 1) / 2 : tiles) * g.nk;
}

// Source and length of segment `seg` of unit u (bytes = 0: no segment).
__device__ __forceinline__ const char* seg_src(const Geo& g, int kind, int u, int seg,
                                               uint32_t& bytes) {
  bytes = 0;
  if (kind == P_LM) {
    const int row = (g.t0 + u) * 16 + (seg >> 1);
    if (row >= g.N) return nullptr;
    bytes = kSegBytes;
    return reinterpret_cast<const char*>(g.w) + (size_t)row * g.K + (seg & 1) * kSegBytes;
  }
  const int slot = seg >> 4, r = seg & 15;
  const int p = u / g.nk, k = u % g.nk;
  int row;
  if (g.pair) {
    const int tile = g.t0 + 2 * p + slot;
    if (tile >= g.t1) return nullptr;
    row = tile * 16 + r;
    if (row >= g.N) return nullptr;
  } else {
    row = (g.t0 + p) * 16 + r + (slot ? g.N : 0);
  }
  const int kb = k * kChunkK, ke = min(g.K, kb + kChunkK);
  bytes = (uint32_t)((ke - kb) / 2);
  return reinterpret_cast<const char*>(g.w) + (size_t)row * (g.K / 2) + kb / 2;
}

// Group scales of segment `seg`: an aligned span holding floats [G0, G0+ng)
// of the row's scale row starts `off` bytes into the copy (16-byte rules of
// cp.async.bulk).  LM head: segment 0 carries the tile's 16 row scales.
__device__ __forceinline__ const char* scale_src(const Geo& g, int kind, int u, int seg,
                                                 uint32_t& bytes, uint32_t& off) {
  bytes = 0;
  off = 0;
  if (kind == P_LM) {
    const int row0 = (g.t0 + u) * 16;
    if (seg != 0) return nullptr;
    const int rows = min(16, g.N - row0);
    bytes = (uint32_t)((rows * 4 + 15) & ~15);
    return reinterpret_cast<const char*>(g.s + row0);
  }
  const int slot = seg >> 4, r = seg & 15;
  const int p = u / g.nk, k = u % g.nk;
  int row;
  if (g.pair) {
    const int tile = g.t0 + 2 * p + slot;
    if (tile >= g.t1) return nullptr;
    row = tile * 16 + r;
    if (row >= g.N) return nullptr;
  } else {
    row = (g.t0 + p) * 16 + r + (slot ? g.N : 0);
  }
  const int gpr = g.K / kGroup;
  const int ng = min(16, gpr - k * 16);
  const size_t start = ((size_t)row * gpr + k * 16) * 4;
  const size_t a0 = start & ~size_t(15);
  off = (uint32_t)(start - a0);
  bytes = (uint32_t)((off + ng * 4 + 15) & ~15u);
  return reinterpret_cast<const char*>(g.s) + a0;
}

// Slots whose 16 rows are one contiguous span (K = 2048 int4, and every int8
// LM tile) move as one weight copy + one scale copy each: few large bulk
// copies instead of 32 row copies.
__device__ __forceinline__ bool contiguous(const Geo& g, int kind) {
  return kind == P_LM || (g.nk == 1 && g.K == kChunkK);
}
__device__ __forceinline__ int scale_stride(const Geo& g, int kind) {
  return contiguous(g, kind) ? 64 : kScaleSeg;
}

// Copy `c` (0..3) of a contiguous unit: c = slot (weights) or 2 + slot (scales).
__device__ __forceinline__ const char* contig_copy(const Geo& g, int kind, int u, int c,
                                                   uint32_t& bytes, uint32_t& dst) {
  bytes = 0;
  dst = 0;
  const int slot = c & 1;
  int row0, rows;
  if (kind == P_LM) {
    if (slot) return nullptr;
    row0 = (g.t0 + u) * 16;
    rows = min(16, g.N - row0);
    if (c < 2) {
      bytes = (uint32_t)rows * g.K;
      return reinterpret_cast<const char*>(g.w) + (size_t)row0 * g.K;
    }
    bytes = (uint32_t)((rows * 4 + 15) & ~15);
    dst = kSegs * kSegBytes;
    return reinterpret_cast<const char*>(g.s + row0);
  }
  if (g.pair) {
    const int tile = g.t0 + 2 * u + slot;
    if (tile >= g.t1) return nullptr;
    row0 = tile * 16;
    rows = min(16, g.N - row0);
  } else {
    row0 = (g.t0 + u) * 16 + (slot ? g.N : 0);
    rows = 16;
  }
  if (c < 2) {
    bytes = (uint32_t)rows * kSegBytes;
    dst = slot * 16 * kSegBytes;
    return reinterpret_cast<const char*>(g.w) + (size_t)row0 * kSegBytes;
  }
  bytes = (uint32_t)rows * 64;
  dst = kSegs * kSegBytes + slot * 16 * 64;
  return reinterpret_cast<const char*>(g.s + (size_t)row0 * 16);
}

__device__ __forceinline__ bool lm_runs(const FusedArgs& a, int tok) {
  return a.lm_every || tok == a.n_tokens - 1;
}

// ---------------------------------------------------------------- producer
// The CTA's unit sequence of the launch: per token, per layer QKV, O,
// GATE_UP, DOWN units, then the LM head's units when it runs.
struct UnitIter {
  int tok, li, kind, u, nu;
  Geo g;
  bool done;
};

__device__ __forceinline__ void iter_load(const FusedArgs& a, UnitIter& it) {
  for (;;) {
    if (it.tok >= a.n_tokens) {
      it.done = true;
      return;
    }
    const bool lm = it.li == a.layers_n;
    if (lm && !lm_runs(a, it.tok)) {  // no LM head for this token
      it.tok++;
      it.li = 0;
      it.kind = P_QKV;
      continue;
    }
    it.g = geo(a, a.layers[lm ? 0 : it.li], it.kind);
    it.nu = units_of(it.g, it.kind);
    if (it.nu > 0) return;
    // empty phase: step to the next one
    if (lm) {
      it.tok++;
      it.li = 0;
      it.kind = P_QKV;
    } else if (it.kind == P_DOWN) {
      it.li++;
      it.kind = it.li == a.layers_n ? P_LM : P_QKV;
    } else {
      it.kind++;
    }
  }
}

__device__ __forceinline__ void iter_begin(const FusedArgs& a, UnitIter& it) {
  it.tok = 0;
  it.li = 0;
  it.kind = P_QKV;
  it.u = 0;
  it.done = false;
  iter_load(a, it);
}

__device__ __forceinline__ void iter_next(const FusedArgs& a, UnitIter& it) {
  if (++it.u < it.nu) return;
  it.u = 0;
  if (it.kind == P_LM) {
    it.tok++;
    it.li = 0;
    it.kind = P_QKV;
  } else if (it.kind == P_DOWN) {
    it.li++;
    it.kind = it.li == a.layers_n ? P_LM : P_QKV;
  } else {
    it.kind++;
  }
  iter_load(a, it);
}

__device__ __forceinline__ void l2_prefetch(const void* p, uint32_t bytes) {
  if (!bytes) return;
  const uintptr_t a = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15);
  const uint32_t n = (uint32_t)((reinterpret_cast<uintptr_t>(p) + bytes - a + 15) & ~uintptr_t(15));
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
}

// Copy list of a unit: lane `lane` handles weight copy (src, bytes -> dst)
// and, for row-wise units, its row's scale span.
__device__ __forceinline__ void unit_copy(const UnitIter& it, int lane, const char*& src,
                                          uint32_t& bytes, uint32_t& dst, const char*& ssrc,
                                          uint32_t& sbytes) {
  uint32_t soff;
  ssrc = nullptr;
  sbytes = 0;
  dst = lane * kSegBytes;
  if (contiguous(it.g, it.kind)) {
    src = lane < 4 ? contig_copy(it.g, it.kind, it.u, lane, bytes, dst) : nullptr;
    if (lane >= 4) bytes = 0;
  } else {
    src = seg_src(it.g, it.kind, it.u, lane, bytes);
    ssrc = scale_src(it.g, it.kind, it.u, lane, sbytes, soff);
  }
}

__device__ void producer(const FusedArgs& a, unsigned char* ring, uint64_t* full, uint64_t* empty) {
  const int lane = threadIdx.x & 31;
  UnitIter it, ahead;
  iter_begin(a, it);
  iter_begin(a, ahead);
  // the L2 prefetch cursor runs l2_ahead units in front of the ring
  for (int i = 0; i < a.l2_ahead && !ahead.done; i++) {
    const char *src, *ssrc;
    uint32_t bytes, dst, sbytes;
    unit_copy(ahead, lane, src, bytes, dst, ssrc, sbytes);
    if (bytes) l2_prefetch(src, bytes);
    if (sbytes) l2_prefetch(ssrc, sbytes);
    iter_next(a, ahead);
  }
  for (uint32_t n = 0; !it.done; n++, iter_next(a, it)) {
    if (!ahead.done) {
      const char *src, *ssrc;
      uint32_t bytes, dst, sbytes;
      unit_copy(ahead, lane, src, bytes, dst, ssrc, sbytes);
      if (bytes) l2_prefetch(src, bytes);
      if (sbytes) l2_prefetch(ssrc, sbytes);
      iter_next(a, ahead);
    }
    const int st = n % kStages;
    const uint32_t round = n / kStages;
    if (!mbar_wait(&empty[st], (round & 1) ^ 1, a.err)) return;
    const char *src, *ssrc;
    uint32_t bytes, dst, sbytes;
    unit_copy(it, lane, src, bytes, dst, ssrc, sbytes);
    if (a.diag == 1) bytes = sbytes = 0;
    uint32_t total = bytes + sbytes;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (lane == 0)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                       smem_addr(&full[st])),
                   "r"(total)
                   : "memory");
    __syncwarp();
    unsigned char* stage = ring + (size_t)st * kStageBytes;
    if (bytes)
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
          "[%3];" ::"r"(smem_addr(stage + dst)),
          "l"(src), "r"(bytes), "r"(smem_addr(&full[st]))
          : "memory");
    if (sbytes)
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
          "[%3];" ::"r"(smem_addr(stage + kSegs * kSegBytes + lane * kScaleSeg)),
          "l"(ssrc), "r"(sbytes), "r"(smem_addr(&full[st]))
          : "memory");
  }
}

// ---------------------------------------------------------------- consumers
// Ring position of the consumer group (same unit sequence as the producer).
struct Cursor {
  uint32_t n;
};

// An int4 GEMV phase: all of this CTA's units, epilogue per completed slot pair.
__device__ __forceinline__ void slot_rows(const Geo& g, int p, int slot, int& rbase, bool& valid) {
  if (g.pair) {
    const int tile = g.t0 + 2 * p + slot;
    valid = tile < g.t1;
    rbase = tile * 16;
  } else {
    valid = true;
    rbase = (g.t0 + p) * 16 + (slot ? g.N : 0);
  }
}

template <int MAXU, bool NORM>
__device__ __forceinline__ void gemv4_phase(const FusedArgs& a, const Geo g, int kind, Cursor& cur,
                                            const unsigned char* ring, uint64_t* full,
                                            uint64_t* empty, const XSrc& xsrc, uint4* xs_base,
                                            float* sred, float (*red)[kConsumerWarps][2][16],
                                            const Epi& epi) {
  const int nu = units_of(g, kind);
  // epilogue thread (slot, i): row of the first unit, its residual/bias read now
  const int eslot = threadIdx.x >> 4, ei = threadIdx.x & 15;
  float pre = 0.f;
  if (threadIdx.x < 32 && nu) {
    int rb;
    bool ok;
    slot_rows(g, 0, eslot, rb, ok);
    if (ok && (g.pair || eslot == 0)) pre = epi_pre(epi, rb + ei);
  }
  const int e = stage_x<MAXU, NORM>(xsrc, g.K, 4, xs_base, sred);
  mark(1);
  if (!nu) return;
  const int K8 = g.K / 8, gpr = g.K / kGroup;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, t = lane & 3;
  const uint4* xs = gq == 0 ? xs_base : xs_base + K8 + 4;
  const bool bl = gq < 2;
  const int sstr = scale_stride(g, kind);
  float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  int pairs_done = 0;
  for (int u = 0; u < nu; u++, cur.n++) {
    const int p = u / g.nk, k = u % g.nk;
    const int ng = min(16, (g.K - k * kChunkK) / kGroup);
    int rbase[2];
    bool sv[2];
    slot_rows(g, p, 0, rbase[0], sv[0]);
    slot_rows(g, p, 1, rbase[1], sv[1]);
    bool gv[2];
#pragma unroll
    for (int i = 0; i < 2; i++) gv[i] = warp + 8 * i < ng && a.diag != 2;
    const int st = cur.n % kStages;
    if (a.diag != 3) mbar_wait(&full[st], (cur.n / kStages) & 1, a.err);
    if (u == 0) mark(2);
    const unsigned char* stage = ring + (size_t)st * kStageBytes;
    const unsigned char* sstage = stage + kSegs * kSegBytes;
    // this warp's two groups in turn, 4 independent accumulator chains each
    float sa[2][2], sb[2][2];
    if (t == 0) {
#pragma unroll
      for (int i = 0; i < 2; i++)
#pragma unroll
        for (int slot = 0; slot < 2; slot++) {
          const int Gl = warp + 8 * i;
          const int ra = rbase[slot] + gq, rb = ra + 8;
          const int oa = sstr == kScaleSeg ? (int)((((size_t)ra * gpr + k * 16) * 4) & 15) : 0;
          const int ob = sstr == kScaleSeg ? (int)((((size_t)rb * gpr + k * 16) * 4) & 15) : 0;
          const bool ok = gv[i] && sv[slot];
          sa[i][slot] = ok ? *reinterpret_cast<const float*>(sstage + (16 * slot + gq) * sstr + oa + 4 * Gl) : 0.f;
          sb[i][slot] = ok ? *reinterpret_cast<const float*>(sstage + (16 * slot + gq + 8) * sstr + ob + 4 * Gl) : 0.f;
        }
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
      if (!gv[i]) continue;
      const int Gl = warp + 8 * i;
      uint4 X[4];
#pragma unroll
      for (int j = 0; j < 4; j++) X[j] = bl ? xs[16 * (k * 16 + Gl) + 4 * j + t] : make_uint4(0, 0, 0, 0);
      uint4 A[2], B[2];
#pragma unroll
      for (int slot = 0; slot < 2; slot++) {
        const unsigned char* ra = stage + (16 * slot + gq) * kSegBytes + Gl * 64 + t * 16;
        A[slot] = sv[slot] ? *reinterpret_cast<const uint4*>(ra) : make_uint4(0, 0, 0, 0);
        B[slot] = sv[slot] ? *reinterpret_cast<const uint4*>(ra + 8 * kSegBytes) : make_uint4(0, 0, 0, 0);
      }
      float c[2][2][4];
#pragma unroll
      for (int slot = 0; slot < 2; slot++)
#pragma unroll
        for (int h = 0; h < 2; h++) c[slot][h][0] = c[slot][h][1] = c[slot][h][2] = c[slot][h][3] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int slot = 0; slot < 2; slot++) {
          const uint32_t wa = j == 0 ? A[slot].x : j == 1 ? A[slot].y : j == 2 ? A[slot].z : A[slot].w;
          const uint32_t wb = j == 0 ? B[slot].x : j == 1 ? B[slot].y : j == 2 ? B[slot].z : B[slot].w;
          uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
          deq_int4(wa, a0, a1, a2, a3);
          deq_int4(wb, b0, b1, b2, b3);
          mma16816(c[slot][j & 1], a0, b0, a1, b1, X[j].x, X[j].y);
          mma16816(c[slot][j & 1], a2, b2, a3, b3, X[j].z, X[j].w);
        }
      if (t == 0) {
#pragma unroll
        for (int slot = 0; slot < 2; slot++) {
          const float* c0 = c[slot][0];
          const float* c1 = c[slot][1];
          acc[slot][0] = fmaf(sa[i][slot], (c0[0] + c1[0]) + (c0[1] + c1[1]), acc[slot][0]);
          acc[slot][1] = fmaf(sb[i][slot], (c0[2] + c1[2]) + (c0[3] + c1[3]), acc[slot][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
    if (u == nu - 1) mark(3);
    if (k == g.nk - 1) {  // slot pair complete: reduce over warps, epilogue
      float (*rb)[2][16] = red[pairs_done & 1];  // double buffered: one barrier per pair
      if (t == 0) {
#pragma unroll
        for (int slot = 0; slot < 2; slot++) {
          rb[warp][slot][gq] = acc[slot][0];
          rb[warp][slot][gq + 8] = acc[slot][1];
        }
      }
      acc[0][0] = acc[0][1] = acc[1][0] = acc[1][1] = 0.f;
      cta_sync();
      if (threadIdx.x < 32) {
        int rbs;
        bool ok;
        slot_rows(g, p, eslot, rbs, ok);
        float v0 = 0.f, v1 = 0.f;
        for (int ww = 0; ww < kConsumerWarps; ww++) {
          v0 += rb[ww][0][ei];
          v1 += rb[ww][1][ei];
        }
        if (e) {
          v0 = ldexpf(v0, e);
          v1 = ldexpf(v1, e);
        }
        if (pairs_done > 0 && ok && (g.pair || eslot == 0)) pre = epi_pre(epi, rbs + ei);
        if (g.pair) {
          if (ok) epilogue_row_pre(epi, rbs + ei, eslot ? v1 : v0, 0.f, pre);
        } else if (eslot == 0) {
          epilogue_row_pre(epi, rbs + ei, v0, v1, pre);  // gate, up
        }
      }
      pairs_done++;
    }
  }
  cta_sync();
}

// int8 LM head phase + this CTA's argmax candidate.
__device__ __forceinline__ void lm_phase(const FusedArgs& a, const Geo g, Cursor& cur, const unsigned char* ring,
                         uint64_t* full, uint64_t* empty, uint2* xs2_base, float* sred,
                         float (*red)[2][16], float& bv, uint32_t& bi) {
  XSrc xf = {};
  xf.mode = X_RMS;
  xf.x = a.hidden;
  xf.norm_g = a.final_norm;
  xf.eps = a.eps;
  xf.f16 = a.f16;
  const int e = stage_x<1>(xf, a.H, 8, xs2_base, sred);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, t = lane & 3;
  const uint2* xs = gq == 0 ? xs2_base : xs2_base + a.H / 4 + 2;
  const bool bl = gq < 2;
  const int nch = a.H / 64;
  const int nu = units_of(g, P_LM);
  for (int u = 0; u < nu; u++, cur.n++) {
    const int tile = g.t0 + u;
    const int n = tile * 16 + threadIdx.x;
    const int st = cur.n % kStages;
    if (a.diag != 3) mbar_wait(&full[st], (cur.n / kStages) & 1, a.err);
    const unsigned char* stage = ring + (size_t)st * kStageBytes;
    const float srow = threadIdx.x < 16 && n < a.V
                           ? *reinterpret_cast<const float*>(stage + kSegs * kSegBytes + 4 * threadIdx.x)
                           : 0.f;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    for (int Ch = warp; Ch < (a.diag == 2 ? 0 : nch); Ch += kConsumerWarps) {
      const int off = (Ch & 15) * 64 + t * 16, h = Ch >> 4;
      const uint4 A = *reinterpret_cast<const uint4*>(stage + (2 * gq + h) * kSegBytes + off);
      const uint4 B = *reinterpret_cast<const uint4*>(stage + (2 * (gq + 8) + h) * kSegBytes + off);
      const uint4* xp = reinterpret_cast<const uint4*>(xs + 16 * Ch + 4 * t);
      const uint4 x01 = bl ? xp[0] : make_uint4(0, 0, 0, 0);
      const uint4 x23 = bl ? xp[1] : make_uint4(0, 0, 0, 0);
      uint32_t a0, a1, b0, b1;
      deq_int8(A.x, a0, a1);
      deq_int8(B.x, b0, b1);
      mma16816(c, a0, b0, a1, b1, x01.x, x01.y);
      deq_int8(A.y, a0, a1);
      deq_int8(B.y, b0, b1);
      mma16816(c, a0, b0, a1, b1, x01.z, x01.w);
      deq_int8(A.z, a0, a1);
      deq_int8(B.z, b0, b1);
      mma16816(c, a0, b0, a1, b1, x23.x, x23.y);
      deq_int8(A.w, a0, a1);
      deq_int8(B.w, b0, b1);
      mma16816(c, a0, b0, a1, b1, x23.z, x23.w);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (t == 0) {
      red[warp][0][gq] = c[0] + c[1];
      red[warp][0][gq + 8] = c[2] + c[3];
    }
    cta_sync();
    if (threadIdx.x < 16) {
      float aa = 0.f;
      for (int ww = 0; ww < kConsumerWarps; ww++) aa += red[ww][0][threadIdx.x];
      if (n < a.V) {
        const float o = __fmul_rn(e ? ldexpf(aa, e) : aa, srow);  // sum first, scale last
        a.logits[n] = o;
        if (beats(o, (uint32_t)n, bv, bi)) {
          bv = o;
          bi = (uint32_t)n;
        }
      }
    }
    cta_sync();
  }
}

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Phase profile hooks (token 0 only; no-ops unless a.prof is set).
__device__ __forceinline__ void prof_start(const FusedArgs& a, int tok, int ph) {
  if (a.prof && tok == 0 && blockIdx.x == 0 && threadIdx.x == 0) a.prof[2 * ph] = gtime();
  // intra-phase marks: layer 2 of token 0, on CTA 1 (holds a tile of every matrix)
  if (threadIdx.x == 0) s_mark_base = (tok == 0 && ph / 5 == 2 && blockIdx.x == 1) ? (ph % 5) * 16 : -1;
  mark(0);
}
__device__ __forceinline__ void prof_end(const FusedArgs& a, int tok, int ph) {
  mark(15);
  if (a.prof && tok == 0) {
    cta_sync();
    if (threadIdx.x == 0) atomicMax(a.prof + 2 * ph + 1, gtime());
  }
}

// ---------------------------------------------------------------- the kernel
template <typename KVT>
__global__ void __launch_bounds__(kFusedThreads, 1) fused_decode_kernel(FusedArgs a) {
  extern __shared__ __align__(1024) unsigned char dsm[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ float sred[32];
  __shared__ float red[2][kConsumerWarps][2][16];
  __shared__ float best_v[kConsumerWarps];
  __shared__ uint32_t best_i[kConsumerWarps];
  __shared__ int last_cta;
  unsigned char* ring = dsm;
  unsigned char* scratch = dsm + kStages * kStageBytes;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&full[i])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(&empty[i])),
                   "r"(kConsumerWarps)
                   : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x >= kCtaThreads) {  // producer warp
    if (a.diag != 3) producer(a, ring, full, empty);
    return;
  }

  unsigned epoch = 0;
  Cursor cur{0};
  const int L = a.layers_n, H = a.H, QD = a.QD, KVD = a.KVD, I = a.I;
  const int NQKV = QD + 2 * KVD;
  uint4* xs = reinterpret_cast<uint4*>(scratch);
  for (int tok = 0; tok < a.n_tokens; tok++) {
    const int pos = a.start_pos + tok;
    for (int li = 0; li < L; li++) {
      const FusedLayer& l = a.layers[li];
      const int ph = li * 5;
      // ---- QKV: (embed +) RMSNorm prologue, q/k/v rows + bias
      prof_start(a, tok, ph);
      {
        XSrc xa = {};
        xa.mode = li == 0 ? X_EMBED_RMS : X_RMS;
        xa.x = a.hidden;
        xa.norm_g = l.in_norm;
        xa.eps = a.eps;
        xa.f16 = a.f16;
        xa.emb_w = a.emb_w;
        xa.emb_s = a.emb_s;
        xa.ids = a.ids;
        xa.fixed_pos = pos;
        xa.hidden_out = a.hidden;
        Epi ep = {};
        ep.mode = EPI_STORE;
        ep.y = a.qkv;
        ep.bias = l.qkv_b;
        ep.N = NQKV;
        ep.split1 = ep.split2 = NQKV;
        gemv4_phase<1, true>(a, geo(a, l, P_QKV), P_QKV, cur, ring, full, empty, xa, xs, sred, red, ep);
      }
      prof_end(a, tok, ph);
      if (!grid_barrier(a.bar, a.err, epoch)) return;
      // ---- attention: RoPE, KV append, split-K, last-item combine
      prof_start(a, tok, ph + 1);
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
        at.kv_f16 = a.f16;
        at.chunk = a.attn_chunk;
        at.pm = a.pm;
        at.pz = a.pz;
        at.po = a.po;
        at.out = a.attn;
        at.counters = a.attn_counters;
        const int chunk = attn_chunk(pos + 1, a.attn_chunk);
        const int ns = (pos + chunk) / chunk;
        for (int it = blockIdx.x; it < ns * a.nkv; it += gridDim.x)
          attn_item<KVT>(at, it % ns, it / ns, reinterpret_cast<float*>(scratch), 0);
      }
      prof_end(a, tok, ph + 1);
      if (!grid_barrier(a.bar, a.err, epoch)) return;
      // ---- O projection + residual
      prof_start(a, tok, ph + 2);
      {
        XSrc xo = {};
        xo.mode = X_PLAIN;
        xo.x = a.attn;
        Epi ep = {};
        ep.mode = EPI_ADD;
        ep.y = a.hidden;
        ep.N = H;
        ep.split1 = ep.split2 = H;
        gemv4_phase<1, false>(a, geo(a, l, P_O), P_O, cur, ring, full, empty, xo, xs, sred, red, ep);
      }
      prof_end(a, tok, ph + 2);
      if (!grid_barrier(a.bar, a.err, epoch)) return;
      // ---- gate/up + SiLU
      prof_start(a, tok, ph + 3);
      {
        XSrc xb = {};
        xb.mode = X_RMS;
        xb.x = a.hidden;
        xb.norm_g = l.post_norm;
        xb.eps = a.eps;
        xb.f16 = a.f16;
        Epi ep = {};
        ep.mode = EPI_SILU;
        ep.y = a.tmp;
        ep.N = I;
        gemv4_phase<1, true>(a, geo(a, l, P_GU), P_GU, cur, ring, full, empty, xb, xs, sred, red, ep);
      }
      prof_end(a, tok, ph + 3);
      if (!grid_barrier(a.bar, a.err, epoch)) return;
      // ---- down projection + residual
      prof_start(a, tok, ph + 4);
      {
        XSrc xd = {};
        xd.mode = X_PLAIN;
        xd.x = a.tmp;
        Epi ep = {};
        ep.mode = EPI_ADD;
        ep.y = a.hidden;
        ep.N = H;
        ep.split1 = ep.split2 = H;
        gemv4_phase<6, false>(a, geo(a, l, P_DOWN), P_DOWN, cur, ring, full, empty, xd, xs, sred, red, ep);
      }
      prof_end(a, tok, ph + 4);
      if (!grid_barrier(a.bar, a.err, epoch)) return;
    }
    // ---- LM head (int8 rows) + argmax + token advance
    if (!lm_runs(a, tok)) continue;
    prof_start(a, tok, 5 * L);
    float bv = -1e30f;
    uint32_t bi = 0xffffffffu;
    lm_phase(a, geo(a, a.layers[0], P_LM), cur, ring, full, empty, reinterpret_cast<uint2*>(scratch),
             sred, red[0], bv, bi);
    if (a.greedy) {
      // per-CTA best, then the last CTA to arrive reduces (ARGMAX, kernels.js:771-784)
      block_best(bv, bi, best_v, best_i);
      if (threadIdx.x == 0) {
        a.cand_v[blockIdx.x] = bv;
        a.cand_i[blockIdx.x] = bi;
        __threadfence();
        last_cta = atomicAdd(a.lm_counter, 1u) == gridDim.x - 1;
      }
      cta_sync();
      if (last_cta) {
        __threadfence();
        float v = -1e30f;
        uint32_t id = 0xffffffffu;
        for (int b = threadIdx.x; b < (int)gridDim.x; b += kCtaThreads) {
          const float cv = __ldcg(a.cand_v + b);
          const uint32_t ci = __ldcg(a.cand_i + b);
          if (beats(cv, ci, v, id)) {
            v = cv;
            id = ci;
          }
        }
        block_best(v, id, best_v, best_i);
        if (threadIdx.x == 0) {
          *a.amax = id;
          a.ids[pos + 1] = id;
          a.out_ids[tok] = id;
          *a.lm_counter = 0u;
          __threadfence();
        }
      }
    }
    prof_end(a, tok, 5 * L);
    if (tok + 1 < a.n_tokens && !grid_barrier(a.bar, a.err, epoch)) return;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) a.state_pos[0] = a.start_pos + a.n_tokens;
}

cudaError_t fused_set_marks(unsigned long long* buf) {
  return cudaMemcpyToSymbol(g_marks, &buf, sizeof(buf));
}

int fused_smem_bytes() {
  const int attn = kAttnMaxChunk * (kKsStride + kHeadDim) * (int)sizeof(float);
  const int frag = (2 * (12288 / 8) + 8) * (int)sizeof(uint4);
  return kStages * kStageBytes + std::max(attn, frag);
}

cudaError_t fused_decode(const FusedArgs& a, cudaStream_t st) {
  const int smem = fused_smem_bytes();
  void (*k)(FusedArgs) = a.f16 ? fused_decode_kernel<__half> : fused_decode_kernel<float>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kFusedThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
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
  return cudaLaunchKernelEx(&cfg, k, a);
}

}  // namespace eg
