// eg_stream.cuh -- streaming GEMV building blocks (ring producer, integer-MMA
// consumers, epilogue warp) and the decode-attention item, shared by the
// per-op kernels (eg_kernels.cu) and the persistent decode kernel
// (eg_fused.cu).
//
// A "run" is a contiguous range of tiles [t_lo, t_hi) of one stream-layout
// matrix (gpr 128-wide groups per tile, one block per (tile, group)); in the
// stream layout it is one contiguous byte range.  The producer warp copies a
// run into the shared-memory ring, `cap` blocks per stage (one
// cp.async.bulk); consumer warp w (of CW) takes the run's blocks w, w + CW,
// w + 2 CW, ... and keeps one running sum per row pair; at the end of each tile
// every consumer warp leaves its partial row sums in red[tj & 1] and the
// epilogue warp sums them and writes the outputs.  Ring positions (stage,
// phase) and the tile hand-off counter tj carry over from one run to the
// next, so a persistent kernel can chain runs of different matrices through
// one ring; every warp walks the same run sequence.
#pragma once
#include "eg_device.cuh"

namespace eg {

// A streaming GEMV CTA: CW consumer warps (a template parameter), then one
// producer warp and one epilogue warp.

// int4 block: R row sets x (1024 bytes of nibbles in fragment order), then
// the 16 R f32 group scales as (row i, row i + 8) pairs; int8 block: 16 rows x
// 128 bytes in fragment order.
__host__ __device__ constexpr int q4_block_bytes(int R) { return R * 1088; }
constexpr int kQ8Block = 2048;

struct RingPos {
  int st, ph;
};

__device__ __forceinline__ void ring_advance(RingPos& rp, int stages) {
  if (++rp.st == stages) {
    rp.st = 0;
    rp.ph ^= 1;
  }
}

// This CTA's slice of an L2 prefetch of [pf, pf + bytes) (16-byte aligned
// pieces of at most 64 KB), issued by one thread.
__device__ __forceinline__ void l2_prefetch_slice(const unsigned char* pf, size_t bytes) {
  if (!pf || !bytes) return;
  const size_t P = gridDim.x, c = blockIdx.x;
  const size_t lo = (bytes * c / P) & ~(size_t)15;
  const size_t hi = c + 1 == P ? bytes & ~(size_t)15 : (bytes * (c + 1) / P) & ~(size_t)15;
  for (size_t o = lo; o < hi; o += 65536) {
    const uint32_t n = (uint32_t)min((size_t)65536, hi - o);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(pf + o), "r"(n) : "memory");
  }
}

// Producer (one warp): one run of nitems blocks of blk bytes from src0.
// pf / pf_bytes (optional): a later kernel's weights to prefetch into L2,
// this CTA's slice issued right after the ring's first fill.
// Returns false when a wait gave up (error recorded).
__device__ __forceinline__ bool ring_produce(unsigned char* ring, uint64_t* full, uint64_t* empty,
                                             int stages, int stage_bytes,
                                             const unsigned char* src0, int nitems, int cap,
                                             int blk, RingPos& rp, int& issued, int* err,
                                             int lane, const unsigned char* pf = nullptr,
                                             size_t pf_bytes = 0) {
  const int nchunks = (nitems + cap - 1) / cap;
  const int fill = min(stages, nchunks);
  if (nchunks == 0 && lane == 0) l2_prefetch_slice(pf, pf_bytes);
  for (int n = 0; n < nchunks; n++) {
    if (!mbar_wait(&empty[rp.st], rp.ph ^ 1, err)) return false;
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)(min(cap, nitems - n * cap) * blk);
      mbar_expect_tx(&full[rp.st], bytes);
      bulk_g2s(ring + (size_t)rp.st * stage_bytes, src0 + (size_t)n * cap * blk, bytes,
               &full[rp.st]);
      if (n == fill - 1) l2_prefetch_slice(pf, pf_bytes);
    }
    __syncwarp();
    issued++;
    ring_advance(rp, stages);
  }
  return true;
}

// Producer exit: the last (up to `stages`) copies issued have landed, so the
// CTA never exits with a bulk copy in flight (bounded even after an error).
__device__ __forceinline__ void ring_drain(uint64_t* full, int stages, RingPos rp, int issued) {
  for (int k = 0; k < stages && k < issued; k++) {
    // step back one stage
    if (rp.st == 0) {
      rp.st = stages - 1;
      rp.ph ^= 1;
    } else {
      rp.st--;
    }
    if (!mbar_wait_bounded(&full[rp.st], rp.ph)) break;
  }
}

// Tile hand-off area of the consumers and the epilogue warp.
template <int CW, int R>
struct TileRed {
  float v[2][CW][R][16];
};

// Consumer side of one hand-off: sum the lanes t = 0, 1, publish the warp's
// partial rows in red[tj & 1] once the epilogue warp released that buffer.
// sc0 / sc1: the final factor of lanes t = 0 / t = 1 (column pairs 0 / 1).
template <int CW, int R>
__device__ __forceinline__ void tile_handoff(TileRed<CW, R>& red, uint64_t* tile_full,
                                             uint64_t* tile_free, int tj, float (&acc)[R][2],
                                             float sc0, float sc1, bool& dead, int* err) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, t = lane & 3;
  const float sc = t ? sc1 : sc0;
#pragma unroll
  for (int r = 0; r < R; r++) {
    acc[r][0] *= sc;
    acc[r][1] *= sc;
  }
#pragma unroll
  for (int r = 0; r < R; r++) {
    acc[r][0] += __shfl_xor_sync(0xffffffffu, acc[r][0], 1);
    acc[r][1] += __shfl_xor_sync(0xffffffffu, acc[r][1], 1);
  }
  const int b = tj & 1;
  if (!dead && !mbar_wait(&tile_free[b], ((tj >> 1) & 1) ^ 1, err)) dead = true;
  if (t == 0) {
#pragma unroll
    for (int r = 0; r < R; r++) {
      red.v[b][warp][r][gq] = acc[r][0];
      red.v[b][warp][r][gq + 8] = acc[r][1];
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++) acc[r][0] = acc[r][1] = 0.f;
  __syncwarp();
  if (lane == 0) mbar_arrive(&tile_full[b]);
}

// Consumers (warps 0 .. CW-1) of one int4 run.  xb / xcor / xf: the staged
// activation (stage_xd).  Lanes gq >= 4 feed B columns 4-7, whose results are never
// used: they load a copy of plane gq & 3 instead of a zero (no predication).  After a failed wait a warp goes on without waiting
// (its results are void; the host sees the error word).
template <int CW, int R>
__device__ void consume_q4_run(const unsigned char* ring, uint64_t* full, uint64_t* empty,
                               int stages, int stage_bytes, int cap, int t_lo, int t_hi, int gpr,
                               const uint2* xb, const int* xcor, const int* xf,
                               TileRed<CW, R>& red, uint64_t* tile_full, uint64_t* tile_free,
                               RingPos& rp, int& tj, bool& dead, int* err) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, t = lane & 3;
  const int blk = q4_block_bytes(R);
  const int nitems = (t_hi - t_lo) * gpr;
  const int nchunks = (nitems + cap - 1) / cap;
  if (nchunks == 0) return;
  float acc[R][2];
#pragma unroll
  for (int r = 0; r < R; r++) acc[r][0] = acc[r][1] = 0.f;
  const int f = *xf;
  const float sc0 = __int_as_float((127 - f) << 23), sc1 = __int_as_float((143 - f) << 23);
  int chunk = 0, chunk_lo = 0;
  if (!dead && !mbar_wait(&full[rp.st], rp.ph, err)) dead = true;
  const unsigned char* stage = ring + (size_t)rp.st * stage_bytes;
  int i = warp;  // block index within the run
  for (int j = 0; j < t_hi - t_lo; j++) {
    const int tile_end = (j + 1) * gpr;
    for (; i < tile_end; i += CW) {
      while (i >= chunk_lo + cap) {  // next stage
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[rp.st]);
        ring_advance(rp, stages);
        chunk++;
        chunk_lo += cap;
        stage = ring + (size_t)rp.st * stage_bytes;
        if (!dead && !mbar_wait(&full[rp.st], rp.ph, err)) dead = true;
      }
      const int g = i - j * gpr;
      const unsigned char* bp = stage + (size_t)(i - chunk_lo) * blk;
      // B: digit plane gq & 3 of this group's 4 k32 blocks
      const uint4* xp = reinterpret_cast<const uint4*>(xb + ((g * 4 + (gq & 3)) * 4 + t) * 4);
      const uint4 X0 = xp[0], X1 = xp[1];
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
        imma16832(cc[r], nib_lo_u8(A[r].x), nib_lo_u8(B[r].x), nib_hi16_u8(A[r].x), nib_hi16_u8(B[r].x), X0.x, X0.y);
        imma16832(cc[r], nib_lo_u8(A[r].y), nib_lo_u8(B[r].y), nib_hi16_u8(A[r].y), nib_hi16_u8(B[r].y), X0.z, X0.w);
        imma16832(cc[r], nib_lo_u8(A[r].z), nib_lo_u8(B[r].z), nib_hi16_u8(A[r].z), nib_hi16_u8(B[r].z), X1.x, X1.y);
        imma16832(cc[r], nib_lo_u8(A[r].w), nib_lo_u8(B[r].w), nib_hi16_u8(A[r].w), nib_hi16_u8(B[r].w), X1.z, X1.w);
      }
      if (t < 2) {  // columns 2t, 2t+1 = digit planes 2t, 2t+1
        const int cor = xcor[2 * g + t];
        const float2* sc = reinterpret_cast<const float2*>(bp + R * 1024);  // (row gq, row gq+8)
#pragma unroll
        for (int r = 0; r < R; r++) {
          const float2 s2 = sc[8 * r + gq];
          acc[r][0] = fmaf(s2.x, (float)(cc[r][0] + 256 * cc[r][1] - cor), acc[r][0]);
          acc[r][1] = fmaf(s2.y, (float)(cc[r][2] + 256 * cc[r][3] - cor), acc[r][1]);
        }
      }
    }
    tile_handoff<CW, R>(red, tile_full, tile_free, tj, acc, sc0, sc1, dead, err);
    tj++;
  }
  // release the current stage and wait/release the later ones this warp had
  // no blocks in, so every stage sees all CW arrivals
  for (; chunk < nchunks; chunk++) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[rp.st]);
    ring_advance(rp, stages);
    if (chunk + 1 < nchunks && !dead && !mbar_wait(&full[rp.st], rp.ph, err)) dead = true;
  }
}

// Consumers of one int8 run (m16n8k32 s8.s8; xb as uint32 [G][p][t][m][2]
// from stage_xd8; no offset correction).
template <int CW>
__device__ void consume_q8_run(const unsigned char* ring, uint64_t* full, uint64_t* empty,
                               int stages, int stage_bytes, int cap, int t_lo, int t_hi, int gpr,
                               const uint32_t* xb, const float* xmul, TileRed<CW, 1>& red,
                               uint64_t* tile_full, uint64_t* tile_free, RingPos& rp, int& tj,
                               bool& dead, int* err) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, t = lane & 3;
  const int nitems = (t_hi - t_lo) * gpr;
  const int nchunks = (nitems + cap - 1) / cap;
  if (nchunks == 0) return;
  float acc[1][2] = {{0.f, 0.f}};
  int chunk = 0, chunk_lo = 0;
  if (!dead && !mbar_wait(&full[rp.st], rp.ph, err)) dead = true;
  const unsigned char* stage = ring + (size_t)rp.st * stage_bytes;
  int i = warp;
  for (int j = 0; j < t_hi - t_lo; j++) {
    const int tile_end = (j + 1) * gpr;
    for (; i < tile_end; i += CW) {
      while (i >= chunk_lo + cap) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[rp.st]);
        ring_advance(rp, stages);
        chunk++;
        chunk_lo += cap;
        stage = ring + (size_t)rp.st * stage_bytes;
        if (!dead && !mbar_wait(&full[rp.st], rp.ph, err)) dead = true;
      }
      const int g = i - j * gpr;
      const unsigned char* bp = stage + (size_t)(i - chunk_lo) * kQ8Block;
      // B: plane gq & 3 (columns 4-7 unused, as in consume_q4_run)
      const uint4* xp = reinterpret_cast<const uint4*>(xb + ((g * 4 + (gq & 3)) * 4 + t) * 8);
      const uint4 X0 = xp[0], X1 = xp[1];
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
        acc[0][0] = fmaf(mul, (float)(cc[0] + 256 * cc[1]), acc[0][0]);
        acc[0][1] = fmaf(mul, (float)(cc[2] + 256 * cc[3]), acc[0][1]);
      }
    }
    tile_handoff<CW, 1>(red, tile_full, tile_free, tj, acc, 1.f, 1.f, dead, err);
    tj++;
  }
  for (; chunk < nchunks; chunk++) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[rp.st]);
    ring_advance(rp, stages);
    if (chunk + 1 < nchunks && !dead && !mbar_wait(&full[rp.st], rp.ph, err)) dead = true;
  }
}

// Epilogue warp of one int4 run: per tile, sum the consumer partials and run
// the epilogue (scale already applied; bias / residual / SiLU / LoRA here).
// pre_ok: the first tile's residual / bias may be read before its hand-off
// (false when the inputs of this run are only ordered by that hand-off).
template <int CW, int R>
__device__ bool epilogue_q4_run(const Epi& e, int t_lo, int t_hi, TileRed<CW, R>& red,
                                uint64_t* tile_full, uint64_t* tile_free, int& tj, bool pre_ok,
                                int* err) {
  const int lane = threadIdx.x & 31;
  const bool lora = e.mods != nullptr;
  float pre = 0.f;
  if (pre_ok && lane < 16 && !lora && t_lo < t_hi) pre = epi_pre(e, t_lo * 16 + lane);
  for (int tile = t_lo; tile < t_hi; tile++, tj++) {
    const int b = tj & 1;
    if (!mbar_wait(&tile_full[b], (tj >> 1) & 1, err)) return false;
    if (!pre_ok && tile == t_lo && lane < 16 && !lora) pre = epi_pre(e, tile * 16 + lane);
    float v = 0.f;
    if (lane < 16 * R)
      for (int ww = 0; ww < CW; ww++) v += red.v[b][ww][lane >> 4][lane & 15];
    __syncwarp();
    if (lane == 0) mbar_arrive(&tile_free[b]);
    const float up = __shfl_down_sync(0xffffffffu, v, 16);
    if (lane < 16) {
      const int row = tile * 16 + lane;
      if (lora)
        epilogue_row(e, row, v, R == 2 ? up : 0.f);
      else
        epilogue_row_pre(e, row, v, R == 2 ? up : 0.f, pre);
      if (!lora && tile + 1 < t_hi) pre = epi_pre(e, row + 16);
    }
  }
  return true;
}

// Epilogue warp of one int8 run: y[n] = row sum * s[n] (sum first, scale
// last) and the warp's best (value, index) in the reference's order.
template <int CW>
__device__ bool epilogue_q8_run(const float* s, float* y, int N, int t_lo, int t_hi,
                                TileRed<CW, 1>& red, uint64_t* tile_full, uint64_t* tile_free,
                                int& tj, float& bv, uint32_t& bi, int* err) {
  const int lane = threadIdx.x & 31;
  float sc = lane < 16 && t_lo < t_hi && t_lo * 16 + lane < N ? __ldg(s + t_lo * 16 + lane) : 0.f;
  for (int tile = t_lo; tile < t_hi; tile++, tj++) {
    const int b = tj & 1;
    if (!mbar_wait(&tile_full[b], (tj >> 1) & 1, err)) return false;
    float v = 0.f;
    if (lane < 16)
      for (int ww = 0; ww < CW; ww++) v += red.v[b][ww][0][lane];
    __syncwarp();
    if (lane == 0) mbar_arrive(&tile_free[b]);
    const int n = tile * 16 + lane;
    if (lane < 16 && n < N) {
      const float o = __fmul_rn(v, sc);
      y[n] = o;
      if (beats(o, (uint32_t)n, bv, bi)) {
        bv = o;
        bi = (uint32_t)n;
      }
      sc = n + 16 < N && tile + 1 < t_hi ? __ldg(s + n + 16) : 0.f;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (beats(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  return true;
}

// ======================================================================
// Decode attention
// ======================================================================
// Work item = one KV head's chunk of <= kAttnKeys keys (the reference's
// CHUNK = 128, runtime.js:330) for `hq` of the query heads that share that
// KV head (GQA), on 512 threads (warps 0-15; named barrier 1).  Each K/V row
// is fetched once per item and used by all its query heads.  hq (1, 2 or 4)
// is chosen on the device from the current context: the fewest heads per
// item such that all items fit the launched CTAs (short contexts spread the
// heads over many CTAs, long contexts share each K/V row among 4 heads);
// CTAs loop over the items when even hq = 4 leaves more items than CTAs.
// Each warp takes keys t0 + w, t0 + w + 16, ...; a lane holds 4 of the 128
// dims.  All K and V rows of the warp are requested before
// griddepcontrol.wait (pdl; the cache rows t != pos were written by earlier
// steps), so an item pays one memory latency for them.
//
// The arithmetic is ATTN_PARTIAL(_F16) (kernels.js:258-345) over the whole
// chunk: M = the chunk's max score, ev = exp(s - M), Z = sum ev,
// po = sum ev * v, all f32; then ATTN_COMBINE(_F16) (kernels.js:346-388)
// over the chunks: o = sum_s exp(pm_s - M) * po_s / sum_s pz_s exp(pm_s - M),
// with po rounded through f16 once per chunk in the f16 variant -- the
// rounding points of the reference, so the two differ only by f32
// summation order.  A single-chunk context is combined in place; longer
// contexts write (pm, pz, po) per chunk and the last item of the head set
// merges them with all 512 threads (__threadfence + arrival counter).  The
// new k (RoPE) / v row of position pos is formed in registers; the first
// item of each KV group appends it to the cache (runtime.js:1509-1514).
constexpr int kAttnWarps = 16;
constexpr int kAttnKeys = 128;  // keys per chunk (runtime.js:330 CHUNK)
constexpr int kAttnKpw = kAttnKeys / kAttnWarps;
constexpr int kAttnHq = 4;      // most query heads per item
static_assert(kAttnHq * kHeadDim == kAttnWarps * 32, "one thread per (head, dim) in the merge");

// Heads per item for a context of nsplit chunks on ncta CTAs, and the item
// count.  Every item of a launch uses the same hq (the arrival counters are
// per item's first head).
__host__ __device__ __forceinline__ int attn_hq(int nh, int nkv, int nsplit, int ncta) {
  const int G = nh / nkv;
  for (int hq = 1; hq < kAttnHq; hq *= 2)
    if (nkv * ((G + hq - 1) / hq) * nsplit <= ncta) return hq;
  return kAttnHq;
}

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

// Long-context items on the tensor cores (attn_item_mma): one item serves
// all query heads of a KV head (at most kAmHeads) over one chunk.
constexpr int kAmHeads = 8;
constexpr int kAmMinSplits = 3;         // contexts of >= 3 chunks take the tensor-core item
constexpr int kAmQPitch = kHeadDim + 8; // halfs per staged q row (conflict-free 16-byte reads)
struct AttnMmaSmem {
  // the chunk's V rows (f16); 16-byte piece c of row r at piece c ^ (r & 7),
  // so the 8 rows of an ldmatrix read fall on distinct banks
  __align__(16) uint16_t v[kAttnKeys][kHeadDim];
  __align__(16) uint32_t ph[kAmHeads][kAttnKeys / 2 + 4];    // P = exp(s - M): f16 hi pairs
  __align__(16) uint32_t pl[kAmHeads][kAttnKeys / 2 + 4];    // and the f16 lo pairs
  float wm[kAttnWarps][kAmHeads], wz[kAttnWarps][kAmHeads];  // per warp max / sum per head
};

// Shared memory of the attention (39 KB; the tensor-core item's staging
// overlays the per-warp partial rows).
struct AttnSmem {
  float wm[kAttnWarps][kAttnHq], wz[kAttnWarps][kAttnHq];
  float mz[kAmHeads][2];  // merge: global max and sum per head
  int last;
  union {
    __align__(16) float wo[kAttnWarps][kAttnHq][kHeadDim];
    AttnMmaSmem m;
  };
};

// RoPE (ROPE_QK) of the 4 dims a lane holds; the partner of dim j < 64 is
// j + 64, held by lane ^ 16.  rnd: round the result to f16 (q in the f16
// variant).
// cj / sj: cos / sin of the lane's 4 pair indices (dim & 63).
__device__ __forceinline__ float4 rope_lane4(float4 x, const float (&cj)[4], const float (&sj)[4],
                                             int f16, bool rnd) {
  const int lane = threadIdx.x & 31;
  float4 o;
  float* e = reinterpret_cast<float*>(&o);
  const float* xi = reinterpret_cast<const float*>(&x);
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const float other = __shfl_xor_sync(0xffffffffu, xi[c], 16);
    float lo = lane < 16 ? xi[c] : other, hi = lane < 16 ? other : xi[c];
    rope_pair(lo, hi, cj[c], sj[c], f16);
    if (rnd) round_h2(lo, hi);
    e[c] = lane < 16 ? lo : hi;
  }
  return o;
}

// Cache row of position t: contiguous, or through a page table of 16-row
// pages (physical row = pages[t / 16] * 16 + t % 16, WRITE_KV_PAGE).
constexpr int kKvPage = 16;
__device__ __forceinline__ size_t kv_row(const uint32_t* pages, int t) {
  return pages ? (size_t)__ldg(pages + t / kKvPage) * kKvPage + (t % kKvPage) : (size_t)t;
}

__device__ __forceinline__ void axpy4(float4& acc, float w, float4 v) {
  acc.x = __fadd_rn(acc.x, __fmul_rn(w, v.x));
  acc.y = __fadd_rn(acc.y, __fmul_rn(w, v.y));
  acc.z = __fadd_rn(acc.z, __fmul_rn(w, v.z));
  acc.w = __fadd_rn(acc.w, __fmul_rn(w, v.w));
}

// The merge of nsplit chunk partials of the head set [h0, h0 + hq) by one
// CTA (ATTN_COMBINE(_F16), kernels.js:346-388): per head the global max and
// the weighted sum of the split sums (one warp per head), then the weighted
// po sums with thread (head, dim quad, split phase) summing every P-th split
// as float4s and the phases added in shared memory.
template <int kPre = 8>
__device__ __forceinline__ void attn_merge(const AttnArgs& a, int h0, int hq, int nsplit, AttnSmem& sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = kHeadDim;
  // thread = (phase p, head j, dim quad q): P = 16 / hq phases; its first
  // kPre splits' po rows and maxima are loaded before anything waits
  const int P = kAttnHq * kAttnWarps / (4 * hq);  // 16 / hq
  const int q = threadIdx.x & 31, j = (threadIdx.x >> 5) % hq, p = (threadIdx.x >> 5) / hq;
  const float* pmj = a.pm + (h0 + j) * a.max_splits;
  const float4* pp = reinterpret_cast<const float4*>(a.po + (size_t)(h0 + j) * a.max_splits * hd) + q;
  float4 pv[kPre];
  float pmv[kPre];
#pragma unroll
  for (int k = 0; k < kPre; k++) {
    const int s2 = p + k * P;
    const bool ok = p < P && s2 < nsplit;
    pv[k] = ok ? __ldcg(pp + (size_t)s2 * (hd / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
    pmv[k] = ok ? __ldcg(pmj + s2) : 0.f;
  }
  if (warp < hq) {  // per head the global max and the weighted sum of the split sums
    const float* pm = a.pm + (h0 + warp) * a.max_splits;
    const float* pz = a.pz + (h0 + warp) * a.max_splits;
    float m2[2], z2[2];  // this lane's splits lane and lane + 32 (nsplit <= 64)
#pragma unroll
    for (int k = 0; k < 2; k++) {
      const int s2 = lane + 32 * k;
      m2[k] = s2 < nsplit ? __ldcg(pm + s2) : -1e30f;
      z2[k] = s2 < nsplit ? __ldcg(pz + s2) : 0.f;
    }
    float M = -1e30f;
    for (int s2 = lane + 64; s2 < nsplit; s2 += 32) M = fmaxf(M, __ldcg(pm + s2));
    M = fmaxf(M, fmaxf(m2[0], m2[1]));
    M = warp_max(M);
    float Z = 0.f;
#pragma unroll
    for (int k = 0; k < 2; k++)
      if (lane + 32 * k < nsplit) Z = __fadd_rn(Z, __fmul_rn(z2[k], expf(m2[k] - M)));
    for (int s2 = lane + 64; s2 < nsplit; s2 += 32)
      Z = __fadd_rn(Z, __fmul_rn(__ldcg(pz + s2), expf(__ldcg(pm + s2) - M)));
    Z = warp_sum(Z);
    if (lane == 0) {
      sm.mz[warp][0] = M;
      sm.mz[warp][1] = Z;
    }
  }
  bar_sync_n<kAttnWarps * 32>();
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  if (p < P) {
    const float M = sm.mz[j][0];
#pragma unroll
    for (int k = 0; k < kPre; k++)
      if (p + k * P < nsplit) axpy4(o, expf(pmv[k] - M), pv[k]);
    // later splits kPre at a time: all loads of a batch before its sums
    for (int base = p + kPre * P; base < nsplit; base += kPre * P) {
#pragma unroll
      for (int k = 0; k < kPre; k++) {
        const int s2 = base + k * P;
        const bool ok = s2 < nsplit;
        pv[k] = ok ? __ldcg(pp + (size_t)s2 * (hd / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
        pmv[k] = ok ? __ldcg(pmj + s2) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < kPre; k++)
        if (base + k * P < nsplit) axpy4(o, expf(pmv[k] - M), pv[k]);
    }
  }
  // phases -> shared memory (wo reused: [phase][head][dim] as 16 x 4 x 128)
  float* red = &sm.wo[0][0][0];
  if (p < P) *reinterpret_cast<float4*>(red + ((size_t)p * hq + j) * hd + 4 * q) = o;
  bar_sync_n<kAttnWarps * 32>();
  const int d = threadIdx.x % hd;
  for (int jj = threadIdx.x / hd; jj < hq; jj += kAttnWarps * 32 / hd) {
    float v = 0.f;
    for (int pp2 = 0; pp2 < P; pp2++) v = __fadd_rn(v, red[((size_t)pp2 * hq + jj) * hd + d]);
    a.out[(h0 + jj) * hd + d] = __fmul_rn(v, 1.0f / sm.mz[jj][1]);
  }
}

// One item: KV head kvh, heads [h0, h0 + nhq), chunk `split` of nsplit.
// NCH = 2 (a two-chunk context): one head (nhq = 1) over BOTH chunks in one
// pass, the chunks taking the place of the head slots (slot c = chunk c, the
// same q), then the two partials merged in registers with the arithmetic and
// order of attn_merge (bit-identical to the cross-CTA merge, without its
// global partials, fence, arrival counter and second pass).
template <typename KVT, int NCH = 1>
__device__ void attn_item(const AttnArgs& a, int kvh, int h0, int nhq, int split, int nsplit,
                          int pos, bool append, int pdl, AttnSmem& sm) {
  static_assert(NCH == 1 || NCH == 2, "one chunk, or two chunks of one head");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = kHeadDim, kvd = a.nkv * hd;
  const int f16 = a.kv_f16;
  const int ctx = pos + 1;
  const int keys = a.chunk > 0 ? a.chunk : kAttnKeys;
  const int nslot = NCH == 1 ? nhq : NCH;  // head slots in use
  int t0[NCH], t1[NCH];
#pragma unroll
  for (int c = 0; c < NCH; c++) {
    t0[c] = (split + c) * keys;
    t1[c] = min(t0[c] + keys, ctx);
  }
  const KVT* kc = reinterpret_cast<const KVT*>(a.kc) + kvh * hd + 4 * lane;
  const KVT* vc = reinterpret_cast<const KVT*>(a.vc) + kvh * hd + 4 * lane;
  KvRow<KVT> K[NCH][kAttnKpw], V[NCH][kAttnKpw];
#pragma unroll
  for (int c = 0; c < NCH; c++)
#pragma unroll
    for (int i = 0; i < kAttnKpw; i++) {
      const int t = t0[c] + warp + kAttnWarps * i;
      if (t < t1[c] && (t != pos || a.appended)) {
        const size_t r = kv_row(a.pages, t);
        K[c][i].load(kc + r * kvd);
        V[c][i].load(vc + r * kvd);
      }
    }
  // the RoPE rows of pos (constant tables) also come before the wait
  const float* cs = a.cosT + (size_t)pos * hd;
  const float* sn = a.sinT + (size_t)pos * hd;
  float cj[4], sj[4];
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const int j = (4 * lane + c) & (hd / 2 - 1);
    cj[c] = __ldg(cs + j);
    sj[c] = __ldg(sn + j);
  }
  if (pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
  // q of each head: ROPE_QK, read through f16 in the f16 variant (ATTN_PARTIAL_F16)
  float4 q4[kAttnHq];
  if (NCH == 1) {
#pragma unroll
    for (int j = 0; j < kAttnHq; j++)
      q4[j] = j < nhq ? rope_lane4(__ldcg(reinterpret_cast<const float4*>(a.qkv + (h0 + j) * hd + 4 * lane)),
                                   cj, sj, f16, f16 != 0)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
  } else {
    const float4 q = rope_lane4(__ldcg(reinterpret_cast<const float4*>(a.qkv + h0 * hd + 4 * lane)), cj, sj, f16,
                                f16 != 0);
#pragma unroll
    for (int j = 0; j < kAttnHq; j++) q4[j] = j < NCH ? q : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const int cp = NCH == 1 ? 0 : (pos - t0[0]) / keys;  // the chunk holding pos
  if (!a.appended && pos >= t0[0] && pos < t1[NCH - 1]) {  // the new row: k = RoPE(k), v, as cached
    const float* kn = a.qkv + a.nh * hd + kvh * hd;
    const float* vn = a.qkv + a.nh * hd + kvd + kvh * hd;
    const float4 kx = rope_lane4(__ldcg(reinterpret_cast<const float4*>(kn + 4 * lane)), cj, sj,
                                 f16, false);
    const float4 vr = __ldcg(reinterpret_cast<const float4*>(vn + 4 * lane));
    KvRow<KVT> kn4, vn4;
    kn4.set(make_float4(kv_round<KVT>(kx.x), kv_round<KVT>(kx.y), kv_round<KVT>(kx.z), kv_round<KVT>(kx.w)));
    vn4.set(make_float4(kv_round<KVT>(vr.x), kv_round<KVT>(vr.y), kv_round<KVT>(vr.z), kv_round<KVT>(vr.w)));
    const int i = (pos - t0[cp]) / kAttnWarps, w = (pos - t0[cp]) % kAttnWarps;
    if (warp == w) {
#pragma unroll
      for (int c = 0; c < NCH; c++)
#pragma unroll
        for (int ii = 0; ii < kAttnKpw; ii++)
          if (c == cp && ii == i) {
            K[c][ii] = kn4;
            V[c][ii] = vn4;
          }
    }
    if (append && warp == 0) {  // one item per KV group appends
      KVT* kw = reinterpret_cast<KVT*>(a.kc) + kv_row(a.pages, pos) * kvd + kvh * hd + 4 * lane;
      KVT* vw = reinterpret_cast<KVT*>(a.vc) + kv_row(a.pages, pos) * kvd + kvh * hd + 4 * lane;
      kw[0] = kv_cvt<KVT>(kx.x); kw[1] = kv_cvt<KVT>(kx.y); kw[2] = kv_cvt<KVT>(kx.z); kw[3] = kv_cvt<KVT>(kx.w);
      vw[0] = kv_cvt<KVT>(vr.x); vw[1] = kv_cvt<KVT>(vr.y); vw[2] = kv_cvt<KVT>(vr.z); vw[3] = kv_cvt<KVT>(vr.w);
    }
  }
  // ---- scores: lane L holds the 4 dims 4L..4L+3 of q (4 slots) and of the
  // warp's 8 keys; the 32 partial dots (key i, slot j) at v = 4i + j are
  // summed over the warp by a transposing butterfly (each round halves the
  // slots a lane keeps), after which lane L holds the whole dot of slot L.
  const float scale = 1.0f / sqrtf((float)hd);
  int nkc[NCH];
#pragma unroll
  for (int c = 0; c < NCH; c++)
    nkc[c] = t1[c] - t0[c] > warp ? (t1[c] - t0[c] - warp + kAttnWarps - 1) / kAttnWarps : 0;
  float pd[kAttnKpw * kAttnHq];
#pragma unroll
  for (int i = 0; i < kAttnKpw; i++) {
#pragma unroll
    for (int j = 0; j < kAttnHq; j++) {
      const float4 k4 = K[NCH == 1 ? 0 : (j < NCH ? j : 0)][i].get();
      float p = __fmul_rn(q4[j].x, k4.x);
      p = fmaf(q4[j].y, k4.y, p);
      p = fmaf(q4[j].z, k4.z, p);
      pd[4 * i + j] = fmaf(q4[j].w, k4.w, p);
    }
  }
#pragma unroll
  for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int k = 0; k < n / 2; k++) {
      const float send = up ? pd[k] : pd[k + n / 2];
      const float keep = up ? pd[k + n / 2] : pd[k];
      pd[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  const int ki = lane >> 2, hj = lane & 3;  // this lane's (key, slot)
  const int nk_hj = NCH == 1 ? nkc[0] : (hj == 1 ? nkc[NCH - 1] : nkc[0]);
  const bool valid = ki < nk_hj && hj < nslot;
  const float sv = valid ? __fmul_rn(pd[0], scale) : -1e30f;
  float m = sv;  // the warp's max per slot: lanes with the same hj
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
  if (lane < kAttnHq) sm.wm[warp][lane] = m;
  bar_sync_n<kAttnWarps * 32>();
  // ---- the chunk's max per slot, then ev = exp(s - M), Z and sum ev * v
  float M = -1e30f;
#pragma unroll
  for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, sm.wm[w][hj]);
  const float ev = valid ? expf(sv - M) : 0.f;
  float z = ev + __shfl_xor_sync(0xffffffffu, ev, 4);
  z += __shfl_xor_sync(0xffffffffu, z, 8);
  z += __shfl_xor_sync(0xffffffffu, z, 16);
  if (lane < kAttnHq) sm.wz[warp][lane] = z;
  float4 acc[kAttnHq];
#pragma unroll
  for (int jj = 0; jj < kAttnHq; jj++) acc[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kAttnKpw; i++) {
    if (NCH == 1 && i >= nkc[0]) break;
    const float4 v40 = V[0][i].get();
#pragma unroll
    for (int jj = 0; jj < kAttnHq; jj++) {
      if (jj >= nslot) break;
      const int cc = NCH == 1 ? 0 : (jj < NCH ? jj : 0);
      if (NCH == 2 && i >= nkc[cc]) continue;
      const float4 v4 = NCH == 1 ? v40 : V[cc][i].get();
      const float e = __shfl_sync(0xffffffffu, ev, 4 * i + jj);
      acc[jj].x = fmaf(e, v4.x, acc[jj].x);
      acc[jj].y = fmaf(e, v4.y, acc[jj].y);
      acc[jj].z = fmaf(e, v4.z, acc[jj].z);
      acc[jj].w = fmaf(e, v4.w, acc[jj].w);
    }
  }
#pragma unroll
  for (int jj = 0; jj < kAttnHq; jj++)
    if (jj < nslot) *reinterpret_cast<float4*>(&sm.wo[warp][jj][4 * lane]) = acc[jj];
  bar_sync_n<kAttnWarps * 32>();
  // ---- one thread per (slot j, dim d): the chunk's partial (pm, pz, po)
  const int j = threadIdx.x / kHeadDim, d = threadIdx.x % kHeadDim;
  float Mc = -1e30f, Z = 0.f, po = 0.f;
  if (j < nslot) {
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) {
      Mc = fmaxf(Mc, sm.wm[w][j]);
      Z = __fadd_rn(Z, sm.wz[w][j]);
      po = __fadd_rn(po, sm.wo[w][j][d]);
    }
    if (f16) po = round_h(po);  // ATTN_COMBINE_F16 reads po through f16
  }
  if (NCH == 2) {
    // ---- ATTN_COMBINE over the two chunks, as attn_merge computes it
    bar_sync_n<kAttnWarps * 32>();  // wo / mz are rewritten below
    if (j < NCH) {
      sm.wo[0][j][d] = po;
      if (d == 0) {
        sm.mz[j][0] = Mc;
        sm.mz[j][1] = Z;
      }
    }
    bar_sync_n<kAttnWarps * 32>();
    if (j == 0) {
      const float m0 = sm.mz[0][0], m1 = sm.mz[1][0];
      const float Mg = fmaxf(fmaxf(-1e30f, m0), m1);
      const float e0 = expf(m0 - Mg), e1 = expf(m1 - Mg);
      const float Zg = __fadd_rn(__fadd_rn(0.f, __fmul_rn(sm.mz[0][1], e0)), __fmul_rn(sm.mz[1][1], e1));
      const float v = __fadd_rn(__fadd_rn(0.f, __fmul_rn(e0, sm.wo[0][0][d])), __fmul_rn(e1, sm.wo[0][1][d]));
      a.out[h0 * hd + d] = __fmul_rn(v, 1.0f / Zg);
    }
    bar_sync_n<kAttnWarps * 32>();  // the shared area is reused by the next item
    return;
  }
  const int h = h0 + j;
  if (nsplit == 1) {
    // ATTN_COMBINE over one chunk: M' = pm, Z' = pz * exp(0), o = 1 * po / Z'
    if (j < nhq) a.out[h * hd + d] = __fmul_rn(po, 1.0f / Z);
    bar_sync_n<kAttnWarps * 32>();  // the shared area is reused by the next item
    return;
  }
  if (j < nhq) {
    a.po[((size_t)h * a.max_splits + split) * hd + d] = po;
    if (d == 0) {
      a.pm[h * a.max_splits + split] = Mc;
      a.pz[h * a.max_splits + split] = Z;
    }
  }
  // ---- several chunks: the last item of the head set merges them
  __threadfence();
  bar_sync_n<kAttnWarps * 32>();
  if (threadIdx.x == 0) sm.last = atomicAdd(a.counters + h0, 1u) == (unsigned)nsplit - 1;
  bar_sync_n<kAttnWarps * 32>();
  const bool last = sm.last != 0;
  if (last) {
    __threadfence();
    attn_merge(a, h0, nhq, nsplit, sm);
    if (threadIdx.x == 0) a.counters[h0] = 0u;  // ready for the next launch
  }
  bar_sync_n<kAttnWarps * 32>();  // the shared area is reused by the next item
}

// Long-context item on the tensor cores (f16 cache, G = nh / nkv <= 8): KV
// head kvh, all G query heads of its group, chunk `split` of nsplit.  The
// arithmetic is ATTN_PARTIAL_F16 (kernels.js:258-345) with the products
// taken by mma.sync m16n8k16 (f16 in, f32 accumulate): scores S = q K^T with
// the heads as the 16 rows (8 used) and warp w's 8 keys as the columns, so
// the K rows and each K row's slice a lane loads are read straight from the
// cache into B fragments; then M = the chunk's max per head, ev = exp(s - M),
// Z = sum ev, all f32 as in attn_item; then po = sum ev v with ev split into
// f16 hi + lo (two MMAs, |ev - hi - lo| <= 2^-22 ev) against the chunk's V
// rows staged in shared memory, warp w producing dims 8w..8w+7 of every head
// over all the chunk's keys (no cross-warp sum of partial rows).  po is read
// through f16 once per chunk as in the f16 variant, and the last item of the
// KV head merges the chunks (attn_merge over its G heads).
//
// The dot over the 128 dims is summed in a permuted order: logical k index
// 2 tq + e of k-step ks is dim 32 tq + 4 ks + e (and 2 tq + 8 + e is dim
// 32 tq + 4 ks + 2 + e), the same map for q (A) and K (B), so lane (g, tq)
// holds dims 32 tq .. 32 tq + 31 of key g and of head g contiguously.
template <typename KVT>
__device__ void attn_item_mma(const AttnArgs& a, int kvh, int split, int pos, int nsplit, int pdl,
                              AttnSmem& sm) {
  AttnMmaSmem& m = sm.m;
  constexpr int NT = kAttnWarps * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int hd = kHeadDim, kvd = a.nkv * hd, G = a.nh / a.nkv, h0 = kvh * G;
  const int ctx = pos + 1;
  const int keys = a.chunk > 0 ? a.chunk : kAttnKeys;
  const int t0 = split * keys, t1 = min(t0 + keys, ctx);
  const bool has_new = !a.appended && pos >= t0 && pos < t1;
  const __half* kc = static_cast<const __half*>(a.kc) + kvh * hd;
  const __half* vc = static_cast<const __half*>(a.vc) + kvh * hd;
  // ---- before the wait: the chunk's cached V rows -> shared memory (rows
  // past t1 zero-filled; the new row is written below), this lane's K slice,
  // and the RoPE row of pos
  for (int i = threadIdx.x; i < kAttnKeys * 16; i += NT) {
    const int r = i >> 4, c8 = i & 15, t = t0 + r;
    if (has_new && t == pos) continue;
    const bool ok = t < t1;
    cp_async16(&m.v[r][8 * (c8 ^ (r & 7))], ok ? vc + kv_row(a.pages, t) * kvd + 8 * c8 : vc, ok ? 16 : 0);
  }
  cp_async_commit();
  const int tk = t0 + 8 * warp + g;  // this lane's key
  uint32_t kw[16];
  {
    const bool ok = tk < t1 && !(has_new && tk == pos);
    const uint4* src = reinterpret_cast<const uint4*>(kc + (ok ? kv_row(a.pages, tk) * kvd : 0) + 32 * tq);
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const uint4 u = ok ? __ldcg(src + c) : make_uint4(0u, 0u, 0u, 0u);
      kw[4 * c] = u.x;
      kw[4 * c + 1] = u.y;
      kw[4 * c + 2] = u.z;
      kw[4 * c + 3] = u.w;
    }
  }
  // this thread's RoPE pair of the post-wait step: dim i and i + 64 of head
  // h0 + (tid >> 6) of q (and of the new k for tid < 64)
  const int pi = threadIdx.x & 63, pj = threadIdx.x >> 6;
  const float rc = __ldg(a.cosT + (size_t)pos * hd + pi), rs = __ldg(a.sinT + (size_t)pos * hd + pi);
  if (pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
  // ---- RoPE (ROPE_QK_F16) of q -> f16 rows qs[head] (heads >= G zero); the
  // new row of pos: k likewise -> kn and the cache, v -> the staged V rows
  // and the cache (runtime.js:1509-1514)
  uint16_t* qs = reinterpret_cast<uint16_t*>(&m.ph[0][0]);  // [8][kAmQPitch], in P's space until P
  uint16_t* kn = reinterpret_cast<uint16_t*>(&m.pl[0][0]);  // [128]
  {
    float lo = 0.f, hi = 0.f;
    if (pj < G) {
      const float* qh = a.qkv + (size_t)(h0 + pj) * hd;
      lo = __ldcg(qh + pi);
      hi = __ldcg(qh + pi + 64);
      rope_pair(lo, hi, rc, rs, 1);
    }
    qs[pj * kAmQPitch + pi] = __half_as_ushort(__float2half_rn(lo));
    qs[pj * kAmQPitch + pi + 64] = __half_as_ushort(__float2half_rn(hi));
  }
  const int r = pos - t0;  // the new row's place in the chunk (has_new)
  if (has_new) {
    if (threadIdx.x < 64) {
      const float* kh = a.qkv + a.nh * hd + kvh * hd;
      float lo = __ldcg(kh + pi), hi = __ldcg(kh + pi + 64);
      rope_pair(lo, hi, rc, rs, 1);
      const __half l16 = __float2half_rn(lo), h16 = __float2half_rn(hi);
      kn[pi] = __half_as_ushort(l16);
      kn[pi + 64] = __half_as_ushort(h16);
      __half* kw0 = static_cast<__half*>(a.kc) + kv_row(a.pages, pos) * kvd + kvh * hd;
      kw0[pi] = l16;
      kw0[pi + 64] = h16;
    }
    if (warp == kAttnWarps - 1) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(a.qkv + a.nh * hd + kvd + kvh * hd) + lane);
      const uint2 u = make_uint2(h2_bits(__floats2half2_rn(v.x, v.y)), h2_bits(__floats2half2_rn(v.z, v.w)));
      *reinterpret_cast<uint2*>(&m.v[r][8 * ((lane >> 1) ^ (r & 7)) + 4 * (lane & 1)]) = u;
      *reinterpret_cast<uint2*>(static_cast<__half*>(a.vc) + kv_row(a.pages, pos) * kvd + kvh * hd + 4 * lane) = u;
    }
  }
  bar_sync_n<NT>();  // qs, kn
  uint32_t qa[16];
  {
    const uint4* src = reinterpret_cast<const uint4*>(qs + g * kAmQPitch + 32 * tq);
#pragma unroll
    for (int c2 = 0; c2 < 4; c2++) {
      const uint4 u = src[c2];
      qa[4 * c2] = u.x;
      qa[4 * c2 + 1] = u.y;
      qa[4 * c2 + 2] = u.z;
      qa[4 * c2 + 3] = u.w;
    }
  }
  if (has_new && warp == r >> 3 && g == (r & 7)) {
    const uint4* src = reinterpret_cast<const uint4*>(kn + 32 * tq);
#pragma unroll
    for (int c2 = 0; c2 < 4; c2++) {
      const uint4 u = src[c2];
      kw[4 * c2] = u.x;
      kw[4 * c2 + 1] = u.y;
      kw[4 * c2 + 2] = u.z;
      kw[4 * c2 + 3] = u.w;
    }
  }
  // ---- scores of head g, keys 8 warp + 2 tq + {0, 1}
  float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int ks = 0; ks < 8; ks++) {
    const uint32_t af[4] = {qa[2 * ks], 0u, qa[2 * ks + 1], 0u};
    mma16816(c, af, kw[2 * ks], kw[2 * ks + 1]);
  }
  const float scale = 1.0f / sqrtf((float)hd);
  const int kb = t0 + 8 * warp + 2 * tq;
  const bool v0 = g < G && kb < t1, v1 = g < G && kb + 1 < t1;
  const float s0 = v0 ? __fmul_rn(c[0], scale) : -1e30f, s1 = v1 ? __fmul_rn(c[1], scale) : -1e30f;
  float mx = fmaxf(s0, s1);
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  if (tq == 0) m.wm[warp][g] = mx;
  bar_sync_n<NT>();
  float M = -1e30f;
#pragma unroll
  for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, m.wm[w][g]);
  const float e0 = v0 ? expf(s0 - M) : 0.f, e1 = v1 ? expf(s1 - M) : 0.f;
  float z = __fadd_rn(e0, e1);
  z = __fadd_rn(z, __shfl_xor_sync(0xffffffffu, z, 1));
  z = __fadd_rn(z, __shfl_xor_sync(0xffffffffu, z, 2));
  if (tq == 0) m.wz[warp][g] = z;
  split2(e0, e1, m.ph[g][4 * warp + tq], m.pl[g][4 * warp + tq]);
  cp_async_wait<0>();
  bar_sync_n<NT>();  // V rows, P, wz
  // ---- po[head g][dims 8 warp + 2 tq + {0, 1}] over the chunk's keys
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  // row 16 s2 + lane (s2 even keeps lane & 7 = row & 7), piece `warp`
  const uint32_t vaddr = smem_addr(&m.v[lane][8 * (warp ^ (lane & 7))]);
#pragma unroll
  for (int s2 = 0; s2 < 8; s2 += 2) {
    uint32_t b[4];
    ldsm_x4_t(vaddr + s2 * 16 * kHeadDim * 2, b[0], b[1], b[2], b[3]);
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int s = s2 + u;
      const uint32_t ah[4] = {m.ph[g][8 * s + tq], 0u, m.ph[g][8 * s + 4 + tq], 0u};
      const uint32_t al[4] = {m.pl[g][8 * s + tq], 0u, m.pl[g][8 * s + 4 + tq], 0u};
      mma16816(o, ah, b[2 * u], b[2 * u + 1]);
      mma16816(o, al, b[2 * u], b[2 * u + 1]);
    }
  }
  float Z = 0.f;
#pragma unroll
  for (int w = 0; w < kAttnWarps; w++) Z = __fadd_rn(Z, m.wz[w][g]);
  if (g < G) {
    const int h = h0 + g;
    *reinterpret_cast<float2*>(a.po + ((size_t)h * a.max_splits + split) * hd + 8 * warp + 2 * tq) =
        make_float2(round_h(o[0]), round_h(o[1]));  // ATTN_COMBINE_F16 reads po through f16
    if (warp == 0 && tq == 0) {
      a.pm[h * a.max_splits + split] = M;
      a.pz[h * a.max_splits + split] = Z;
    }
  }
  // ---- the last item of the KV head merges its chunks
  __threadfence();
  bar_sync_n<NT>();
  if (threadIdx.x == 0) sm.last = atomicAdd(a.counters + h0, 1u) == (unsigned)nsplit - 1;
  bar_sync_n<NT>();
  if (sm.last != 0) {
    __threadfence();
    attn_merge<16>(a, h0, G, nsplit, sm);  // 8 heads: 2 phases, 16 splits a thread
    if (threadIdx.x == 0) a.counters[h0] = 0u;  // ready for the next launch
  }
  bar_sync_n<NT>();  // the shared area is reused by the next item
}

// All items of one attention launch, taken by CTA `cta` of `ncta`.
// Every item of a launch as tensor-core items (any context; f16 cache,
// G <= 8), taken by CTA `cta` of `ncta`.
template <typename KVT>
__device__ void attn_run_mma(const AttnArgs& a, int cta, int ncta, int pdl, AttnSmem& sm) {
  const int pos = (a.pos ? __ldcg(a.pos) : a.fixed_pos) + a.pos_off;
  const int keys = a.chunk > 0 ? a.chunk : kAttnKeys;
  const int nsplit = (pos + keys) / keys;
  bool waited = !pdl;
  for (int it = cta; it < a.nkv * nsplit; it += ncta) {
    attn_item_mma<KVT>(a, it % a.nkv, it / a.nkv, pos, nsplit, waited ? 0 : 1, sm);
    waited = true;
  }
  if (!waited) {  // no item for this CTA: still order the launch chain
    pdl_wait();
    pdl_launch_dependents();
  }
}

// MMA: long contexts of an f16 cache take attn_item_mma (the batched
// attention; the single-stream decode launches attn_run_mma's own kernel for
// them instead, chosen on the host, so that its short-context kernel keeps
// none of the tensor-core item's code).
template <typename KVT, bool MMA = true>
__device__ void attn_run(const AttnArgs& a, int cta, int ncta, int pdl, AttnSmem& sm) {
  // The position and the cached rows t != pos were written before the
  // producing GEMV started (it triggers this launch only after its own
  // griddepcontrol.wait).
  const int pos = (a.pos ? __ldcg(a.pos) : a.fixed_pos) + a.pos_off;
  const int keys = a.chunk > 0 ? a.chunk : kAttnKeys;
  const int nsplit = (pos + keys) / keys;
  const int G = a.nh / a.nkv;
  bool waited = !pdl;
  // f16 cache, >= 3 chunks: one tensor-core item per (KV head, chunk)
  if (MMA && sizeof(KVT) == 2 && nsplit >= kAmMinSplits && G <= kAmHeads) {
    attn_run_mma<KVT>(a, cta, ncta, pdl, sm);
    return;
  }
  // f16 cache: one item per query head over both chunks, merged in place
  // (the f32 cache's rows are twice as wide and would spill)
  if (sizeof(KVT) == 2 && nsplit == 2) {
    for (int h = cta; h < a.nh; h += ncta) {
      attn_item<KVT, 2>(a, h / G, h, 1, 0, 2, pos, h % G == 0, waited ? 0 : 1, sm);
      waited = true;
    }
    if (!waited) {
      pdl_wait();
      pdl_launch_dependents();
    }
    return;
  }
  const int hq = attn_hq(a.nh, a.nkv, nsplit, ncta);
  const int subs = (G + hq - 1) / hq;
  const int items = a.nkv * subs * nsplit;
  for (int it = cta; it < items; it += ncta) {
    const int split = it / (a.nkv * subs), r = it % (a.nkv * subs);
    const int kvh = r / subs, sub = r % subs;
    attn_item<KVT>(a, kvh, kvh * G + sub * hq, min(hq, G - sub * hq), split, nsplit, pos, sub == 0,
                   waited ? 0 : 1, sm);
    waited = true;
  }
  if (!waited) {  // no item for this CTA: still order the launch chain
    pdl_wait();
    pdl_launch_dependents();
  }
}

}  // namespace eg
