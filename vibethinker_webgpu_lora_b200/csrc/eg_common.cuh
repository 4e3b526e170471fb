// eg_common.cuh -- device helpers shared by the Emberglass B200 kernels.
//
// Dequantisation of the reference's packed weights straight into f16 MMA
// fragments, the m16n8k16 tensor-core dot-product step, and small
// reductions.  Weight layouts are the reference's own (row-major packed
// words, src/qwgpu/quantize.js:28-111), so no re-tiling happens at upload.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define EG_DEV __device__ __forceinline__

namespace eg {

constexpr int kGroup = 128;   // int4 group size (quantize.js:81, kernels.js:901 `bk >> 7`)
constexpr int kHeadDim = 128;  // attention kernels are specialised for head_dim 128

// ---------------------------------------------------------------- bit tricks
// d = mask ? (a ^ c) : c, one LOP3.  Used to drop nibbles/bytes into the
// mantissa of an f16 whose exponent encodes 1024, flipping the sign bit of
// each two's-complement field into offset binary on the way.
EG_DEV uint32_t lop3_sel(uint32_t a, uint32_t mask, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(mask), "r"(c));
  return d;
}
EG_DEV uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// One packed int4 word (8 two's-complement nibbles, nibble j = k 8c+j,
// quantize.js:107) -> four f16x2 registers holding exact integers:
//   p0 = (q0, q4)  p1 = (16 q1, 16 q5)  p2 = (q2, q6)  p3 = (16 q3, 16 q7).
// The x16 factors are cancelled by pre-dividing the matching x entries by 16
// (exact powers of two).
EG_DEV void deq_int4(uint32_t w, uint32_t& p0, uint32_t& p1, uint32_t& p2, uint32_t& p3) {
  const uint32_t w8 = w >> 8;
  p0 = hsub2(lop3_sel(w, 0x000F000Fu, 0x64086408u), 0x64086408u);
  p1 = hsub2(lop3_sel(w, 0x00F000F0u, 0x64806480u), 0x64806480u);
  p2 = hsub2(lop3_sel(w8, 0x000F000Fu, 0x64086408u), 0x64086408u);
  p3 = hsub2(lop3_sel(w8, 0x00F000F0u, 0x64806480u), 0x64806480u);
}

// One packed int8 word (4 int8, little-endian, quantize.js:51-54) ->
//   p0 = (q0, q2)  p1 = (q1, q3), exact in f16.
EG_DEV void deq_int8(uint32_t w, uint32_t& p0, uint32_t& p1) {
  p0 = hsub2(lop3_sel(w, 0x00FF00FFu, 0x64806480u), 0x64806480u);
  p1 = hsub2(lop3_sel(w >> 8, 0x00FF00FFu, 0x64806480u), 0x64806480u);
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, f32 accumulate.
EG_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                     uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A(16x32 u8, row) * B(32x8 s8, col) + C, s32 accumulate (exact).
EG_DEV void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                      uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A(16x32 s8, row) * B(32x8 s8, col) + C, s32 accumulate (exact).
EG_DEV void imma16832_ss(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Nibbles 0,2,4,6 (lo) or 1,3,5,7 (hi) of a packed int4 word as four bytes
// q + 8 in [0, 15] (offset binary), one LOP3 (+ one shift).
EG_DEV uint32_t nib_lo_u8(uint32_t w) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(w), "r"(0x0F0F0F0Fu), "r"(0x08080808u));
  return d;
}
EG_DEV uint32_t nib_hi_u8(uint32_t w) { return nib_lo_u8(w >> 4); }

EG_DEV uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
// Split f32 values into (hi, lo) f16 pairs with v ~= hi + lo (22 significant
// bits), so a tensor-core dot of exact integer weights with hi and lo columns
// reproduces an f32 dot to within f32 rounding.
// (Paired f32->f16 conversions: the single-value conversion runs on the
// narrow XU pipe, the paired one at ~4x its rate.)
EG_DEV void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}
// Round two f32 values to f16 and back (each rounded once, RNE).
EG_DEV void round_h2(float& a, float& b) {
  const float2 r = __half22float2(__floats2half2_rn(a, b));
  a = r.x;
  b = r.y;
}

EG_DEV float round_h(float v) { return __half2float(__float2half_rn(v)); }

EG_DEV uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---------------------------------------------------------------- reductions
EG_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
EG_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// The building blocks in eg_device.cuh run on a 256-thread group: the whole
// CTA of a per-op kernel, or the 8 consumer warps of the fused kernel (whose
// producer warp never joins).  Named barrier 1 over those 256 threads.
constexpr int kCtaThreads = 256;
EG_DEV void cta_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Programmatic dependent launch: wait for the producing kernel's writes /
// allow the next kernel in the stream to start its independent prologue.
EG_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
EG_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// "x beats (v, idx)" in the reference's selection order: larger value, ties
// to the lower index; NaN never wins and values below -1e30 are never taken
// (kernels.js:775-776 initialise v = -1e30, idx = 0xffffffff).
EG_DEV bool beats(float x, uint32_t i, float v, uint32_t idx) {
  return x > v || (x == v && i < idx);
}

}  // namespace eg
