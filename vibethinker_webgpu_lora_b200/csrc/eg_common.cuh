// eg_common.cuh -- device helpers shared by the Emberglass B200 kernels:
// the integer tensor-core dot-product steps of the streaming GEMVs, the
// nibble-to-byte step of the int4 weights, f16 rounding helpers and small
// reductions.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define EG_DEV __device__ __forceinline__

namespace eg {

constexpr int kGroup = 128;   // int4 group size (quantize.js:81, kernels.js:901 `bk >> 7`)
constexpr int kHeadDim = 128;  // attention kernels are specialised for head_dim 128

// Nibbles 0,2,4,6 of a packed int4 word (8 two's-complement nibbles, nibble
// j = k 8c+j, quantize.js:107) as four bytes q + 8 in [0, 15] (offset
// binary): one LOP3.
EG_DEV uint32_t nib_lo_u8(uint32_t w) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(w), "r"(0x0F0F0F0Fu), "r"(0x08080808u));
  return d;
}
// Nibbles 1,3,5,7 in place: four bytes 16 (q + 8) in [0, 240], one LOP3 (the
// factor 16 is taken out of the matching activation elements).
EG_DEV uint32_t nib_hi16_u8(uint32_t w) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(w), "r"(0xF0F0F0F0u), "r"(0x80808080u));
  return d;
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

// Round two f32 values to f16 and back (each rounded once, RNE).
EG_DEV void round_h2(float& a, float& b) {
  const float2 r = __half22float2(__floats2half2_rn(a, b));
  a = r.x;
  b = r.y;
}

EG_DEV float round_h(float v) { return __half2float(__float2half_rn(v)); }

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

// The small standalone ops (RMSNorm, LoRA-A) run on a 256-thread CTA and
// synchronise with named barrier 1 over those 256 threads; the streaming
// kernels pass their consumer thread count to the *_n helpers of
// eg_device.cuh instead (their producer and epilogue warps never join).
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
