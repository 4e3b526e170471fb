// eg_prefill.h -- launch API of the whole-prompt prefill kernels (the
// reference's prefillBatch, runtime.js:1936-2087): the token embedding of a
// pass, RoPE of its q/k rows with the K/V rows into the cache, and the
// causal prefill attention.  The projections of a pass run through the
// tcgen05 GEMM (gemv_q4_tc in whole-prompt mode, eg_batch.h).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace eg {

// EMBED_T (kernels.js:619-634): hidden[t][k] = f32(q8[ids[t]][k]) * scale[ids[t]].
void prefill_embed(const uint32_t* ids, const uint32_t* emb_w, const float* emb_s, int T, int H, float* hidden,
                   cudaStream_t st);

// ROPE_T / ROPE_T_F16 (kernels.js:588-618) of rows t = 0..T-1 (position
// pos0 + t) of qkv [T][qkv_stride] = q [nh*128] | k [nkv*128] | v: q is
// rotated in place, k rotated and v copied into cache rows pos0 + t of the
// dense caches kc / vc ([rows][nkv*128], f16 or f32 as kv_f16 says).
void prefill_rope_append(float* qkv, int T, int qkv_stride, int nh, int nkv, int pos0, const float* cosT,
                         const float* sinT, int kv_f16, void* kc, void* vc, cudaStream_t st);

// ATTN_PREFILL_BLOCK (kernels.js:684-770): query rows t = 0..T-1 (absolute
// position q_start + t, q roped in qkv) over cache rows 0..ctx-1, causal,
// an online softmax over 128-key blocks aligned at key 0; out [T][out_stride].
struct PrefillAttn {
  const float* qkv;
  int qkv_stride;
  const void* kc;
  const void* vc;
  int nh, nkv, kv_f16;
  int T, q_start, ctx;
  float* out;
  int out_stride;
};
void attn_prefill(const PrefillAttn& a, cudaStream_t st);

}  // namespace eg
