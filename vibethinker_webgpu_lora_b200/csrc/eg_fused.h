// eg_fused.h -- launch API of the persistent fused decode kernel.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace eg {

// Device pointers of one layer (the runtime keeps an array of these in HBM).
struct FusedLayer {
  const uint32_t *qkv_w, *o_w, *gu_w, *d_w;
  const float *qkv_s, *o_s, *gu_s, *d_s, *qkv_b, *in_norm, *post_norm;
  void *kc, *vc;
};

struct FusedArgs {
  const FusedLayer* layers;  // device array [layers_n]
  int layers_n, H, QD, KVD, I, V, nh, nkv;
  float eps;
  int f16;
  const uint32_t* emb_w;
  const float* emb_s;
  const float* final_norm;
  const float *cosT, *sinT;
  float *hidden, *qkv, *attn, *tmp, *logits;
  float *pm, *pz, *po;
  unsigned* attn_counters;
  int max_splits, attn_chunk;
  uint32_t* ids;      // token id per position; ids[start_pos] is the first input
  uint32_t* amax;
  uint32_t* out_ids;  // greedy: out_ids[t] = token produced by step t
  int* state_pos;     // receives start_pos + n_tokens
  float* cand_v;
  uint32_t* cand_i;
  unsigned* lm_counter;  // zero between launches
  unsigned* bar;         // zeroed before each launch
  int* err;              // zeroed before each launch; 1 = a barrier wait timed out
  int start_pos, n_tokens;
  int greedy;    // 1: argmax after every LM head, chained into ids[pos+1]
  int lm_every;  // 0: run the LM head only for the last token (prefill)
  // Optional phase profile of token 0: prof[2*ph] = phase start on CTA 0,
  // prof[2*ph+1] = latest work end over all CTAs (globaltimer ns).
  unsigned long long* prof;
  int l2_ahead;  // units the producer's L2 prefetch runs ahead of the ring
  int diag;      // measurement only: 1 = no weight copies, 2 = no GEMV math
};

// One cooperative launch over all SMs; returns the launch error.
cudaError_t fused_decode(const FusedArgs& a, cudaStream_t st);
int fused_smem_bytes();
// Profiling: point the intra-phase timeline at buf (80 slots) or null.
cudaError_t fused_set_marks(unsigned long long* buf);

}  // namespace eg
