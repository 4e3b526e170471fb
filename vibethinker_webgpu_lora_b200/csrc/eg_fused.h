// eg_fused.h -- launch API of the persistent decode kernel.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace eg {

// Device pointers of one layer (the runtime keeps an array of these in HBM).
struct FusedLayer {
  const unsigned char *qkv, *o, *gu, *d;  // int4 matrices, stream layout
  const float *qkv_b, *in_norm, *post_norm;
  void *kc, *vc;
};

struct FusedArgs {
  const FusedLayer* layers;  // device array [layers_n]
  int layers_n, H, QD, KVD, I, V, nh, nkv;
  float eps;
  int f16;
  const uint32_t* emb_w;     // int8 rows (EMBED_BUF)
  const float* emb_s;
  const unsigned char* lm;   // the same matrix in the int8 stream layout (LM head)
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
  float* cand_v;      // [gridDim.x] LM-head argmax candidates
  uint32_t* cand_i;
  unsigned* bar;      // zeroed before each launch
  int* err;           // zeroed before each launch; 1 = a bounded wait gave up
  int start_pos, n_tokens;
  int greedy;    // 1: argmax after every LM head, chained into ids[pos+1]
  int lm_every;  // 0: run the LM head only for the last token (prefill)
  // Optional phase profile of token 0: prof[2*ph] = phase start on CTA 0,
  // prof[2*ph+1] = latest end of the phase's work over all CTAs (ns).
  unsigned long long* prof;
};

// One cooperative launch over all SMs; returns the launch error.
cudaError_t fused_decode(const FusedArgs& a, cudaStream_t st);
int fused_smem_bytes(const FusedArgs& a);

}  // namespace eg
