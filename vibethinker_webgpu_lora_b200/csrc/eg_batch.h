// eg_batch.h -- launch API of the multi-sequence batched decode kernels.
//
// Up to kBatchMax "lanes" (one per sequence) step together: every weight
// tile is streamed from HBM once per step and multiplied against all lanes'
// activations.  The reference decodes one sequence at a time (runtime.js:
// 1466-1571); a batch step computes, for every lane, exactly that step's
// math on the lane's own KV cache and position.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "eg_kernels.h"

namespace eg {

constexpr int kBatchMax = 16;
// Most tokens of one whole-prompt (tcgen05) GEMM call or prefill block.
constexpr int kPrefillMaxT = 8192;

// Per-sequence state on the device.  Slot s holds its token ids
// ids[s * slot_ctx + t], its position pos[s] (the token consumed by the next
// step) and len[s] (ids known so far: the prompt, then generated tokens).
struct SeqTable {
  const int* lane_slot;  // [kBatchMax] slot of each lane
  int* pos;              // [slots]
  int* len;              // [slots]
  uint32_t* ids;         // [slots][slot_ctx]
  int slot_ctx;
  uint32_t vocab;        // ids >= vocab (argmax of all-NaN logits) are stored as 0
  // Chunked prefill: every lane is the same slot and lane v is position
  // pos[slot] + v (its token ids[pos + v]); a step moves pos on by the lane
  // count.
  int chunk;
};

// Where each lane's GEMV input comes from: XSrc of lane 0 with x (and
// hidden_out) advanced by `stride` floats per lane; X_EMBED_RMS takes the
// lane's token id at its position from the sequence table.
struct BatchSrc {
  XSrc x;
  int stride;
  SeqTable seq;
};

// Staged activations of all lanes (global memory): the int4 GEMV's digit
// planes (stage_xd: xb 512 B per 128-group, xcor 2 words per group, xf one
// exponent) or the int8 GEMV's (stage_xd8: xb 512 B per group, xmul 2 per
// group); lane v's planes start at v * gpr_max groups.
struct BatchPlanes {
  void* xb;
  int* xcor;     // int4 only
  float* xmul;   // int8 only
  int* xf;       // int4 only
  int gpr_max;
  // int4 only, optional: the same digit planes as the B operand of the
  // tcgen05 GEMV (gemv_q4_tc): per group, N = 4 tc_tpad columns (lane v,
  // plane p at column 4v + p) x 128 bytes, K-major 8 x 16-byte core
  // matrices, the 8 k-chunks N / 8 core matrices apart.
  void* xtc;
  int tc_tpad;
  // int4 only, optional, instead of the digit planes: the f16 hi/lo operand
  // of the whole-prompt GEMM (stage_xd's xh), tiles of 128 lanes, each
  // gpr_max groups x 64 KB
  void* xh;
};

// Epilogue of a batched int4 GEMV: the single-lane epilogue (bias /
// residual / SiLU) with y advanced by ystride per lane.  LoRA enters as
// lora_pre[lane * lstride + row] (gate rows then up rows for SiLU), each
// value the single-lane epilogue's lora_dot, computed ahead by lora_b_batch;
// e.mods is not used by the batched GEMV.
struct BatchEpi {
  Epi e;
  int ystride, dstride;
  const float* lora_pre;
  int lstride;
  // tcgen05 path only, the whole-prompt prefill's arithmetic
  // (prefillBatch, runtime.js:1936-2087): add_first: EPI_ADD is
  // (y + W x) + LoRA as GEMM4_ADD_T then LORA_B_ADD_T; silu_f16: SiLU(g) and
  // u meet in f16 (SILUMUL_F16, kernels.js:499-512).
  int add_first, silu_f16;
};

// Batched int4 GEMV on the tcgen05 tensor cores (eg_tc.cu): the epilogue
// of gemv_q4_batch for up to 32 lanes (xp.xtc staged by batch_stage_q4),
// R = 2 for GATE_UP_SILU.  The weights come as int8 A images expanded once
// at load (q4_tc_to_a8: per (octet, group) the 128 x 128 operand bytes in the
// MMA's shared-memory layout, plus each MMA row's group scale); the CTAs split
// the (octet, group) items (split-K); part / counters are the split-octet
// scratch (gemv_q4_tc_part_bytes, counters zero between launches).
void gemv_q4_tc(const unsigned char* a8, const float* sc, int N, int K, int R, int lanes, const BatchPlanes& xp,
                const BatchEpi& be, float* part, unsigned* counters, int* err, cudaStream_t st, bool pdl);
size_t gemv_q4_tc_part_bytes();
int gemv_q4_tc_max_octets();
// The octet-major regrouping of the stream layout (q4_stream_to_tc), the
// source of the A images.
size_t q4_tc_bytes(int N, int K, int R);
void q4_stream_to_tc(const unsigned char* ws, int N, int K, int R, unsigned char* out, cudaStream_t st);
size_t q4_a8_bytes(int N, int K, int R);
size_t q4_row_scale_bytes(int N, int K, int R);
void q4_tc_to_a8(const unsigned char* wc, int N, int K, int R, unsigned char* a8, float* sc, cudaStream_t st);

// Whole-prompt GEMM on the tcgen05 tensor cores (eg_tc.cu), for more than 32
// token rows, kind::f16: A images expanded once from the tc layout
// (q4_tc_to_a16: per (octet, group) the 128 x 128 nibble values as f16), the
// row scales of q4_tc_to_a8, B = the rows' f16 hi/lo operand (xp.xh, staged
// by batch_stage_q4), gemv_q4_tc's epilogue.
size_t q4_a16_bytes(int N, int K, int R);
void q4_tc_to_a16(const unsigned char* wc, int N, int K, int R, unsigned char* a16, cudaStream_t st);
void gemm_q4_prefill(const unsigned char* a16, const float* sc, int N, int K, int R, int lanes,
                     const BatchPlanes& xp, const BatchEpi& be, int* err, cudaStream_t st);

// pdl: launched as programmatic dependents of the previous kernel (each
// kernel waits with griddepcontrol.wait before reading earlier outputs).
// mods / nmods / max_rank / d / dstride (optional): the LoRA A rows of the
// nmods modules at mods over each lane's staged vector, d + v * dstride as
// lora_a_batch writes them, folded into the staging when nmods * max_rank
// <= kStageLoraRows (returns true); otherwise nothing is computed (false)
// and the caller runs lora_a_batch.
bool batch_stage_q4(const BatchSrc& s, int K, int lanes, const BatchPlanes& xp, cudaStream_t st, bool pdl,
                    const LoraMod* mods = nullptr, int nmods = 0, int max_rank = 0, float* d = nullptr,
                    int dstride = 0);
void batch_stage_q8(const BatchSrc& s, int K, int lanes, const BatchPlanes& xp, cudaStream_t st,
                    bool pdl);
void gemv_q4_batch(const unsigned char* ws, int N, int K, int lanes, const BatchPlanes& xp,
                   const BatchEpi& be, int* err, cudaStream_t st, bool pdl);
void gemv_q8_batch(const unsigned char* ws, const float* s, int N, int K, int lanes,
                   const BatchPlanes& xp, float* y, int ystride, int* err, cudaStream_t st,
                   bool pdl);

// Attention of every lane: AttnArgs of lane 0 (kc/vc = the layer's slot-0
// cache) with qkv/out/partials advanced per lane, the cache by the lane's
// slot, the position from the sequence table.
struct AttnBatch {
  SeqTable seq;
  int qkv_stride, out_stride, part_stride;  // floats per lane (part: pm/pz; po = 128x)
  size_t kv_slot_bytes;                     // one slot's cache of one layer (dense)
  // Paged slots: kc / vc are the layer's page pool and slot s's page table
  // is page_table[s * max_pages ..]; null = dense slots.
  const uint32_t* page_table;
  int max_pages;
};
void attn_batch(const AttnArgs& a, const AttnBatch& b, int lanes, cudaStream_t st, bool pdl);

// Chunked prefill, before the attention: lane v's k row (RoPE at its
// position) and v row of qkv + v * qkv_stride go into the cache rows of
// positions pos + v, rounded as the cache stores them (the attention
// item's append, runtime.js:1509-1514).
void kv_append_batch(const AttnArgs& a, const AttnBatch& b, int lanes, cudaStream_t st);

// LoRA B side of every lane: out[v * be.lstride + row] = the single-lane
// epilogue's lora_dot for that row (e.mods, e.lora_d + v * dstride); rows =
// N, or 2N for SiLU (gate rows, then up rows).
void lora_b_batch(const BatchEpi& be, int rows, int lanes, float* out, cudaStream_t st, bool pdl);

// LORA_A of every lane: d + v * dstride.
void lora_a_batch(const BatchSrc& s, int K, const LoraMod* mods, int nmods, int max_rank, float* d,
                  int dstride, int lanes, cudaStream_t st, bool pdl);

// Per-lane argmax / top-k / sample over logits [lanes][n].
void argmax_batch(const float* logits, int n, int lanes, uint32_t* out, float* cand_v,
                  uint32_t* cand_i, cudaStream_t st);
void topk_batch(const float* logits, int n, int k, int lanes, uint32_t* ids, float* vals,
                float* cand_v, uint32_t* cand_i, cudaStream_t st);
int topk_batch_cand(int n, int k);  // candidate slots per lane
// r[step * kBatchMax + lane], step = *step_ctr (advanced by batch_advance).
void sample_batch(const uint32_t* ids, const float* vals, int k, float temp, const float* r,
                  const int* step_ctr, int lanes, uint32_t* out, cudaStream_t st);

// End of a batch step: lane v's choice[v] becomes the slot's next token
// when the slot is past its known ids; out[*step_ctr * lanes + v] = the
// token at the new position; positions advance; *step_ctr += 1.
void batch_advance(SeqTable seq, const uint32_t* choice, int lanes, uint32_t* out, int* step_ctr,
                   cudaStream_t st);

}  // namespace eg
