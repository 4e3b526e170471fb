// eg_kernels.h -- internal launch API of the Emberglass B200 kernels.
// Everything here takes device pointers and a stream; the C ABI in
// eg_runtime.cu is built on top of it.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace eg {

// One LoRA module in device memory (src/lora_gpu.js:96-109 layout):
// A [rank][in] f32, B [rank][out] f32, y += scale * (A x) . B.
struct LoraMod {
  const float* A;
  const float* B;
  int rank;
  float scale;
};

enum XMode { X_PLAIN = 0, X_RMS = 1, X_EMBED_RMS = 2 };

// Where a GEMV's input vector comes from (its prologue).
struct XSrc {
  int mode;
  const float* x;       // X_PLAIN: the vector; X_RMS: hidden state to normalise
  const float* norm_g;  // RMSNorm weight
  float eps;
  int f16;              // RMSNORM_F16 arithmetic (kernels.js:145-166)
  // X_EMBED_RMS: hidden = embed(ids[*pos]) (EMBED_BUF, kernels.js:537-550),
  // written to hidden_out by block 0, then normalised.
  const uint32_t* emb_w;
  const float* emb_s;
  const int* pos;       // device position, or null to use fixed_pos
  const uint32_t* ids;
  float* hidden_out;
  int fixed_pos;
  int use_fixed_id;   // X_EMBED_RMS: 1 = embed fixed_id instead of ids[pos]
  uint32_t fixed_id;
};

enum EpiMode { EPI_STORE = 0, EPI_ADD = 1, EPI_SILU = 2 };

struct Epi {
  int mode;
  float* y;
  const float* bias;  // EPI_STORE only, may be null
  int N;              // output rows (EPI_SILU: rows of one half)
  // LoRA: up to 3 modules split by output row (q/k/v), or gate/up for SILU.
  const LoraMod* mods;  // null => no LoRA
  const float* lora_d;  // [3][kMaxRank] d = A x
  int split1, split2;   // row boundaries between module 0/1 and 1/2
};

constexpr int kMaxRank = 256;
constexpr int kCandMax = 148;  // candidate blocks of the argmax/top-k stage 1

// Final step of a greedy/advance decode step, run by the LM head's last block.
struct StepTail {
  int* pos;            // device position counter, incremented by one
  uint32_t* ids;       // token id per position: ids[pos+1] = argmax (greedy)
  uint32_t* amax;      // s.amax equivalent
  uint32_t* out_ids;   // out_ids[*out_idx] = argmax (greedy)
  int* out_idx;
  int greedy;          // 0: only advance pos
  float* cand_v;       // [grid] per-block best value
  uint32_t* cand_i;    // [grid] per-block best index
  unsigned* counter;   // last-block-done counter (self-resetting)
  // Shard mode (advance = 0): only the best (value, id + id0) is written to
  // (*best_v, *amax); the decode state is untouched.
  int advance;
  uint32_t id0;
  float* best_v;
};

int sm_count();

// Error word of the streaming int4 GEMV, set when a bounded wait gives up.
struct GemvWork {
  int* err;
  // Optional L2 prefetch of a later kernel's weights (the next matrix of the
  // step): each CTA's producer prefetches its 1/grid slice of
  // [pf, pf + pf_bytes) once its own first ring stages are issued, so the
  // HBM stream runs ahead of the dependency chain.  16-byte aligned.
  const unsigned char* pf = nullptr;
  size_t pf_bytes = 0;
};
int gemv_q4_ctas();

// int4 matrices are kept on the device in the "stream" layout: blocks of
// 16 rows x 128 k (R = 2: the gate tile and its up tile) in MMA fragment
// order, each followed by its 16R group scales, tile-major.  q4_to_stream
// builds it from the reference layout (packed u32 [R*N][K/8], scale f32
// [R*N][K/128], quantize.js:81-111).
size_t q4_stream_bytes(int N, int K, int R);
void q4_to_stream(const uint32_t* w, const float* s, int N, int K, int R, unsigned char* out,
                  cudaStream_t st);

// y = W4 x over a stream-layout matrix (R = 2 for EPI_SILU: rows n and N+n
// of a packed [gate;up] matrix).  Requires K % 128 == 0, K <= 12288.
void gemv_q4(const unsigned char* ws, int N, int K, const XSrc& x, const Epi& e, cudaStream_t st,
             bool pdl, const GemvWork& wk);
// int8 row matrices in the "stream" layout: 16 x 128 blocks of m16n8k32 A
// fragments, tile-major; q8_to_stream builds it from int8 rows (4 per u32,
// quantize.js:28-57), zero-padding K to a multiple of 128.
size_t q8_stream_bytes(int N, int K);
void q8_to_stream(const uint32_t* w, int N, int K, unsigned char* out, cudaStream_t st);
// y = (W8 x) * scale[n] over a stream-layout matrix.  tail != null fuses
// argmax/advance.  Requires K % 4 == 0, K <= 12288.
void gemv_q8(const unsigned char* ws, const float* s, int N, int K, const XSrc& x, float* y,
             const StepTail* tail, cudaStream_t st, bool pdl, const GemvWork& wk);
struct AttnArgs {
  const float* qkv;  // raw q [nh*128] | k [nkv*128] | v [nkv*128] from the QKV GEMV
  void* kc;          // [max_ctx][nkv][128] f16 or f32
  void* vc;
  const float* cosT;
  const float* sinT;
  const int* pos;    // device: current position (ctx = pos + 1)
  int fixed_pos;     // used when pos == null
  int nh, nkv, max_splits;
  int ctx_bound;     // upper bound of pos + 1 for this launch (sizes the grid)
  int kv_f16;        // 1: f16 cache + ATTN_*_F16 / ROPE_QK_F16 numerics
  int chunk;         // keys per split: 0 = 128 (the reference's CHUNK); else 16..128, % 16 == 0
  float *pm, *pz, *po;  // partials [nh][max_splits], po [nh][max_splits][128]
  float* out;        // attention output [nh*128]
  unsigned* counters;  // [nh] split-arrival counters (one per item's first head), zero between launches
  // Paged cache (WRITE_KV_PAGE / ATTN_PARTIAL_PAGED, kernels.js:1657-1911):
  // row t lives at physical row pages[t / 16] * 16 + t % 16 of kc / vc;
  // null = contiguous rows.
  const uint32_t* pages;
  // Chunked prefill: the query position is *pos + pos_off, and with
  // `appended` the cache already holds every row up to it (written by
  // kv_append_batch), so all rows are read from the cache and none is
  // appended here.
  int pos_off, appended;
};
// Keys per split when AttnArgs::chunk is 0 (the reference's CHUNK).
constexpr int kAttnDefaultChunk = 128;
int attn_max_splits(int max_ctx);
int attn_ctas(const AttnArgs& a, int lanes);
// long_ctx: the launch runs at a position where attn_long holds (the
// tensor-core items of attn_run_mma); either kernel is correct at any
// position, the choice is only speed.
bool attn_long(const AttnArgs& a, int pos);
void attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl, bool long_ctx);

// y[r] += A[r] . x for up to 3 modules (LORA_A, kernels.js:60-78); x from src.
void lora_a(const XSrc& x, int K, const LoraMod* mods, int nmods, int max_rank, float* d,
            cudaStream_t st, bool pdl);

void rmsnorm(const float* x, const float* g, int K, float eps, int f16, float* y, cudaStream_t st);
void rope_qk(float* q, float* k, int nq, int nkv, int pos, const float* cosT, const float* sinT,
             int f16, cudaStream_t st);
void embed_rows(const uint32_t* w, const float* s, const uint32_t* id_dev, int H, float* out,
                cudaStream_t st);

// Sampling (kernels.js:771-883).
void argmax(const float* logits, int n, uint32_t* out, float* cand_v, uint32_t* cand_i,
            cudaStream_t st);
int topk_cand_blocks(int n);
void topk(const float* logits, int n, int k, uint32_t* ids, float* vals, float* cand_v,
          uint32_t* cand_i, cudaStream_t st);
void sample_topk(const uint32_t* ids, const float* vals, int k, float temp, float r,
                 uint32_t* out, uint32_t* out2, cudaStream_t st);

void copy_u32(const uint32_t* src, uint32_t* dst, cudaStream_t st);

}  // namespace eg
