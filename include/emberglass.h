/*
 * emberglass.h -- C ABI of libemberglass_cuda.so, the B200 (sm_100a)
 * replacement for the Emberglass WebGPU decode path
 * (maceip/vibethinker-webgpu-lora, src/qwgpu/runtime.js `QwenWGPU`).
 *
 * Conventions
 *  - Every function returns an eg_status (0 = EG_OK).  On failure
 *    eg_last_error() returns a thread-local message; the reference throws a
 *    JS Error with the same text at the cited line.
 *  - Plain pointers and sizes only.  Runtime entry points (eg_token, ...)
 *    take HOST buffers and do their own host<->device copies; single-op
 *    entry points (eg_op_*) take DEVICE pointers and a cudaStream_t passed as
 *    void* (NULL = legacy default stream) and are asynchronous.
 *  - All calls on one eg_rt are serialised on that runtime's stream; the
 *    library starts no threads of its own for device work.  Concurrent
 *    readback calls on one handle fail with EG_ERR_BUSY, as the reference's
 *    busy flags do (runtime.js:1603-1605, :1649-1650, :1686-1687).
 *  - Weight layouts are the reference's: int4 = 8 two's-complement nibbles
 *    per u32, low nibble = lowest k, f32 scale per (row, 128-group)
 *    (quantize.js:81-111); int8 = 4 per u32 little-endian with one f32 scale
 *    per row (quantize.js:28-57).
 */
#ifndef EMBERGLASS_H
#define EMBERGLASS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EG_API __attribute__((visibility("default")))

typedef enum {
  EG_OK = 0,
  EG_ERR_ARG = 1,      /* bad argument / shape (reference: throw new Error) */
  EG_ERR_CUDA = 2,     /* a CUDA call failed */
  EG_ERR_STATE = 3,    /* call not valid in the current state */
  EG_ERR_OOM = 4,      /* device or host allocation failed */
  EG_ERR_BUSY = 5,     /* concurrent readback on one handle */
  EG_ERR_DEVICE = 6    /* a kernel reported a failed bounded wait */
} eg_status;

typedef struct eg_rt eg_rt;
typedef struct eg_lora eg_lora;

/* QWEN25_3B in src/config.js:27-48. */
typedef struct {
  int hidden_size;        /* 2048 */
  int num_layers;         /* 36 */
  int num_heads;          /* 16 */
  int num_kv_heads;       /* 2 */
  int head_dim;           /* 128 (the only value the kernels support) */
  int intermediate_size;  /* 11008 */
  int vocab_size;         /* 151936 */
  float rms_norm_eps;     /* 1e-6 */
  double rope_theta;      /* 1e6 */
  int tie_word_embeddings;/* must be 1 (model_schema.js:43-45) */
  int attention_bias;     /* q/k/v bias (config.js:46) */
} eg_config;

/* QwenWGPU constructor opts (runtime.js:85-128, :541-570) plus B200 knobs. */
typedef struct {
  int device;              /* CUDA ordinal */
  int max_ctx;             /* KV cache length, default 8192 */
  int max_prefill_t;       /* prefill cap, default = max_ctx */
  int kv_f16;              /* 1: f16 KV cache with the reference's f16 staging
                              numerics (setUseF16, runtime.js:146-151, the
                              default on shader-f16 devices); 0: f32 path */
  int decode_batch_capacity; /* tokens per eg_decode_greedy call, default 32 */
  int sampling_top_k;      /* default 40 */
  int max_sampling_top_k;  /* default 64 (max 64) */
  int attn_chunk;          /* keys per attention split: 0 = 128 (the reference's
                              CHUNK, runtime.js:330), else 16..128 step 16 */
  int use_graphs;          /* capture the decode step in a CUDA graph (default 1) */
  int use_pdl;             /* programmatic dependent launch (default 1) */
  int use_fused;           /* 1: persistent fused decode kernel (one cooperative
                              launch per token batch) when no LoRA is active;
                              0 (default): per-op kernels in a CUDA graph */
  int prefill_chunk;       /* prompt positions per batched prefill step (2..16,
                              default 16): every weight tile is read once per
                              chunk; 0 = one decode step per prompt token */
  int use_tc_batch;        /* 1: the int4 GEMVs of batched steps of 4 or more
                              lanes (batched decode, chunked prefill) run on
                              the tcgen05 tensor cores (keeps a second,
                              octet-major copy of the int4 weights); 0
                              (default): the integer mma.sync path */
  int prefill_tc;          /* 1 (default): eg_prefill runs prefillBatch's own
                              arithmetic (runtime.js:1936-2087: GEMM4 over the
                              prompt, ROPE_T, ATTN_PREFILL_BLOCK, SILUMUL) as
                              whole-prompt tcgen05 GEMMs and a tensor-core
                              prefill attention (keeps the octet-major weight
                              copy, plus prefill scratch sized for
                              max_prefill_t or prefill_chunk_size positions);
                              0: positions through the decode step's
                              arithmetic (prefill_chunk above) */
  int prefill_chunk_size;  /* prefillChunkSize (runtime.js:118, :1940-1942),
                              prefill_tc only: 0 (default) = the whole prompt
                              in one pass (_prefillFull); n > 0 = passes of n
                              positions (_prefillChunked) */
  int use_l2_prefetch;     /* 1 (default): in the per-op decode step every int4
                              GEMV also prefetches a later matrix of the step
                              into L2 (cp.async.bulk.prefetch), so HBM streams
                              ahead of the kernel chain; 0: off */
} eg_options;

EG_API const char* eg_last_error(void);
EG_API const char* eg_version(void);
EG_API void eg_default_config(eg_config* c);   /* QWEN25_3B */
EG_API void eg_default_options(eg_options* o);

/* new QwenWGPU(device, cfg, opts), runtime.js:87-101.  Allocates nothing
 * large until weights arrive. */
EG_API eg_status eg_create(const eg_config* cfg, const eg_options* opt, eg_rt** out);
EG_API eg_status eg_destroy(eg_rt* rt);

/* ---------------- quantisers (host, bit-exact with quantize.js) ---------- */
/* quantizeInt4Group, quantize.js:81-111.  packed: N*K/8 u32, scale: N*K/group f32. */
EG_API eg_status eg_quantize_int4_group(const float* W, int N, int K, int group,
                                        uint32_t* packed, float* scale);
/* quantizeInt8RowMajor, quantize.js:28-57.  packed: N*K/4 u32, scale: N f32. */
EG_API eg_status eg_quantize_int8_rows(const float* W, int N, int K, uint32_t* packed,
                                       float* scale);

/* ---------------- weights (build(source), runtime.js:326-539) ------------- */
/* ModelUploader.visit (model_uploader.js:39-63): one HF-named f32 tensor,
 * quantised per the schema (model_schema.js:53-126): int4 g128 for the seven
 * projections, int8 rows for model.embed_tokens.weight, f32 for norms and
 * q/k/v biases.  q/k/v and gate/up are packed as _buildPackedProjectionBuffers
 * does (runtime.js:607-659).  Shape errors: "shape mismatch for <name>: ...". */
EG_API eg_status eg_upload_tensor(eg_rt* rt, const char* name, const float* data,
                                  const int64_t* shape, int ndim);
/* Same, for a tensor the caller already quantised in the reference layout.
 * kind: 4 = int4 (packed N*K/8 u32 + N*K/128 scales), 8 = int8 rows. */
EG_API eg_status eg_upload_quantized(eg_rt* rt, const char* name, int kind,
                                     const uint32_t* packed, const float* scale,
                                     const int64_t* shape, int ndim);
/* Streaming safetensors model load (safetensors_loader.js:83-126 +
 * ModelUploader.visit, model_uploader.js:39-63): `path` is a .safetensors
 * file or a directory with model.safetensors.index.json (sharded) or
 * model.safetensors.  Each tensor is decoded from BF16 / F16 / F32 to f32
 * and passed to eg_upload_tensor (schema check, quantisation, upload;
 * unknown names skipped, a repeated name is an error).  *n_visited = the
 * tensors read.  Call eg_finalize afterwards. */
EG_API eg_status eg_load_safetensors(eg_rt* rt, const char* path, int* n_visited);
/* Host-only: decode one tensor of a safetensors file / model directory to
 * f32 (out == NULL: shape query only).  shape receives up to 8 dims. */
EG_API eg_status eg_safetensors_tensor(const char* path, const char* name, float* out,
                                       int64_t capacity, int64_t* shape, int* ndim);
/* build('mock') equivalent with seeded weights instead of zeros: every
 * matrix and q/k/v bias ~ N(0, std) from the SplitMix64/Box-Muller stream
 * of tensor id t (seed_t = stream(seed)[t]; embed t=0, layer i projection p
 * (q,k,v,o,gate,up,down) t=16i+1+p, bias b t=16i+8+b), norms = 1. */
EG_API eg_status eg_build_synthetic(eg_rt* rt, uint64_t seed, double std_w);
/* uploader.finalize + schema.assertComplete (model_schema.js:117-124):
 * "missing N required tensor(s): ..." ; then RoPE tables and KV cache, and
 * the conversion of every int4 matrix and of the LM head into the library's
 * streaming layout (the reference-layout int4 copies are freed). */
EG_API eg_status eg_finalize(eg_rt* rt);

/* ---------------- decode (runtime.js:1466-1793) --------------------------- */
/* token(id, pos), runtime.js:1735-1741: embed id, one decode step at pos,
 * logits left on the device. */
EG_API eg_status eg_token(eg_rt* rt, uint32_t id, int pos);
/* decodeBatch(startPos, K), runtime.js:1776-1793: K = min(K, capacity,
 * max_ctx - start_pos) chained greedy tokens starting from the token held in
 * s.amax; ids copied to out_ids (K entries), *n_out = K. */
EG_API eg_status eg_decode_greedy(eg_rt* rt, int start_pos, int K, uint32_t* out_ids,
                                  int* n_out);
/* decodeBatch without the readback: enqueue K chained greedy steps on the
 * runtime's stream and return at once (ids stay on the device until
 * eg_read_ids).  K is clamped as in eg_decode_greedy; *n_out = K. */
EG_API eg_status eg_decode_greedy_async(eg_rt* rt, int start_pos, int K, int* n_out);
/* Copy the first n ids produced by the last decode call to host memory. */
EG_API eg_status eg_read_ids(eg_rt* rt, uint32_t* out_ids, int n);
/* The runtime's cudaStream_t (as void*), for callers that order their own
 * work (or CUDA events) after the runtime's. */
EG_API void* eg_stream(eg_rt* rt);
/* Wait for all work queued on the runtime; reports asynchronous errors. */
EG_API eg_status eg_sync(eg_rt* rt);
/* prefillBatch(ids), runtime.js:1936-1945: positions 0..T-1; throws
 * "prompt T > maxPrefillT M" / "prompt T > maxCtx M".  Logits of the last
 * position are left on the device and decoding continues at position T.
 * prefill_tc (default): passes of the whole prompt (or prefill_chunk_size
 * positions) through the tcgen05 GEMMs and the prefill attention, the
 * reference's prefill arithmetic.  prefill_tc = 0: positions 0..T-2 in
 * batched chunks of prefill_chunk positions (K/V rows only), the last
 * through the decode step. */
EG_API eg_status eg_prefill(eg_rt* rt, const uint32_t* ids, int T);
/* argmaxLogits(), runtime.js:1602-1629: writes s.amax and returns it. */
EG_API eg_status eg_argmax(eg_rt* rt, uint32_t* out_id);
/* topKLogits(k), runtime.js:1648-1678: k clamped to [1, max_sampling_top_k,
 * vocab]; *k_out = k.  Order: value desc, ties to the lower id. */
EG_API eg_status eg_topk(eg_rt* rt, int k, uint32_t* ids, float* vals, int* k_out);
/* sampleToken(temp, r), runtime.js:1685-1732 (r clamped to [0,1]). */
EG_API eg_status eg_sample(eg_rt* rt, float temp, float r, uint32_t* out_id);
/* readLogits(), runtime.js:1633-1646: vocab floats. */
EG_API eg_status eg_read_logits(eg_rt* rt, float* out);
/* Final hidden state (s.hidden) after the last step: hidden_size floats. */
EG_API eg_status eg_read_hidden(eg_rt* rt, float* out);
/* generate(ids, n, {sample, temp}), runtime.js:2481-2516.  r_seq supplies
 * the uniforms sampleToken would draw (n entries; ignored when !sample). */
EG_API eg_status eg_generate(eg_rt* rt, const uint32_t* prompt, int n_prompt, int max_new,
                             int sample, float temp, const float* r_seq, uint32_t* out_ids);

/* ---------------- LoRA (lora_gpu.js:65-113, runtime.js:717-734) ----------- */
typedef struct {
  const char* key;        /* "layers.I.self_attn.q_proj" (moduleKeyFromTensorName) */
  const float* A;         /* lora_A as stored: [r][in] or [in][r] */
  int64_t a_rows, a_cols;
  const float* B;         /* lora_B as stored: [out][r] or [r][out] */
  int64_t b_rows, b_cols;
  float scale;            /* MLX scale | alpha/r | 2.0 (lora_gpu.js:73-80,108) */
} eg_lora_module;

/* The orientation step of loadLoraAdapterGPU (lora_gpu.js:100-107), on the
 * host: rank = the smallest of A's and B's dimensions; A is transposed to
 * [rank][in_dim] unless it already has rank rows (PEFT lora_A [r][in] stays,
 * MLX lora_a [in][r] turns), B likewise to [rank][out_dim] (PEFT lora_B
 * [out][r] turns, MLX lora_b [r][out] stays).  A_out holds rank*in_dim
 * floats, B_out rank*out_dim.  EG_ERR_ARG when the shapes do not fit. */
EG_API eg_status eg_lora_orient(const float* A, int64_t a_rows, int64_t a_cols, const float* B,
                               int64_t b_rows, int64_t b_cols, int64_t in_dim, int64_t out_dim,
                               float* A_out, float* B_out, int* rank);
/* loadLoraAdapterGPU: rank = smallest dim, A -> [r][in], B -> [r][out]
 * (lora_gpu.js:100-107); device copies owned by the adapter. */
EG_API eg_status eg_lora_create(eg_rt* rt, int n, const eg_lora_module* mods, eg_lora** out);
EG_API eg_status eg_lora_destroy(eg_rt* rt, eg_lora* lora);
/* Replace one module's A/B contents in place (same shapes). */
EG_API eg_status eg_lora_update(eg_rt* rt, eg_lora* lora, const char* key, const float* A,
                                const float* B);
EG_API eg_status eg_set_lora(eg_rt* rt, eg_lora* lora);      /* setLora */
EG_API eg_status eg_clear_lora(eg_rt* rt);                    /* clearLora */
EG_API eg_status eg_invalidate_lora(eg_rt* rt);               /* invalidateLora */

/* ---------------- observability ------------------------------------------ */
/* enableProf/profToken (runtime.js:775-806): one token at (id, pos) with a
 * CUDA event around each kernel; us[] per category in this order:
 * embed+qkv, attn, o, gate_up, down, lm_head.  n_cat receives 6. */
EG_API eg_status eg_profile_token(eg_rt* rt, uint32_t id, int pos, double* us, int* n_cat);
/* The fused path's counterpart of profToken: one greedy step at start_pos
 * (input token = s.amax) with globaltimer stamps; out_ns[2p] = start of phase
 * p on the first CTA, out_ns[2p+1] = latest end of phase p's work over all
 * CTAs.  Phases: 5 per layer (qkv, attn, o, gate_up, down) then the LM head;
 * *n_out = 2 * (5 * num_layers + 1). */
EG_API eg_status eg_profile_fused(eg_rt* rt, int start_pos, uint64_t* out_ns, int n_max,
                                  int* n_out);
/* Vocab-split LM head (multi-GPU single-stream decode; each rank holds the
 * full model and owns a slice of the vocabulary): final RMSNorm of `hidden`
 * (device f32 [hidden_size], e.g. broadcast from the rank that ran the
 * layers), the int8 LM head over rows [row0, row0 + rows) (row0 % 16 == 0)
 * and their argmax: *best_val / *best_id (device; global id, ties to the
 * lower id, as ARGMAX kernels.js:771-784).  logits: device f32 [rows] or
 * NULL (then the runtime's logits buffer at row0 is used).  Asynchronous on
 * `stream` like the single ops; it shares the runtime's argmax scratch, so
 * the caller orders it after the runtime's own stream.  The ranks' (value, id) pairs merge
 * to the single-GPU argmax (vibethinker_webgpu_lora_b200/parallel.py). */
EG_API eg_status eg_lm_head_shard(eg_rt* rt, const float* hidden, int row0, int rows,
                                  float* logits, float* best_val, uint32_t* best_id, void* stream);
/* ---------------- multi-sequence batched decode ---------------------------
 * The reference decodes one sequence per runtime (step(), runtime.js:
 * 1466-1571); these calls run that step for up to 16 sequences at once, each
 * lane with its own KV cache, position and token ids, every weight tile read
 * once per step for all lanes.
 * eg_seq_init: n_slots sequence slots of slot_ctx positions each (KV caches
 * allocated here; 0 frees them); every slot starts empty. */
EG_API eg_status eg_seq_init(eg_rt* rt, int n_slots, int slot_ctx);
/* Paged variant (PagedAttentionManager, runtime.js:2573-2616, with
 * WRITE_KV_PAGE / ATTN_PARTIAL_PAGED, kernels.js:1657-1911): the slots share
 * a pool of n_pages pages of 16 positions per layer; a slot takes pages as
 * its positions are reached (ensureBlocks) and returns them when it gets a
 * new prompt or is released (freeSeq).  A batch call that would need more
 * pages than are free fails with EG_ERR_OOM before launching anything (the
 * reference instead invents block ids past its pool). */
EG_API eg_status eg_seq_init_paged(eg_rt* rt, int n_slots, int slot_ctx, int n_pages);
/* freeSeq: the slot becomes empty and its pages return to the pool. */
EG_API eg_status eg_seq_release(eg_rt* rt, int slot);
/* Free and total pages of the pool (0 / 0 for dense slots). */
EG_API eg_status eg_seq_pages(eg_rt* rt, int* free_pages, int* total_pages);
/* The slot's prompt: ids[0..T) become its known tokens, its position 0. */
EG_API eg_status eg_seq_set_prompt(eg_rt* rt, int slot, const uint32_t* ids, int T);
/* Prefill the slot's prompt up to its last token in batched chunks of 16
 * positions (each chunk one pass over the weights; K/V rows only, no
 * logits); the next batch step consumes the last prompt token. */
EG_API eg_status eg_seq_prefill(eg_rt* rt, int slot);
/* Position (the token the next step consumes) and count of known ids. */
EG_API eg_status eg_seq_state(eg_rt* rt, int slot, int* pos, int* len);
/* `steps` batched steps over the slots seq_ids[0..nseq) (1 <= nseq <= 16,
 * distinct).  A step consumes each slot's token at its position and moves it
 * one on; a slot still inside its prompt keeps the prompt's next token
 * (prefill), a slot past it appends the greedy token (argmax, ties to the
 * lower id).  out[step * nseq + j] = slot j's token at its new position.
 * Requires pos + steps <= slot_ctx - 1 for every slot. */
EG_API eg_status eg_batch_decode(eg_rt* rt, int nseq, const int* seq_ids, int steps,
                                 uint32_t* out);
/* As eg_batch_decode, choosing tokens by topKLogits(k) + sampleToken(temp,
 * r) (runtime.js:1648-1732) with r[step * nseq + j] for slot j. */
EG_API eg_status eg_batch_sample(eg_rt* rt, int nseq, const int* seq_ids, int steps, int k,
                                 float temp, const float* r, uint32_t* out);
/* Logits of lane j (the j-th slot of the last batch call) after its last
 * step: vocab floats. */
EG_API eg_status eg_batch_read_logits(eg_rt* rt, int lane, float* out);
/* memoryFootprintBytes (runtime.js:661-681). */
EG_API eg_status eg_memory_footprint(eg_rt* rt, int64_t* kv_bytes, int64_t* weight_bytes,
                                     int64_t* scratch_bytes);
/* Kernel launches one decode step issues (lastDispatchCount, runtime.js:743). */
EG_API int eg_launches_per_step(eg_rt* rt);

/* ---------------- single ops (kernels.js WGSL entry points) --------------- */
/* GEMV4 / GEMV4_ADD, kernels.js:884-971: y = W4 x (+bias) ; accumulate=1
 * gives y += W4 x.  group must be 128, K % 128 == 0, any N >= 1. */
EG_API eg_status eg_op_gemv_q4(const float* x, const uint32_t* w, const float* scale,
                               const float* bias, int N, int K, int group, float* y,
                               int accumulate, void* stream);
/* The upload-once form of GEMV4 (the reference converts nothing per call:
 * ModelUploader writes the packed weights once, model_uploader.js:39-63, and
 * every gemv4() dispatch reads them, runtime.js:944-964).  eg_op_q4_stream_bytes
 * gives the size of the device layout the library streams (16-row x 128-k
 * blocks with their group scales); eg_op_q4_to_stream writes it from the
 * reference layout (packed u32 [R*N][K/8], f32 scales [R*N][K/128]);
 * eg_op_gemv_q4_stream then runs y = W4 x (+bias) over it with no
 * conversion and no allocation.  err: one device int, zero before the call,
 * set nonzero if a bounded wait inside the kernel gave up.  pdl = 1 lets the
 * launch overlap the tail of the previous kernel on the stream. */
EG_API eg_status eg_op_q4_stream_bytes(int N, int K, int R, uint64_t* bytes);
EG_API eg_status eg_op_q4_to_stream(const uint32_t* w, const float* scale, int N, int K, int R,
                                    void* out, void* stream);
EG_API eg_status eg_op_gemv_q4_stream(const float* x, const void* ws, const float* bias, int N,
                                      int K, float* y, int* err, int pdl, void* stream);
/* The tensor-core weight layout: the stream-layout blocks regrouped
 * octet-major (128-row octets, group, tile), so that the tcgen05 GEMM
 * streams each pipeline stage as one contiguous copy.  Built once, like the
 * stream layout. */
EG_API eg_status eg_op_q4_tc_bytes(int N, int K, int R, uint64_t* bytes);
EG_API eg_status eg_op_q4_stream_to_tc(const void* ws, int N, int K, int R, void* out, void* stream);
/* GEMM4 / GEMM4_ADD_T, kernels.js:389-473: Y[t][n] = W4 x_t (+bias) for
 * T token vectors x [T][K]; accumulate = 1 gives Y += W4 x_t.  use_tc = 1:
 * the tcgen05 tensor-core path (T <= 32) over the tc layout
 * (eg_op_q4_stream_to_tc); 0: the integer mma.sync path (T <= 16) over the
 * stream layout (eg_op_q4_to_stream).  Uses library scratch memory for the
 * staged activations. */
EG_API eg_status eg_op_gemm_q4_stream(const float* x, int T, const void* ws, const float* bias, int N,
                                      int K, float* y, int accumulate, int use_tc, void* stream);
/* GATE_UP_SILU_GEMV4, kernels.js:1021-1072: w/scale hold 2N rows [gate;up]. */
EG_API eg_status eg_op_gate_up_silu(const float* x, const uint32_t* w, const float* scale,
                                    int N, int K, float* y, void* stream);
/* GEMV (int8 rows), kernels.js:20-59: y = (W8 x) * scale[n]. */
EG_API eg_status eg_op_gemv_q8(const float* x, const uint32_t* w, const float* scale, int N,
                               int K, float* y, void* stream);
/* RMSNORM / RMSNORM_F16, kernels.js:128-166. */
EG_API eg_status eg_op_rmsnorm(const float* x, const float* g, int K, float eps, int f16,
                               float* y, void* stream);
/* ROPE_QK / ROPE_QK_F16, kernels.js:205-257 (in place, head_dim 128). */
EG_API eg_status eg_op_rope_qk(float* q, float* k, int nq, int nkv, int pos, const float* cos_t,
                               const float* sin_t, int f16, void* stream);
/* ROPE_QK + KV append (runtime.js:1509-1514) + ATTN_PARTIAL/ATTN_COMBINE
 * (kernels.js:258-388; _F16 variants when kv_f16): qkv = raw [q | k | v],
 * caches [max_ctx][nkv][128] (f16 when kv_f16 else f32); attends over
 * positions 0..pos.  chunk = keys per split: 0 = 128, the reference's fixed
 * CHUNK (runtime.js:330), else a multiple of 16 up to 128.  Uses library
 * scratch memory for the split partials. */
EG_API eg_status eg_op_attn_decode(const float* qkv, void* k_cache, void* v_cache,
                                   const float* cos_t, const float* sin_t, int nh, int nkv,
                                   int pos, int max_ctx, int kv_f16, int chunk, float* out,
                                   void* stream);
/* ROPE_T (kernels.js:588-618) + the K/V rows + ATTN_PREFILL_BLOCK
 * (kernels.js:684-770) of one prefill pass, on the tensor cores:
 * qkv = T raw rows [q | k | v] (nh + 2 nkv heads of 128) for positions
 * q_start .. q_start + T - 1; q is rotated in place, k rotated and v copied
 * into cache rows q_start + t of the dense caches [max_ctx][nkv][128] (f16
 * when kv_f16 else f32), then every row attends causally over cache rows
 * 0 .. q_start + T - 1 in 128-key online-softmax blocks.  out [T][nh*128].
 * Allocates nothing. */
EG_API eg_status eg_op_attn_prefill(float* qkv, int T, void* k_cache, void* v_cache, const float* cos_t,
                                    const float* sin_t, int nh, int nkv, int q_start, int max_ctx, int kv_f16,
                                    float* out, void* stream);
/* No counterpart in the reference.  eg_op_attn_decode for callers that must
 * not allocate device memory at call time (a framework whose caching
 * allocator already holds the device memory, or a latency-critical loop that
 * cannot take cudaMalloc's implicit synchronisation): same arguments and
 * results, with the split partials in a 2 MB static device array loaded with
 * the library instead of library-allocated scratch.  Rejects calls needing
 * nh * ceil((pos+1) / keys) > 4096 slots (EG_ERR_ARG), keys = chunk, or 128
 * when chunk = 0 (e.g. 32 heads at pos 4095 fit with chunk 0).  All calls
 * share the array: calls that overlap on the GPU race.  The first call on a
 * device looks up the array's device address; make it before any stream
 * capture. */
EG_API eg_status eg_op_attn_decode_noalloc(const float* qkv, void* k_cache, void* v_cache,
                                           const float* cos_t, const float* sin_t, int nh,
                                           int nkv, int pos, int max_ctx, int kv_f16, int chunk,
                                           float* out, void* stream);
/* EMBED_BUF, kernels.js:537-550: id read from device memory. */
EG_API eg_status eg_op_embed(const uint32_t* w, const float* scale, const uint32_t* id, int H,
                             float* out, void* stream);
/* LORA_A, kernels.js:60-78: d[r] = A[r] . x. */
EG_API eg_status eg_op_lora_a(const float* x, const float* A, int K, int rank, float* d,
                              void* stream);
/* ARGMAX, kernels.js:771-784 (ties -> lowest index; uses library scratch). */
EG_API eg_status eg_op_argmax(const float* logits, int n, uint32_t* out, void* stream);
/* TOPK_SELECT x k, kernels.js:785-813 (1 <= k <= 64; uses library scratch). */
EG_API eg_status eg_op_topk(const float* logits, int n, int k, uint32_t* ids, float* vals,
                            void* stream);
/* SAMPLE_TOPK, kernels.js:814-883 (k <= 64). */
EG_API eg_status eg_op_sample_topk(const uint32_t* ids, const float* vals, int k, float temp,
                                   float r, uint32_t* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* EMBERGLASS_H */
