// eg_runtime.cu -- the QwenWGPU-equivalent runtime behind the C ABI.
//
// One runtime = one CUDA device + one stream.  Weights live in HBM in the
// reference's packed layouts; q/k/v and gate/up are concatenated at upload as
// _buildPackedProjectionBuffers does (runtime.js:607-659).  The decode step
// (runtime.js:1466-1571) is a fixed sequence of kernels whose only changing
// inputs (position, token id) live in device memory, so the whole step is
// captured once in a CUDA graph and replayed per token; the LM head's last
// block runs argmax and advances the position, so decodeBatch's chain of K
// greedy tokens (runtime.js:1776-1793) needs no host round trip.
#include <stdarg.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "eg_batch.h"
#include "eg_fused.h"
#include "eg_host.h"
#include "eg_kernels.h"
#include "eg_prefill.h"
#include "emberglass.h"

namespace eg {

static thread_local char g_err[1024] = "";

eg_status fail(eg_status st, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return st;
}

#define CK(x)                                                                              \
  do {                                                                                     \
    cudaError_t e_ = (x);                                                                  \
    if (e_ != cudaSuccess) return eg::fail(EG_ERR_CUDA, "%s: %s", #x, cudaGetErrorString(e_)); \
  } while (0)

struct Layer {
  uint32_t *qkv_w = nullptr, *o_w = nullptr, *gu_w = nullptr, *d_w = nullptr;
  float *qkv_s = nullptr, *o_s = nullptr, *gu_s = nullptr, *d_s = nullptr, *qkv_b = nullptr;
  float *in_norm = nullptr, *post_norm = nullptr;
  void *kc = nullptr, *vc = nullptr;
  // stream-layout copies of the int4 matrices (q4_to_stream), built at finalize
  unsigned char *qkv_t = nullptr, *o_t = nullptr, *gu_t = nullptr, *d_t = nullptr;
  // tcgen05 paths (use_tc_batch or prefill_tc), built at finalize from the
  // octet-major regrouping (q4_stream_to_tc, freed afterwards): int8 A images
  // of the split-K GEMV, each MMA row's group scales, and (prefill_tc) the f16
  // A images of the whole-prompt GEMM
  unsigned char *qkv_a8 = nullptr, *o_a8 = nullptr, *gu_a8 = nullptr, *d_a8 = nullptr;
  float *qkv_sc = nullptr, *o_sc = nullptr, *gu_sc = nullptr, *d_sc = nullptr;
  unsigned char *qkv_a = nullptr, *o_a = nullptr, *gu_a = nullptr, *d_a = nullptr;
};

struct DevState {
  int pos;
  int out_idx;
};

}  // namespace eg

struct eg_lora {
  std::vector<eg::LoraMod> table;  // [layers*7], rank 0 where absent
  std::vector<void*> allocs;
  std::vector<int64_t> shapes;     // per slot: rank, in, out
  int max_rank = 0;
};

struct eg_rt {
  eg_config c{};
  eg_options o{};
  cudaStream_t st = nullptr;
  std::vector<eg::Layer> L;
  uint32_t* emb_w = nullptr;
  float* emb_s = nullptr;
  unsigned char* emb_t = nullptr;  // LM head in the int8 stream layout (emb_w stays for EMBED)
  float* final_norm = nullptr;
  float *cosT = nullptr, *sinT = nullptr;
  float *hidden = nullptr, *qkv = nullptr, *attn = nullptr, *tmp = nullptr, *logits = nullptr;
  float *pm = nullptr, *pz = nullptr, *po = nullptr, *lora_d = nullptr;
  eg::DevState* state = nullptr;
  uint32_t *ids = nullptr, *amax = nullptr, *out_ids = nullptr, *sampled = nullptr;
  float* cand_v = nullptr;
  uint32_t* cand_i = nullptr;
  unsigned* counter = nullptr;
  unsigned* attn_counters = nullptr;
  unsigned* lm_counter = nullptr;
  unsigned* fused_sync = nullptr;     // [0] barrier counter, [1] error word
  eg::FusedLayer* d_layers = nullptr;  // device copy of the per-layer pointers
  uint32_t* sample_ids = nullptr;
  float* sample_vals = nullptr;
  eg::LoraMod* lora_table = nullptr;  // device [layers*7]
  uint32_t* h_small = nullptr;        // pinned readback staging
  int max_splits = 0;
  std::vector<void*> allocs;
  std::set<std::string> seen;
  bool finalized = false;
  eg_lora* active = nullptr;
  cudaGraphExec_t graph[2][2][2] = {};  // [greedy][lora][long-context attention]
  int graph_rank[2][2] = {};
  int launches_per_step = 0;
  std::atomic<bool> busy{false};
  int64_t weight_bytes = 0, kv_bytes = 0, scratch_bytes = 0;
  // multi-sequence slots and the batched step's scratch (eg_seq_init)
  int seq_slots = 0, seq_ctx = 0, b_max_splits = 0, b_gpr = 0, b_out_cap = 0, b_r_cap = 0;
  std::vector<void*> seq_kc, seq_vc;        // per layer: [slots][seq_ctx][kv dim]
  std::vector<int> h_seq_pos, h_seq_len;    // host mirror of the slots' pos / len
  int *seq_pos = nullptr, *seq_len = nullptr, *lane_slot = nullptr, *b_step = nullptr;
  uint32_t* seq_ids = nullptr;
  float *b_hidden = nullptr, *b_qkv = nullptr, *b_attn = nullptr, *b_tmp = nullptr,
        *b_logits = nullptr, *b_pm = nullptr, *b_pz = nullptr, *b_po = nullptr,
        *b_lora_d = nullptr, *b_lora_y = nullptr, *b_xmul = nullptr, *b_cand_v = nullptr, *b_topk_vals = nullptr,
        *b_r = nullptr;
  void* b_xb = nullptr;
  void* b_xtc = nullptr;      // tcgen05 B planes (gpr x 64 columns x 128 B)
  float* b_tc_part = nullptr; // tcgen05 GEMV split-octet partials
  unsigned* b_tc_cnt = nullptr;
  int *b_xcor = nullptr, *b_xf = nullptr;
  unsigned* b_attn_counters = nullptr;
  uint32_t *b_choice = nullptr, *b_cand_i = nullptr, *b_topk_ids = nullptr, *b_out = nullptr;
  int seq_lanes_last = 0;
  // paged slots (eg_seq_init_paged): pool of seq_pool_pages 16-row pages per
  // layer, slot s's table at seq_page_table[s * seq_max_pages]
  int seq_pool_pages = 0, seq_max_pages = 0;
  uint32_t* seq_page_table = nullptr;
  int64_t batch_mark = -1;  // scratch_bytes before the batch scratch was allocated
  std::vector<std::vector<uint32_t>> h_pages;  // pages held by each slot
  std::vector<uint32_t> free_pages;
  // whole-prompt prefill (prefill_tc): scratch for p_cap positions per pass,
  // the LoRA part allocated on the first pass with an adapter active
  int p_cap = 0, p_gpr = 0;
  float *p_hidden = nullptr, *p_qkv = nullptr, *p_attn = nullptr, *p_tmp = nullptr;
  float *p_lora_d = nullptr, *p_lora_y = nullptr, *p_part = nullptr;
  void *p_xb = nullptr, *p_xtc = nullptr, *p_xh = nullptr;
  int *p_xcor = nullptr, *p_xf = nullptr;
  unsigned* p_cnt = nullptr;
};

namespace eg {

static eg_status dalloc(eg_rt* rt, void** p, size_t bytes, int64_t* counter) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e != cudaSuccess) return fail(EG_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  rt->allocs.push_back(*p);
  if (counter) *counter += (int64_t)bytes;
  return EG_OK;
}
static void dfree(eg_rt* rt, void** p, int64_t bytes, int64_t* counter) {
  if (!*p) return;
  for (auto& a : rt->allocs)
    if (a == *p) a = nullptr;
  cudaFree(*p);
  *p = nullptr;
  if (counter) *counter -= bytes;
}
#define DALLOC(ptr, bytes, ctr)                                                          \
  do {                                                                                   \
    void* p_ = nullptr;                                                                  \
    eg_status s_ = eg::dalloc(rt, &p_, (bytes), (ctr));                                  \
    if (s_) return s_;                                                                   \
    (ptr) = reinterpret_cast<decltype(ptr)>(p_);                                         \
  } while (0)

struct Busy {
  eg_rt* rt;
  bool ok;
  explicit Busy(eg_rt* r) : rt(r) { ok = !rt->busy.exchange(true); }
  ~Busy() {
    if (ok) rt->busy.store(false);
  }
};

static void drop_graphs(eg_rt* rt) {
  for (auto& g : rt->graph)
    for (auto& gl : g)
      for (auto& x : gl)
        if (x) {
          cudaGraphExecDestroy(x);
          x = nullptr;
        }
}

// ------------------------------------------------------------------ schema
// Tensor names and shapes of model_schema.js:53-113.
enum Role { R_EMBED, R_FINAL_NORM, R_IN_NORM, R_POST_NORM, R_PROJ, R_BIAS, R_UNKNOWN };
struct Desc {
  Role role = R_UNKNOWN;
  int layer = -1, proj = -1;  // proj 0..6 = q,k,v,o,gate,up,down ; bias 0..2
  int64_t rows = 0, cols = 0;  // expected shape (cols 0 => 1-D)
};

static const char* kProj[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                               "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj",
                               "mlp.down_proj"};

static void proj_shape(const eg_config& c, int p, int64_t* N, int64_t* K) {
  const int64_t H = c.hidden_size, QD = (int64_t)c.num_heads * c.head_dim,
                KVD = (int64_t)c.num_kv_heads * c.head_dim, I = c.intermediate_size;
  const int64_t t[7][2] = {{QD, H}, {KVD, H}, {KVD, H}, {H, QD}, {I, H}, {I, H}, {H, I}};
  *N = t[p][0];
  *K = t[p][1];
}

static Desc describe(const eg_config& c, const char* name) {
  Desc d;
  if (!strcmp(name, "model.embed_tokens.weight")) {
    d.role = R_EMBED;
    d.rows = c.vocab_size;
    d.cols = c.hidden_size;
    return d;
  }
  if (!strcmp(name, "model.norm.weight")) {
    d.role = R_FINAL_NORM;
    d.rows = c.hidden_size;
    return d;
  }
  int layer = -1, off = 0;
  if (sscanf(name, "model.layers.%d.%n", &layer, &off) != 1 || off == 0 || layer < 0 ||
      layer >= c.num_layers)
    return d;
  const char* rest = name + off;
  d.layer = layer;
  if (!strcmp(rest, "input_layernorm.weight")) {
    d.role = R_IN_NORM;
    d.rows = c.hidden_size;
    return d;
  }
  if (!strcmp(rest, "post_attention_layernorm.weight")) {
    d.role = R_POST_NORM;
    d.rows = c.hidden_size;
    return d;
  }
  for (int p = 0; p < 7; p++) {
    const size_t n = strlen(kProj[p]);
    if (strncmp(rest, kProj[p], n)) continue;
    if (!strcmp(rest + n, ".weight")) {
      d.role = R_PROJ;
      d.proj = p;
      proj_shape(c, p, &d.rows, &d.cols);
      return d;
    }
    if (p < 3 && c.attention_bias && !strcmp(rest + n, ".bias")) {
      d.role = R_BIAS;
      d.proj = p;
      int64_t K;
      proj_shape(c, p, &d.rows, &K);
      return d;
    }
  }
  return d;
}

static std::vector<std::string> expected_names(const eg_config& c) {
  std::vector<std::string> v = {"model.embed_tokens.weight", "model.norm.weight"};
  char buf[128];
  for (int i = 0; i < c.num_layers; i++) {
    snprintf(buf, sizeof buf, "model.layers.%d.input_layernorm.weight", i);
    v.push_back(buf);
    snprintf(buf, sizeof buf, "model.layers.%d.post_attention_layernorm.weight", i);
    v.push_back(buf);
    for (int p = 0; p < 7; p++) {
      snprintf(buf, sizeof buf, "model.layers.%d.%s.weight", i, kProj[p]);
      v.push_back(buf);
      if (p < 3 && c.attention_bias) {
        snprintf(buf, sizeof buf, "model.layers.%d.%s.bias", i, kProj[p]);
        v.push_back(buf);
      }
    }
  }
  return v;
}

static eg_status check_shape(const char* name, const Desc& d, const int64_t* shape, int ndim) {
  const int want = d.cols ? 2 : 1;
  bool ok = ndim == want && shape && shape[0] == d.rows && (want == 1 || shape[1] == d.cols);
  if (ok) return EG_OK;
  char got[64] = "", exp[64];
  for (int i = 0; i < ndim && shape; i++)
    snprintf(got + strlen(got), sizeof got - strlen(got), i ? ",%lld" : "%lld", (long long)shape[i]);
  if (want == 2)
    snprintf(exp, sizeof exp, "%lld,%lld", (long long)d.rows, (long long)d.cols);
  else
    snprintf(exp, sizeof exp, "%lld", (long long)d.rows);
  return fail(EG_ERR_ARG, "shape mismatch for %s: got [%s], expected [%s]", name, got, exp);
}

// Allocate every weight buffer (once, on the first upload).
static eg_status alloc_weights(eg_rt* rt) {
  if (!rt->L.empty()) return EG_OK;
  const eg_config& c = rt->c;
  const int64_t H = c.hidden_size, QD = (int64_t)c.num_heads * c.head_dim,
                KVD = (int64_t)c.num_kv_heads * c.head_dim, I = c.intermediate_size;
  const int64_t NQKV = QD + 2 * KVD;
  int64_t* wb = &rt->weight_bytes;
  rt->L.resize(c.num_layers);
  for (auto& l : rt->L) {
    DALLOC(l.qkv_w, NQKV * H / 2, wb);
    DALLOC(l.qkv_s, NQKV * (H / 128) * 4, wb);
    DALLOC(l.qkv_b, NQKV * 4, wb);
    DALLOC(l.o_w, H * QD / 2, wb);
    DALLOC(l.o_s, H * (QD / 128) * 4, wb);
    DALLOC(l.gu_w, 2 * I * H / 2, wb);
    DALLOC(l.gu_s, 2 * I * (H / 128) * 4, wb);
    DALLOC(l.d_w, H * I / 2, wb);
    DALLOC(l.d_s, H * (I / 128) * 4, wb);
    DALLOC(l.in_norm, H * 4, wb);
    DALLOC(l.post_norm, H * 4, wb);
    CK(cudaMemsetAsync(l.qkv_b, 0, NQKV * 4, rt->st));  // enc.clearBuffer(bias), runtime.js:625
  }
  DALLOC(rt->emb_w, (int64_t)c.vocab_size * H, wb);
  DALLOC(rt->emb_s, (int64_t)c.vocab_size * 4, wb);
  DALLOC(rt->final_norm, H * 4, wb);
  return EG_OK;
}

// Destination of a projection/bias inside the packed buffers.
static void proj_dest(eg_rt* rt, const Desc& d, uint32_t** w, float** s, int64_t* row0) {
  const eg_config& c = rt->c;
  const int64_t QD = (int64_t)c.num_heads * c.head_dim, KVD = (int64_t)c.num_kv_heads * c.head_dim;
  eg::Layer& l = rt->L[d.layer];
  switch (d.proj) {
    case 0: *w = l.qkv_w; *s = l.qkv_s; *row0 = 0; break;
    case 1: *w = l.qkv_w; *s = l.qkv_s; *row0 = QD; break;
    case 2: *w = l.qkv_w; *s = l.qkv_s; *row0 = QD + KVD; break;
    case 3: *w = l.o_w; *s = l.o_s; *row0 = 0; break;
    case 4: *w = l.gu_w; *s = l.gu_s; *row0 = 0; break;
    case 5: *w = l.gu_w; *s = l.gu_s; *row0 = c.intermediate_size; break;
    default: *w = l.d_w; *s = l.d_s; *row0 = 0; break;
  }
}

static eg_status put_quantized(eg_rt* rt, const char* name, const Desc& d, int kind,
                               const uint32_t* packed, const float* scale) {
  if (d.role == R_EMBED) {
    if (kind != 8) return fail(EG_ERR_ARG, "%s must be int8 rows", name);
    CK(cudaMemcpyAsync(rt->emb_w, packed, d.rows * d.cols, cudaMemcpyHostToDevice, rt->st));
    CK(cudaMemcpyAsync(rt->emb_s, scale, d.rows * 4, cudaMemcpyHostToDevice, rt->st));
  } else {
    if (kind != 4) return fail(EG_ERR_ARG, "%s must be int4 group-128", name);
    uint32_t* w;
    float* s;
    int64_t row0;
    proj_dest(rt, d, &w, &s, &row0);
    const int64_t gpr = d.cols / 128;
    CK(cudaMemcpyAsync(w + row0 * d.cols / 8, packed, d.rows * d.cols / 2, cudaMemcpyHostToDevice,
                       rt->st));
    CK(cudaMemcpyAsync(s + row0 * gpr, scale, d.rows * gpr * 4, cudaMemcpyHostToDevice, rt->st));
  }
  CK(cudaStreamSynchronize(rt->st));
  rt->seen.insert(name);
  return EG_OK;
}

static eg_status put_f32(eg_rt* rt, const char* name, const Desc& d, const float* data) {
  float* dst = nullptr;
  switch (d.role) {
    case R_FINAL_NORM: dst = rt->final_norm; break;
    case R_IN_NORM: dst = rt->L[d.layer].in_norm; break;
    case R_POST_NORM: dst = rt->L[d.layer].post_norm; break;
    case R_BIAS: {
      const eg_config& c = rt->c;
      const int64_t QD = (int64_t)c.num_heads * c.head_dim,
                    KVD = (int64_t)c.num_kv_heads * c.head_dim;
      dst = rt->L[d.layer].qkv_b + (d.proj == 0 ? 0 : d.proj == 1 ? QD : QD + KVD);
      break;
    }
    default: return fail(EG_ERR_ARG, "%s is not an f32 tensor", name);
  }
  CK(cudaMemcpyAsync(dst, data, d.rows * 4, cudaMemcpyHostToDevice, rt->st));
  CK(cudaStreamSynchronize(rt->st));
  rt->seen.insert(name);
  return EG_OK;
}

static eg_status upload_f32_tensor(eg_rt* rt, const char* name, const Desc& d, const float* data) {
  if (d.role == R_EMBED) {
    std::vector<uint32_t> pk((size_t)d.rows * d.cols / 4);
    std::vector<float> sc((size_t)d.rows);
    eg_status s = eg_quantize_int8_rows(data, (int)d.rows, (int)d.cols, pk.data(), sc.data());
    if (s) return s;
    return put_quantized(rt, name, d, 8, pk.data(), sc.data());
  }
  if (d.role == R_PROJ) {
    std::vector<uint32_t> pk((size_t)d.rows * d.cols / 8);
    std::vector<float> sc((size_t)d.rows * d.cols / 128);
    eg_status s = eg_quantize_int4_group(data, (int)d.rows, (int)d.cols, 128, pk.data(), sc.data());
    if (s) return s;
    return put_quantized(rt, name, d, 4, pk.data(), sc.data());
  }
  return put_f32(rt, name, d, data);
}

// ------------------------------------------------------------------ the step
struct StepOpts {
  bool greedy, lora, pdl;
  int lora_rank;
  std::vector<cudaEvent_t>* marks;  // profiling: event after each category
  bool long_ctx;                    // the step's position takes the long-context attention
};

static void mark(eg_rt* rt, const StepOpts& so, int cat, std::vector<int>* cats) {
  if (!so.marks) return;
  cudaEvent_t e;
  cudaEventCreate(&e);
  cudaEventRecord(e, rt->st);
  so.marks->push_back(e);
  cats->push_back(cat);
}

// One decode step at the device-resident position: runtime.js:1466-1571
// with default flags, plus EMBED_BUF in front and (greedy) ARGMAX behind.
static int enqueue_step(eg_rt* rt, const StepOpts& so, std::vector<int>* cats) {
  const eg_config& c = rt->c;
  const int H = c.hidden_size, hd = c.head_dim, QD = c.num_heads * hd, KVD = c.num_kv_heads * hd;
  const int I = c.intermediate_size, NQKV = QD + 2 * KVD;
  cudaStream_t st = rt->st;
  const bool pdl = so.pdl;
  int launches = 0;
  const LoraMod* lt = rt->lora_table;
  const GemvWork wk{reinterpret_cast<int*>(rt->fused_sync + 1)};
  // each GEMV prefetches a later matrix of the step into L2: QKV the layer's
  // gate_up, O its down, gate_up the next QKV, down the next O
  auto pf = [&](const unsigned char* p, size_t bytes) {
    GemvWork w = wk;
    if (rt->o.use_l2_prefetch) {
      w.pf = p;
      w.pf_bytes = bytes;
    }
    return w;
  };
  for (int i = 0; i < c.num_layers; i++) {
    const Layer& l = rt->L[i];
    const Layer* nl = i + 1 < c.num_layers ? &rt->L[i + 1] : nullptr;
    XSrc xa = {};
    xa.mode = i == 0 ? X_EMBED_RMS : X_RMS;
    xa.x = rt->hidden;
    xa.norm_g = l.in_norm;
    xa.eps = c.rms_norm_eps;
    xa.f16 = rt->o.kv_f16;
    xa.emb_w = rt->emb_w;
    xa.emb_s = rt->emb_s;
    xa.pos = &rt->state->pos;
    xa.ids = rt->ids;
    xa.hidden_out = rt->hidden;
    if (so.lora) {
      XSrc xl = xa;
      xl.hidden_out = nullptr;
      lora_a(xl, H, lt + i * 7 + 0, 3, so.lora_rank, rt->lora_d, st, pdl);
      launches++;
    }
    Epi e = {};
    e.mode = EPI_STORE;
    e.y = rt->qkv;
    e.bias = c.attention_bias ? l.qkv_b : nullptr;
    e.N = NQKV;
    e.mods = so.lora ? lt + i * 7 + 0 : nullptr;
    e.lora_d = rt->lora_d;
    e.split1 = QD;
    e.split2 = QD + KVD;
    gemv_q4(l.qkv_t, NQKV, H, xa, e, st, pdl, pf(l.gu_t, q4_stream_bytes(I, H, 2)));
    launches++;
    mark(rt, so, 0, cats);

    AttnArgs a = {};
    a.qkv = rt->qkv;
    a.kc = l.kc;
    a.vc = l.vc;
    a.cosT = rt->cosT;
    a.sinT = rt->sinT;
    a.pos = &rt->state->pos;
    a.nh = c.num_heads;
    a.nkv = c.num_kv_heads;
    a.max_splits = rt->max_splits;
    a.ctx_bound = rt->o.max_ctx;
    a.kv_f16 = rt->o.kv_f16;
    a.chunk = rt->o.attn_chunk;
    a.pm = rt->pm;
    a.pz = rt->pz;
    a.po = rt->po;
    a.out = rt->attn;
    a.counters = rt->attn_counters;
    attn_decode(a, st, pdl, so.long_ctx);
    launches += 1;
    mark(rt, so, 1, cats);

    XSrc xo = {};
    xo.mode = X_PLAIN;
    xo.x = rt->attn;
    if (so.lora) {
      lora_a(xo, QD, lt + i * 7 + 3, 1, so.lora_rank, rt->lora_d, st, pdl);
      launches++;
    }
    Epi eo = {};
    eo.mode = EPI_ADD;  // GEMV4_ADD: hidden += Wo attn (runtime.js:1531)
    eo.y = rt->hidden;
    eo.N = H;
    eo.mods = so.lora ? lt + i * 7 + 3 : nullptr;
    eo.lora_d = rt->lora_d;
    eo.split1 = eo.split2 = H;
    gemv_q4(l.o_t, H, QD, xo, eo, st, pdl, pf(l.d_t, q4_stream_bytes(H, I, 1)));
    launches++;
    mark(rt, so, 2, cats);

    XSrc xb = {};
    xb.mode = X_RMS;
    xb.x = rt->hidden;
    xb.norm_g = l.post_norm;
    xb.eps = c.rms_norm_eps;
    xb.f16 = rt->o.kv_f16;
    if (so.lora) {
      lora_a(xb, H, lt + i * 7 + 4, 2, so.lora_rank, rt->lora_d, st, pdl);
      launches++;
    }
    Epi eg = {};
    eg.mode = EPI_SILU;
    eg.y = rt->tmp;
    eg.N = I;
    eg.mods = so.lora ? lt + i * 7 + 4 : nullptr;
    eg.lora_d = rt->lora_d;
    gemv_q4(l.gu_t, I, H, xb, eg, st, pdl,
            nl ? pf(nl->qkv_t, q4_stream_bytes(NQKV, H, 1)) : wk);
    launches++;
    mark(rt, so, 3, cats);

    XSrc xd = {};
    xd.mode = X_PLAIN;
    xd.x = rt->tmp;
    if (so.lora) {
      lora_a(xd, I, lt + i * 7 + 6, 1, so.lora_rank, rt->lora_d, st, pdl);
      launches++;
    }
    Epi ed = {};
    ed.mode = EPI_ADD;
    ed.y = rt->hidden;
    ed.N = H;
    ed.mods = so.lora ? lt + i * 7 + 6 : nullptr;
    ed.lora_d = rt->lora_d;
    ed.split1 = ed.split2 = H;
    gemv_q4(l.d_t, H, I, xd, ed, st, pdl, nl ? pf(nl->o_t, q4_stream_bytes(H, QD, 1)) : wk);
    launches++;
    mark(rt, so, 4, cats);
  }
  XSrc xf = {};
  xf.mode = X_RMS;
  xf.x = rt->hidden;
  xf.norm_g = rt->final_norm;
  xf.eps = c.rms_norm_eps;
  xf.f16 = rt->o.kv_f16;
  StepTail tail = {};
  tail.pos = &rt->state->pos;
  tail.ids = rt->ids;
  tail.amax = rt->amax;
  tail.out_ids = rt->out_ids;
  tail.out_idx = &rt->state->out_idx;
  tail.greedy = so.greedy ? 1 : 0;
  tail.cand_v = rt->cand_v;
  tail.cand_i = rt->cand_i;
  tail.counter = rt->counter;
  tail.advance = 1;
  gemv_q8(rt->emb_t, rt->emb_s, c.vocab_size, H, xf, rt->logits, &tail, st, pdl, wk);
  launches++;
  mark(rt, so, 5, cats);
  return launches;
}

// Attention of a decode step at position pos: the long-context kernel?
static bool step_long(eg_rt* rt, int pos) {
  AttnArgs a = {};
  a.nh = rt->c.num_heads;
  a.nkv = rt->c.num_kv_heads;
  a.kv_f16 = rt->o.kv_f16;
  a.chunk = rt->o.attn_chunk;
  return attn_long(a, pos);
}

// One decode step at position pos (the device state's position).
static eg_status run_step(eg_rt* rt, bool greedy, int pos) {
  const bool lora = rt->active != nullptr;
  const int rank = lora ? rt->active->max_rank : 0;
  const bool lg = step_long(rt, pos);
  StepOpts so{greedy, lora, rt->o.use_pdl != 0, rank, nullptr, lg};
  if (!rt->o.use_graphs) {
    rt->launches_per_step = enqueue_step(rt, so, nullptr);
    CK(cudaGetLastError());
    return EG_OK;
  }
  cudaGraphExec_t& ge = rt->graph[greedy][lora][lg];
  if (ge && lora && rt->graph_rank[greedy][lg] < rank) {
    cudaGraphExecDestroy(ge);
    ge = nullptr;
  }
  if (!ge) {
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(rt->st, cudaStreamCaptureModeThreadLocal));
    rt->launches_per_step = enqueue_step(rt, so, nullptr);
    cudaError_t e1 = cudaGetLastError();
    cudaError_t e2 = cudaStreamEndCapture(rt->st, &g);
    if (e1 != cudaSuccess) return fail(EG_ERR_CUDA, "step capture: %s", cudaGetErrorString(e1));
    if (e2 != cudaSuccess) return fail(EG_ERR_CUDA, "end capture: %s", cudaGetErrorString(e2));
    cudaError_t e3 = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e3 != cudaSuccess) return fail(EG_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e3));
    if (lora) rt->graph_rank[greedy][lg] = rank;
  }
  CK(cudaGraphLaunch(ge, rt->st));
  return EG_OK;
}

__global__ void set_state_kernel(DevState* s, uint32_t* ids, int pos, int out_idx, int set_id,
                                 uint32_t id, const uint32_t* id_from) {
  s->pos = pos;
  s->out_idx = out_idx;
  if (set_id) ids[pos] = id_from ? *id_from : id;
}

static eg_status set_state(eg_rt* rt, int pos, int set_id, uint32_t id, const uint32_t* id_from) {
  set_state_kernel<<<1, 1, 0, rt->st>>>(rt->state, rt->ids, pos, 0, set_id, id, id_from);
  CK(cudaGetLastError());
  return EG_OK;
}

static eg_status need_ready(eg_rt* rt) {
  if (!rt) return fail(EG_ERR_ARG, "null runtime");
  if (!rt->finalized) return fail(EG_ERR_STATE, "runtime not built: call eg_finalize first");
  return EG_OK;
}

static eg_status sync(eg_rt* rt) {
  CK(cudaStreamSynchronize(rt->st));
  if (rt->fused_sync) {
    unsigned err = 0;
    CK(cudaMemcpy(&err, rt->fused_sync + 1, 4, cudaMemcpyDeviceToHost));
    if (err) return fail(EG_ERR_DEVICE, "a bounded device-side wait timed out");
  }
  return EG_OK;
}

static bool fused_ok(eg_rt* rt) {
  const eg_config& c = rt->c;
  return rt->o.use_fused && !rt->active && c.hidden_size <= 4096 &&
         c.num_heads * c.head_dim <= 4096 && c.intermediate_size <= 12288;
}

// n decode steps from start_pos in one cooperative launch (ids[start_pos..]
// already hold the input tokens; greedy chains argmax into the next id).
static eg_status run_fused(eg_rt* rt, int start_pos, int n, bool greedy, bool lm_every,
                           unsigned long long* prof = nullptr) {
  const eg_config& c = rt->c;
  CK(cudaMemsetAsync(rt->fused_sync, 0, 2 * sizeof(unsigned), rt->st));
  FusedArgs a = {};
  a.layers = rt->d_layers;
  a.layers_n = c.num_layers;
  a.H = c.hidden_size;
  a.QD = c.num_heads * c.head_dim;
  a.KVD = c.num_kv_heads * c.head_dim;
  a.I = c.intermediate_size;
  a.V = c.vocab_size;
  a.nh = c.num_heads;
  a.nkv = c.num_kv_heads;
  a.eps = c.rms_norm_eps;
  a.f16 = rt->o.kv_f16;
  a.emb_w = rt->emb_w;
  a.emb_s = rt->emb_s;
  a.lm = rt->emb_t;
  a.final_norm = rt->final_norm;
  a.cosT = rt->cosT;
  a.sinT = rt->sinT;
  a.hidden = rt->hidden;
  a.qkv = rt->qkv;
  a.attn = rt->attn;
  a.tmp = rt->tmp;
  a.logits = rt->logits;
  a.pm = rt->pm;
  a.pz = rt->pz;
  a.po = rt->po;
  a.attn_counters = rt->attn_counters;
  a.max_splits = rt->max_splits;
  a.attn_chunk = rt->o.attn_chunk;
  a.ids = rt->ids;
  a.amax = rt->amax;
  a.out_ids = rt->out_ids;
  a.state_pos = &rt->state->pos;
  a.cand_v = rt->cand_v;
  a.cand_i = rt->cand_i;
  a.bar = rt->fused_sync;
  a.err = reinterpret_cast<int*>(rt->fused_sync + 1);
  a.start_pos = start_pos;
  a.n_tokens = n;
  a.greedy = greedy ? 1 : 0;
  a.lm_every = lm_every ? 1 : 0;
  a.prof = prof;
  CK(fused_decode(a, rt->st));
  rt->launches_per_step = 1;
  return EG_OK;
}

// n decode steps from start_pos: fused when possible, else the graph step.
static eg_status run_tokens(eg_rt* rt, int start_pos, int n, bool greedy, bool lm_every) {
  if (fused_ok(rt)) return run_fused(rt, start_pos, n, greedy, lm_every);
  for (int k = 0; k < n; k++) {
    eg_status s = run_step(rt, greedy, start_pos + k);
    if (s) return s;
  }
  return EG_OK;
}

static bool parse_key(const char* key, int layers, int* layer, int* proj) {
  int i = -1, off = 0;
  char sub[64] = "";
  if (!key || sscanf(key, "layers.%d.%n", &i, &off) != 1 || off == 0) return false;
  if (i < 0 || i >= layers) return false;
  snprintf(sub, sizeof sub, "%s", key + off);
  for (int p = 0; p < 7; p++)
    if (!strcmp(sub, kProj[p])) {
      *layer = i;
      *proj = p;
      return true;
    }
  return false;
}

// Per-device scratch for single-op entry points.
struct OpScratch {
  std::mutex mu;
  void* p = nullptr;
  size_t bytes = 0;
};
static OpScratch g_scratch[64];
static eg_status op_scratch(size_t bytes, void** out) {
  int dev = 0;
  CK(cudaGetDevice(&dev));
  OpScratch& s = g_scratch[dev & 63];
  std::lock_guard<std::mutex> lk(s.mu);
  if (s.bytes < bytes) {
    if (s.p) {
      CK(cudaDeviceSynchronize());
      cudaFree(s.p);
      s.p = nullptr;
      s.bytes = 0;
    }
    CK(cudaMalloc(&s.p, bytes));
    s.bytes = bytes;
  }
  *out = s.p;
  return EG_OK;
}


// Scratch of one single-op streaming GEMV: the error word and the matrix
// converted to the stream layout (the single-op entry points take the
// reference layout; the conversion is one extra pass over the weights).
static eg_status op_gemv_work(int N, int K, int R, const uint32_t* w, const float* scale,
                              const unsigned char** ws, GemvWork* wk, cudaStream_t st) {
  void* scr = nullptr;
  eg_status s = op_scratch(256 + q4_stream_bytes(N, K, R), &scr);
  if (s) return s;
  char* b = static_cast<char*>(scr);
  wk->err = reinterpret_cast<int*>(b);
  CK(cudaMemsetAsync(b, 0, 4, st));
  unsigned char* t = reinterpret_cast<unsigned char*>(b + 256);
  q4_to_stream(w, scale, N, K, R, t, st);
  CK(cudaGetLastError());
  *ws = t;
  return EG_OK;
}

}  // namespace eg

using namespace eg;

extern "C" {

EG_API const char* eg_last_error(void) { return g_err; }
EG_API const char* eg_version(void) { return "emberglass-b200 0.1 (sm_100a)"; }

EG_API void eg_default_config(eg_config* c) {
  if (!c) return;
  *c = eg_config{2048, 36, 16, 2, 128, 11008, 151936, 1e-6f, 1000000.0, 1, 1};
}
EG_API void eg_default_options(eg_options* o) {
  if (!o) return;
  *o = eg_options{0, 8192, 0, 1, 32, 40, 64, 0, 1, 1, 0, 16, 0, 1, 0, 1};
}

EG_API eg_status eg_create(const eg_config* cfg, const eg_options* opt, eg_rt** out) {
  if (!cfg || !out) return fail(EG_ERR_ARG, "eg_create: null argument");
  *out = nullptr;
  const eg_config& c = *cfg;
  if (!c.tie_word_embeddings)
    return fail(EG_ERR_ARG, "QwenWGPU currently requires tied input/output embeddings");
  if (c.head_dim != 128) return fail(EG_ERR_ARG, "head_dim must be 128");
  if (c.num_heads <= 0 || c.num_heads > 64 || c.num_kv_heads <= 0 ||
      c.num_heads % c.num_kv_heads || c.num_heads / c.num_kv_heads > 8)
    return fail(EG_ERR_ARG,
                "num_heads must be a multiple of num_kv_heads (group <= 8), at most 64 heads");
  if (c.hidden_size % 128 || c.intermediate_size % 128 || (c.num_heads * c.head_dim) % 128 ||
      c.hidden_size > 12288 || c.intermediate_size > 12288)
    return fail(EG_ERR_ARG, "hidden/intermediate sizes must be multiples of 128, at most 12288");
  if (c.vocab_size <= 0 || c.vocab_size > 148 * 2048 || c.num_layers <= 0)
    return fail(EG_ERR_ARG, "vocab_size must be in [1, 303104]");
  eg_options o;
  eg_default_options(&o);
  if (opt) o = *opt;
  if (o.max_ctx <= 0) o.max_ctx = 8192;
  if (o.max_prefill_t <= 0 || o.max_prefill_t > o.max_ctx) o.max_prefill_t = o.max_ctx;
  if (o.decode_batch_capacity <= 0) o.decode_batch_capacity = 32;
  o.prefill_chunk = o.prefill_chunk < 2 ? 0 : std::min(o.prefill_chunk, (int)kBatchMax);
  if (o.prefill_chunk_size < 0) return fail(EG_ERR_ARG, "prefill_chunk_size must be >= 0");
  if (o.max_prefill_t > kPrefillMaxT && o.prefill_tc &&
      (o.prefill_chunk_size == 0 || o.prefill_chunk_size > kPrefillMaxT))
    o.prefill_chunk_size = kPrefillMaxT;  // one pass holds at most kPrefillMaxT positions
  if (o.max_sampling_top_k <= 0 || o.max_sampling_top_k > 64) o.max_sampling_top_k = 64;
  if (o.sampling_top_k <= 0) o.sampling_top_k = 40;
  o.max_sampling_top_k = std::max(o.max_sampling_top_k, std::min(o.sampling_top_k, 64));
  if (o.attn_chunk < 0 || o.attn_chunk > 128 || o.attn_chunk % 16)
    return fail(EG_ERR_ARG, "attn_chunk must be 0 or a multiple of 16 up to 128");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || o.device < 0 || o.device >= ndev)
    return fail(EG_ERR_CUDA, "no CUDA device %d", o.device);
  CK(cudaSetDevice(o.device));
  eg_rt* rt = new eg_rt();
  rt->c = c;
  rt->o = o;
  if (cudaStreamCreateWithFlags(&rt->st, cudaStreamNonBlocking) != cudaSuccess) {
    delete rt;
    return fail(EG_ERR_CUDA, "stream create failed");
  }
  *out = rt;
  return EG_OK;
}

EG_API eg_status eg_destroy(eg_rt* rt) {
  if (!rt) return EG_OK;
  cudaSetDevice(rt->o.device);
  cudaStreamSynchronize(rt->st);
  drop_graphs(rt);
  for (void* p : rt->allocs) cudaFree(p);
  if (rt->h_small) cudaFreeHost(rt->h_small);
  cudaStreamDestroy(rt->st);
  delete rt;
  return EG_OK;
}

EG_API eg_status eg_upload_tensor(eg_rt* rt, const char* name, const float* data,
                                  const int64_t* shape, int ndim) {
  if (!rt || !name || !data) return fail(EG_ERR_ARG, "eg_upload_tensor: null argument");
  if (rt->finalized) return fail(EG_ERR_STATE, "weights are already finalized");
  CK(cudaSetDevice(rt->o.device));
  Desc d = describe(rt->c, name);
  if (d.role == R_UNKNOWN) return EG_OK;  // schema.validateTensor: unknown names are skipped
  if (rt->seen.count(name)) return fail(EG_ERR_ARG, "duplicate tensor %s", name);  // visit()
  eg_status s = check_shape(name, d, shape, ndim);
  if (s) return s;
  if ((s = alloc_weights(rt))) return s;
  return upload_f32_tensor(rt, name, d, data);
}

EG_API eg_status eg_upload_quantized(eg_rt* rt, const char* name, int kind, const uint32_t* packed,
                                     const float* scale, const int64_t* shape, int ndim) {
  if (!rt || !name || !packed || !scale) return fail(EG_ERR_ARG, "eg_upload_quantized: null argument");
  if (rt->finalized) return fail(EG_ERR_STATE, "weights are already finalized");
  CK(cudaSetDevice(rt->o.device));
  Desc d = describe(rt->c, name);
  if (d.role != R_PROJ && d.role != R_EMBED)
    return fail(EG_ERR_ARG, "%s is not a quantised tensor", name);
  if (rt->seen.count(name)) return fail(EG_ERR_ARG, "duplicate tensor %s", name);
  eg_status s = check_shape(name, d, shape, ndim);
  if (s) return s;
  if ((s = alloc_weights(rt))) return s;
  return put_quantized(rt, name, d, kind, packed, scale);
}

EG_API eg_status eg_build_synthetic(eg_rt* rt, uint64_t seed, double std_w) {
  if (!rt) return fail(EG_ERR_ARG, "null runtime");
  if (rt->finalized) return fail(EG_ERR_STATE, "weights are already finalized");
  CK(cudaSetDevice(rt->o.device));
  eg_status s = alloc_weights(rt);
  if (s) return s;
  const eg_config& c = rt->c;
  const int H = c.hidden_size;
  {  // embedding in row chunks (int8 rows quantise independently)
    const int rows = 8192;
    std::vector<float> f((size_t)rows * H);
    std::vector<uint32_t> pk((size_t)rows * H / 4);
    std::vector<float> sc(rows);
    const uint64_t sd = stream_at(seed, 0);
    for (int r0 = 0; r0 < c.vocab_size; r0 += rows) {
      const int nr = std::min(rows, c.vocab_size - r0);
      fill_normal(f.data(), (int64_t)nr * H, sd, std_w, (int64_t)r0 * H);
      if ((s = eg_quantize_int8_rows(f.data(), nr, H, pk.data(), sc.data()))) return s;
      CK(cudaMemcpy(rt->emb_w + (size_t)r0 * H / 4, pk.data(), (size_t)nr * H, cudaMemcpyHostToDevice));
      CK(cudaMemcpy(rt->emb_s + r0, sc.data(), (size_t)nr * 4, cudaMemcpyHostToDevice));
    }
    rt->seen.insert("model.embed_tokens.weight");
  }
  std::vector<float> ones(std::max(H, 1), 1.0f);
  int64_t shp[2] = {H, 0};
  if ((s = eg_upload_tensor(rt, "model.norm.weight", ones.data(), shp, 1))) return s;
  std::vector<float> f;
  char name[160];
  for (int i = 0; i < c.num_layers; i++) {
    snprintf(name, sizeof name, "model.layers.%d.input_layernorm.weight", i);
    if ((s = eg_upload_tensor(rt, name, ones.data(), shp, 1))) return s;
    snprintf(name, sizeof name, "model.layers.%d.post_attention_layernorm.weight", i);
    if ((s = eg_upload_tensor(rt, name, ones.data(), shp, 1))) return s;
    for (int p = 0; p < 7; p++) {
      int64_t sh[2];
      proj_shape(c, p, &sh[0], &sh[1]);
      f.resize((size_t)sh[0] * sh[1]);
      fill_normal(f.data(), sh[0] * sh[1], stream_at(seed, 16 * i + 1 + p), std_w, 0);
      snprintf(name, sizeof name, "model.layers.%d.%s.weight", i, kProj[p]);
      if ((s = eg_upload_tensor(rt, name, f.data(), sh, 2))) return s;
      if (p < 3 && c.attention_bias) {
        f.resize(sh[0]);
        fill_normal(f.data(), sh[0], stream_at(seed, 16 * i + 8 + p), std_w, 0);
        snprintf(name, sizeof name, "model.layers.%d.%s.bias", i, kProj[p]);
        if ((s = eg_upload_tensor(rt, name, f.data(), sh, 1))) return s;
      }
    }
  }
  return EG_OK;
}

EG_API eg_status eg_finalize(eg_rt* rt) {
  if (!rt) return fail(EG_ERR_ARG, "null runtime");
  if (rt->finalized) return EG_OK;
  CK(cudaSetDevice(rt->o.device));
  std::vector<std::string> missing;
  for (auto& n : expected_names(rt->c))
    if (!rt->seen.count(n)) missing.push_back(n);
  if (!missing.empty()) {
    std::string sample;
    for (size_t i = 0; i < missing.size() && i < 12; i++) sample += (i ? ", " : "") + missing[i];
    return fail(EG_ERR_STATE, "missing %zu required tensor(s): %s%s", missing.size(),
                sample.c_str(), missing.size() > 12 ? ", ..." : "");
  }
  const eg_config& c = rt->c;
  const int hd = c.head_dim, H = c.hidden_size, QD = c.num_heads * hd, KVD = c.num_kv_heads * hd;
  const int mc = rt->o.max_ctx;
  std::vector<float> cs((size_t)mc * hd), sn((size_t)mc * hd);
  rope_tables(mc, hd, c.rope_theta, cs.data(), sn.data());
  int64_t* sb = &rt->scratch_bytes;
  DALLOC(rt->cosT, cs.size() * 4, sb);
  DALLOC(rt->sinT, sn.size() * 4, sb);
  CK(cudaMemcpy(rt->cosT, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(rt->sinT, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  {  // stream layouts of the int4 matrices and of the LM head
    const int I = c.intermediate_size, NQKV = QD + 2 * KVD;
    int64_t* wb = &rt->weight_bytes;
    for (auto& l : rt->L) {
      DALLOC(l.qkv_t, q4_stream_bytes(NQKV, H, 1), wb);
      DALLOC(l.o_t, q4_stream_bytes(H, QD, 1), wb);
      DALLOC(l.gu_t, q4_stream_bytes(I, H, 2), wb);
      DALLOC(l.d_t, q4_stream_bytes(H, I, 1), wb);
      q4_to_stream(l.qkv_w, l.qkv_s, NQKV, H, 1, l.qkv_t, rt->st);
      q4_to_stream(l.o_w, l.o_s, H, QD, 1, l.o_t, rt->st);
      q4_to_stream(l.gu_w, l.gu_s, I, H, 2, l.gu_t, rt->st);
      q4_to_stream(l.d_w, l.d_s, H, I, 1, l.d_t, rt->st);
      CK(cudaGetLastError());
      if (rt->o.use_tc_batch || rt->o.prefill_tc) {
        const int Ns[4] = {NQKV, H, I, H}, Ks[4] = {H, QD, H, I}, Rs[4] = {1, 1, 2, 1};
        const unsigned char* src[4] = {l.qkv_t, l.o_t, l.gu_t, l.d_t};
        unsigned char** a8[4] = {&l.qkv_a8, &l.o_a8, &l.gu_a8, &l.d_a8};
        float** sc[4] = {&l.qkv_sc, &l.o_sc, &l.gu_sc, &l.d_sc};
        unsigned char** a16[4] = {&l.qkv_a, &l.o_a, &l.gu_a, &l.d_a};
        for (int m = 0; m < 4; m++) {
          const size_t tcb = q4_tc_bytes(Ns[m], Ks[m], Rs[m]);
          unsigned char* wc = nullptr;
          DALLOC(wc, tcb, nullptr);
          q4_stream_to_tc(src[m], Ns[m], Ks[m], Rs[m], wc, rt->st);
          DALLOC(*a8[m], q4_a8_bytes(Ns[m], Ks[m], Rs[m]), wb);
          DALLOC(*sc[m], q4_row_scale_bytes(Ns[m], Ks[m], Rs[m]), wb);
          q4_tc_to_a8(wc, Ns[m], Ks[m], Rs[m], *a8[m], *sc[m], rt->st);
          if (rt->o.prefill_tc) {
            DALLOC(*a16[m], q4_a16_bytes(Ns[m], Ks[m], Rs[m]), wb);
            q4_tc_to_a16(wc, Ns[m], Ks[m], Rs[m], *a16[m], rt->st);
          }
          CK(cudaGetLastError());
          CK(cudaStreamSynchronize(rt->st));
          dfree(rt, (void**)&wc, 0, nullptr);
        }
      }
    }
    DALLOC(rt->emb_t, q8_stream_bytes(c.vocab_size, H), wb);
    q8_to_stream(rt->emb_w, c.vocab_size, H, rt->emb_t, rt->st);
    CK(cudaGetLastError());
    {  // the stream layouts replace the reference-layout copies
      CK(cudaStreamSynchronize(rt->st));
      for (auto& l : rt->L) {
        dfree(rt, (void**)&l.qkv_w, (int64_t)NQKV * H / 2, wb);
        dfree(rt, (void**)&l.qkv_s, (int64_t)NQKV * (H / 128) * 4, wb);
        dfree(rt, (void**)&l.o_w, (int64_t)H * QD / 2, wb);
        dfree(rt, (void**)&l.o_s, (int64_t)H * (QD / 128) * 4, wb);
        dfree(rt, (void**)&l.gu_w, (int64_t)2 * I * H / 2, wb);
        dfree(rt, (void**)&l.gu_s, (int64_t)2 * I * (H / 128) * 4, wb);
        dfree(rt, (void**)&l.d_w, (int64_t)H * I / 2, wb);
        dfree(rt, (void**)&l.d_s, (int64_t)H * (I / 128) * 4, wb);
      }
    }
  }
  const size_t kvel = (size_t)mc * KVD * (rt->o.kv_f16 ? 2 : 4);
  for (auto& l : rt->L) {
    DALLOC(l.kc, kvel, &rt->kv_bytes);
    DALLOC(l.vc, kvel, &rt->kv_bytes);
    CK(cudaMemset(l.kc, 0, kvel));
    CK(cudaMemset(l.vc, 0, kvel));
  }
  rt->max_splits = attn_max_splits(mc);
  DALLOC(rt->hidden, H * 4, sb);
  DALLOC(rt->qkv, (QD + 2 * KVD) * 4, sb);
  DALLOC(rt->attn, QD * 4, sb);
  DALLOC(rt->tmp, (size_t)c.intermediate_size * 4, sb);
  DALLOC(rt->logits, (size_t)c.vocab_size * 4, sb);
  DALLOC(rt->pm, (size_t)c.num_heads * rt->max_splits * 4, sb);
  DALLOC(rt->pz, (size_t)c.num_heads * rt->max_splits * 4, sb);
  DALLOC(rt->po, (size_t)c.num_heads * rt->max_splits * hd * 4, sb);
  DALLOC(rt->lora_d, 3 * kMaxRank * 4, sb);
  DALLOC(rt->state, sizeof(DevState), sb);
  DALLOC(rt->ids, ((size_t)mc + 1) * 4, sb);
  DALLOC(rt->amax, 4, sb);
  DALLOC(rt->sampled, 4, sb);
  DALLOC(rt->out_ids, (size_t)std::max(rt->o.decode_batch_capacity, mc) * 4, sb);
  const int ncand = std::max(sm_count() * 4, 148 * 64);
  DALLOC(rt->cand_v, (size_t)ncand * 4, sb);
  DALLOC(rt->cand_i, (size_t)ncand * 4, sb);
  DALLOC(rt->counter, 4, sb);
  DALLOC(rt->attn_counters, 64 * 4, sb);
  DALLOC(rt->lm_counter, 4, sb);
  DALLOC(rt->fused_sync, 2 * 4, sb);
  CK(cudaMemset(rt->lm_counter, 0, 4));
  CK(cudaMemset(rt->fused_sync, 0, 8));
  CK(cudaMemset(rt->attn_counters, 0, 64 * 4));
  DALLOC(rt->sample_ids, 64 * 4, sb);
  DALLOC(rt->sample_vals, 64 * 4, sb);
  DALLOC(rt->lora_table, (size_t)c.num_layers * 7 * sizeof(LoraMod), sb);
  CK(cudaMemset(rt->counter, 0, 4));
  CK(cudaMemset(rt->hidden, 0, H * 4));
  CK(cudaMemset(rt->logits, 0, (size_t)c.vocab_size * 4));
  CK(cudaMemset(rt->ids, 0, ((size_t)mc + 1) * 4));
  CK(cudaMemset(rt->amax, 0, 4));
  CK(cudaMemset(rt->state, 0, sizeof(DevState)));
  CK(cudaMemset(rt->lora_table, 0, (size_t)c.num_layers * 7 * sizeof(LoraMod)));
  {
    std::vector<FusedLayer> fl(c.num_layers);
    for (int i = 0; i < c.num_layers; i++) {
      const Layer& l = rt->L[i];
      fl[i] = FusedLayer{l.qkv_t, l.o_t, l.gu_t, l.d_t, c.attention_bias ? l.qkv_b : nullptr,
                         l.in_norm, l.post_norm, l.kc, l.vc};
    }
    DALLOC(rt->d_layers, fl.size() * sizeof(FusedLayer), sb);
    CK(cudaMemcpy(rt->d_layers, fl.data(), fl.size() * sizeof(FusedLayer), cudaMemcpyHostToDevice));
  }
  // ids of a decode batch / a generate call, or topk's 64 ids + 64 values
  CK(cudaMallocHost(&rt->h_small, (size_t)std::max(std::max(mc, rt->o.decode_batch_capacity), 128) * 4 + 64));
  CK(cudaDeviceSynchronize());
  rt->finalized = true;
  return EG_OK;
}

EG_API eg_status eg_token(eg_rt* rt, uint32_t id, int pos) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (pos < 0 || pos >= rt->o.max_ctx) return fail(EG_ERR_ARG, "pos %d outside [0, %d)", pos, rt->o.max_ctx);
  if (id >= (uint32_t)rt->c.vocab_size) return fail(EG_ERR_ARG, "token id %u >= vocab", id);
  CK(cudaSetDevice(rt->o.device));
  if ((s = set_state(rt, pos, 1, id, nullptr))) return s;
  return run_tokens(rt, pos, 1, false, true);
}

EG_API eg_status eg_decode_greedy(eg_rt* rt, int start_pos, int K, uint32_t* out_ids, int* n_out) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (n_out) *n_out = 0;
  K = std::min(K, std::min(rt->o.decode_batch_capacity, rt->o.max_ctx - start_pos));
  if (K <= 0) return EG_OK;
  if (start_pos < 0) return fail(EG_ERR_ARG, "start_pos %d < 0", start_pos);
  Busy b(rt);
  if (!b.ok) return fail(EG_ERR_BUSY, "decodeBatch() is already in flight");
  CK(cudaSetDevice(rt->o.device));
  if ((s = set_state(rt, start_pos, 1, 0, rt->amax))) return s;  // embed s.amax at start_pos
  if ((s = run_tokens(rt, start_pos, K, true, true))) return s;
  CK(cudaMemcpyAsync(rt->h_small, rt->out_ids, (size_t)K * 4, cudaMemcpyDeviceToHost, rt->st));
  if ((s = sync(rt))) return s;
  if (out_ids) memcpy(out_ids, rt->h_small, (size_t)K * 4);
  if (n_out) *n_out = K;
  return EG_OK;
}

EG_API eg_status eg_decode_greedy_async(eg_rt* rt, int start_pos, int K, int* n_out) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (n_out) *n_out = 0;
  if (start_pos < 0) return fail(EG_ERR_ARG, "start_pos %d < 0", start_pos);
  K = std::min(K, std::min(rt->o.decode_batch_capacity, rt->o.max_ctx - start_pos));
  if (K <= 0) return EG_OK;
  CK(cudaSetDevice(rt->o.device));
  if ((s = set_state(rt, start_pos, 1, 0, rt->amax))) return s;
  if ((s = run_tokens(rt, start_pos, K, true, true))) return s;
  if (n_out) *n_out = K;
  return EG_OK;
}

EG_API eg_status eg_read_ids(eg_rt* rt, uint32_t* out_ids, int n) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (n < 0 || n > std::max(rt->o.decode_batch_capacity, rt->o.max_ctx) || (n && !out_ids))
    return fail(EG_ERR_ARG, "read_ids: bad count");
  CK(cudaSetDevice(rt->o.device));
  CK(cudaMemcpyAsync(rt->h_small, rt->out_ids, (size_t)n * 4, cudaMemcpyDeviceToHost, rt->st));
  if ((s = sync(rt))) return s;
  memcpy(out_ids, rt->h_small, (size_t)n * 4);
  return EG_OK;
}

EG_API void* eg_stream(eg_rt* rt) { return rt ? (void*)rt->st : nullptr; }

EG_API eg_status eg_sync(eg_rt* rt) {
  if (!rt) return fail(EG_ERR_ARG, "null runtime");
  CK(cudaSetDevice(rt->o.device));
  return sync(rt);
}

static eg_status prefill_main_chunks(eg_rt* rt, int npos, int chunk);
static eg_status prefill_tc_run(eg_rt* rt, int T);

EG_API eg_status eg_prefill(eg_rt* rt, const uint32_t* ids, int T) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (!ids || T <= 0) return fail(EG_ERR_ARG, "prefill: empty prompt");
  if (T > rt->o.max_prefill_t) return fail(EG_ERR_ARG, "prompt %d > maxPrefillT %d", T, rt->o.max_prefill_t);
  if (T > rt->o.max_ctx) return fail(EG_ERR_ARG, "prompt %d > maxCtx %d", T, rt->o.max_ctx);
  for (int t = 0; t < T; t++)
    if (ids[t] >= (uint32_t)rt->c.vocab_size) return fail(EG_ERR_ARG, "token id %u >= vocab", ids[t]);
  CK(cudaSetDevice(rt->o.device));
  CK(cudaMemcpyAsync(rt->ids, ids, (size_t)T * 4, cudaMemcpyHostToDevice, rt->st));
  if ((s = set_state(rt, 0, 0, 0, nullptr))) return s;
  if (rt->o.prefill_tc) return prefill_tc_run(rt, T);
  // positions 0..T-2 in batched chunks (their K/V rows only), then the last
  // position through the decode step, which leaves its logits
  const int chunk = rt->o.prefill_chunk, pre = chunk ? T - 1 : 0;
  if (pre >= 2) {
    if ((s = prefill_main_chunks(rt, pre, chunk))) return s;
    return run_tokens(rt, pre, T - pre, false, false);
  }
  if ((s = run_tokens(rt, 0, T, false, false))) return s;  // logits of the last position only
  return EG_OK;
}

EG_API eg_status eg_argmax(eg_rt* rt, uint32_t* out_id) {
  eg_status s = need_ready(rt);
  if (s) return s;
  Busy b(rt);
  if (!b.ok) return fail(EG_ERR_BUSY, "argmaxLogits() is already in flight; concurrent generation is not supported");
  CK(cudaSetDevice(rt->o.device));
  argmax(rt->logits, rt->c.vocab_size, rt->amax, rt->cand_v, rt->cand_i, rt->st);
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(rt->h_small, rt->amax, 4, cudaMemcpyDeviceToHost, rt->st));
  if ((s = sync(rt))) return s;
  if (out_id) *out_id = rt->h_small[0];
  return EG_OK;
}

EG_API eg_status eg_topk(eg_rt* rt, int k, uint32_t* ids, float* vals, int* k_out) {
  eg_status s = need_ready(rt);
  if (s) return s;
  Busy b(rt);
  if (!b.ok) return fail(EG_ERR_BUSY, "topKLogits() is already in flight; concurrent sampling is not supported");
  k = std::min(std::max(1, k), std::min(rt->o.max_sampling_top_k, rt->c.vocab_size));
  CK(cudaSetDevice(rt->o.device));
  topk(rt->logits, rt->c.vocab_size, k, rt->sample_ids, rt->sample_vals, rt->cand_v, rt->cand_i, rt->st);
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(rt->h_small, rt->sample_ids, (size_t)k * 4, cudaMemcpyDeviceToHost, rt->st));
  CK(cudaMemcpyAsync(rt->h_small + 64, rt->sample_vals, (size_t)k * 4, cudaMemcpyDeviceToHost, rt->st));
  if ((s = sync(rt))) return s;
  if (ids) memcpy(ids, rt->h_small, (size_t)k * 4);
  if (vals) memcpy(vals, rt->h_small + 64, (size_t)k * 4);
  if (k_out) *k_out = k;
  return EG_OK;
}

static eg_status sample_dev(eg_rt* rt, float temp, float r, uint32_t* also) {
  const int k = std::min(std::min(rt->o.sampling_top_k, rt->o.max_sampling_top_k), rt->c.vocab_size);
  topk(rt->logits, rt->c.vocab_size, k, rt->sample_ids, rt->sample_vals, rt->cand_v, rt->cand_i, rt->st);
  r = std::max(0.f, std::min(1.f, r));
  sample_topk(rt->sample_ids, rt->sample_vals, k, temp > 0 ? temp : 1.0f, r, rt->sampled, also, rt->st);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_sample(eg_rt* rt, float temp, float r, uint32_t* out_id) {
  eg_status s = need_ready(rt);
  if (s) return s;
  Busy b(rt);
  if (!b.ok) return fail(EG_ERR_BUSY, "sampleToken: top-k selection already in flight");
  CK(cudaSetDevice(rt->o.device));
  if ((s = sample_dev(rt, temp, r, nullptr))) return s;
  CK(cudaMemcpyAsync(rt->h_small, rt->sampled, 4, cudaMemcpyDeviceToHost, rt->st));
  if ((s = sync(rt))) return s;
  if (out_id) *out_id = rt->h_small[0];
  return EG_OK;
}

EG_API eg_status eg_read_logits(eg_rt* rt, float* out) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (!out) return fail(EG_ERR_ARG, "null output");
  CK(cudaSetDevice(rt->o.device));
  CK(cudaMemcpyAsync(out, rt->logits, (size_t)rt->c.vocab_size * 4, cudaMemcpyDeviceToHost, rt->st));
  return sync(rt);
}

EG_API eg_status eg_read_hidden(eg_rt* rt, float* out) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (!out) return fail(EG_ERR_ARG, "null output");
  CK(cudaSetDevice(rt->o.device));
  CK(cudaMemcpyAsync(out, rt->hidden, (size_t)rt->c.hidden_size * 4, cudaMemcpyDeviceToHost, rt->st));
  return sync(rt);
}

EG_API eg_status eg_lm_head_shard(eg_rt* rt, const float* hidden, int row0, int rows,
                                  float* logits, float* best_val, uint32_t* best_id, void* stream) {
  eg_status s = need_ready(rt);
  if (s) return s;
  const eg_config& c = rt->c;
  if (!hidden || !best_val || !best_id) return fail(EG_ERR_ARG, "lm_head_shard: null argument");
  if (row0 < 0 || rows <= 0 || row0 % 16 || row0 + rows > c.vocab_size)
    return fail(EG_ERR_ARG, "lm_head_shard: rows [%d, %d) must lie in the vocab, row0 %% 16 == 0",
                row0, row0 + rows);
  CK(cudaSetDevice(rt->o.device));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  XSrc xf = {};
  xf.mode = X_RMS;  // final RMSNorm of the (broadcast) hidden state
  xf.x = hidden;
  xf.norm_g = rt->final_norm;
  xf.eps = c.rms_norm_eps;
  xf.f16 = rt->o.kv_f16;
  StepTail tail = {};
  tail.cand_v = rt->cand_v;
  tail.cand_i = rt->cand_i;
  tail.counter = rt->counter;
  tail.amax = best_id;
  tail.best_v = best_val;
  tail.id0 = (uint32_t)row0;
  tail.advance = 0;
  const int H = c.hidden_size, gpr = (H + 127) / 128;
  const GemvWork wk{reinterpret_cast<int*>(rt->fused_sync + 1)};
  // the shard's rows are a contiguous run of the stream layout (16-row tiles)
  gemv_q8(rt->emb_t + (size_t)(row0 / 16) * gpr * 2048, rt->emb_s + row0, rows, H, xf,
          logits ? logits : rt->logits + row0, &tail, st, false, wk);
  CK(cudaGetLastError());
  return EG_OK;
}

// ------------------------------------------------------------------ multi-sequence
// Sequence slots and the batched step.  The reference decodes one sequence
// per runtime (runtime.js:1466-1571); here up to kBatchMax slots step
// together, each with its own KV cache, position and token ids, and each
// lane's math is the single-sequence step's.
static eg_status seq_free(eg_rt* rt) {
  if (!rt->seq_slots) return EG_OK;
  CK(cudaStreamSynchronize(rt->st));
  const eg_config& c = rt->c;
  const size_t rows = rt->seq_pool_pages ? (size_t)rt->seq_pool_pages * 16
                                          : (size_t)rt->seq_slots * rt->seq_ctx;
  const size_t kvb = rows * c.num_kv_heads * c.head_dim * (rt->o.kv_f16 ? 2 : 4);
  for (size_t i = 0; i < rt->seq_kc.size(); i++) {
    dfree(rt, &rt->seq_kc[i], (int64_t)kvb, &rt->kv_bytes);
    dfree(rt, &rt->seq_vc[i], (int64_t)kvb, &rt->kv_bytes);
  }
  rt->seq_kc.clear();
  rt->seq_vc.clear();
  void** sp[] = {(void**)&rt->seq_pos, (void**)&rt->seq_len, (void**)&rt->lane_slot,
                 (void**)&rt->b_step, (void**)&rt->seq_ids, (void**)&rt->b_hidden,
                 (void**)&rt->b_qkv, (void**)&rt->b_attn, (void**)&rt->b_tmp,
                 (void**)&rt->b_logits, (void**)&rt->b_pm, (void**)&rt->b_pz, (void**)&rt->b_po,
                 (void**)&rt->b_lora_d, (void**)&rt->b_lora_y, (void**)&rt->b_xmul, (void**)&rt->b_cand_v,
                 (void**)&rt->b_topk_vals, (void**)&rt->b_r, (void**)&rt->b_xb,
                 (void**)&rt->b_xcor, (void**)&rt->b_xf, (void**)&rt->b_attn_counters,
                 (void**)&rt->b_choice, (void**)&rt->b_cand_i, (void**)&rt->b_topk_ids,
                 (void**)&rt->b_out, (void**)&rt->seq_page_table, (void**)&rt->b_xtc,
                 (void**)&rt->b_tc_part, (void**)&rt->b_tc_cnt};
  for (void** q : sp) dfree(rt, q, 0, nullptr);
  if (rt->batch_mark >= 0) rt->scratch_bytes = rt->batch_mark;  // everything since is freed
  rt->batch_mark = -1;
  rt->seq_pool_pages = rt->seq_max_pages = 0;
  rt->h_pages.clear();
  rt->free_pages.clear();
  rt->seq_slots = rt->seq_ctx = rt->b_out_cap = rt->b_r_cap = 0;
  rt->h_seq_pos.clear();
  rt->h_seq_len.clear();
  return EG_OK;
}

// Scratch of the batched step (16 lanes), shared by the sequence slots and
// the chunked prefill of the single stream; sized for max_ctx.
static eg_status batch_scratch(eg_rt* rt) {
  if (rt->b_hidden) return EG_OK;
  rt->batch_mark = rt->scratch_bytes;
  const eg_config& c = rt->c;
  const int H = c.hidden_size, hd = c.head_dim, QD = c.num_heads * hd, KVD = c.num_kv_heads * hd;
  const int I = c.intermediate_size, NQKV = QD + 2 * KVD, V = c.vocab_size, B = kBatchMax;
  int64_t* sb = &rt->scratch_bytes;
  rt->b_max_splits = rt->max_splits;
  rt->b_gpr = (std::max(std::max(H, QD), I) + 127) / 128;
  DALLOC(rt->lane_slot, B * 4, sb);
  DALLOC(rt->b_step, 4, sb);
  DALLOC(rt->b_hidden, (size_t)B * H * 4, sb);
  DALLOC(rt->b_qkv, (size_t)B * NQKV * 4, sb);
  DALLOC(rt->b_attn, (size_t)B * QD * 4, sb);
  DALLOC(rt->b_tmp, (size_t)B * I * 4, sb);
  DALLOC(rt->b_logits, (size_t)B * V * 4, sb);
  const size_t part = (size_t)c.num_heads * rt->b_max_splits;
  DALLOC(rt->b_pm, B * part * 4, sb);
  DALLOC(rt->b_pz, B * part * 4, sb);
  DALLOC(rt->b_po, B * part * hd * 4, sb);
  DALLOC(rt->b_lora_d, (size_t)B * 3 * kMaxRank * 4, sb);
  DALLOC(rt->b_lora_y, (size_t)B * std::max(std::max(NQKV, 2 * I), H) * 4, sb);
  DALLOC(rt->b_xb, (size_t)B * rt->b_gpr * 512, sb);
  DALLOC(rt->b_xtc, (size_t)rt->b_gpr * 4 * kBatchMax * 128, sb);
  DALLOC(rt->b_tc_part, gemv_q4_tc_part_bytes(), sb);
  DALLOC(rt->b_tc_cnt, (size_t)gemv_q4_tc_max_octets() * 4, sb);
  DALLOC(rt->b_xcor, (size_t)B * rt->b_gpr * 2 * 4, sb);
  DALLOC(rt->b_xmul, (size_t)B * rt->b_gpr * 2 * 4, sb);
  DALLOC(rt->b_xf, B * 4, sb);
  DALLOC(rt->b_attn_counters, B * 64 * 4, sb);
  DALLOC(rt->b_choice, B * 4, sb);
  const size_t ncand = (size_t)B * std::max(topk_batch_cand(V, 64), kCandMax);
  DALLOC(rt->b_cand_v, ncand * 4, sb);
  DALLOC(rt->b_cand_i, ncand * 4, sb);
  DALLOC(rt->b_topk_ids, B * 64 * 4, sb);
  DALLOC(rt->b_topk_vals, B * 64 * 4, sb);
  CK(cudaMemsetAsync(rt->lane_slot, 0, B * 4, rt->st));
  CK(cudaMemsetAsync(rt->b_xb, 0, (size_t)B * rt->b_gpr * 512, rt->st));
  CK(cudaMemsetAsync(rt->b_xtc, 0, (size_t)rt->b_gpr * 4 * kBatchMax * 128, rt->st));
  CK(cudaMemsetAsync(rt->b_tc_cnt, 0, (size_t)gemv_q4_tc_max_octets() * 4, rt->st));
  CK(cudaMemsetAsync(rt->b_xcor, 0, (size_t)B * rt->b_gpr * 8, rt->st));
  CK(cudaMemsetAsync(rt->b_xmul, 0, (size_t)B * rt->b_gpr * 8, rt->st));
  CK(cudaMemsetAsync(rt->b_xf, 0, B * 4, rt->st));
  CK(cudaMemsetAsync(rt->b_attn_counters, 0, B * 64 * 4, rt->st));
  return EG_OK;
}

static eg_status seq_alloc(eg_rt* rt, int n_slots, int slot_ctx, int n_pages);

// n_pages == 0: every slot owns slot_ctx contiguous rows; n_pages > 0: the
// slots share a pool of n_pages 16-row pages per layer (PagedAttentionManager,
// runtime.js:2573-2616), allocated as positions are reached.
static eg_status seq_setup(eg_rt* rt, int n_slots, int slot_ctx, int n_pages) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (n_slots < 0 || n_slots > 4096 || (n_slots && (slot_ctx < 2 || slot_ctx > rt->o.max_ctx)))
    return fail(EG_ERR_ARG, "seq_init: %d slots of %d positions (2 <= ctx <= maxCtx %d)", n_slots,
                slot_ctx, rt->o.max_ctx);
  if (n_pages < 0 || n_pages > (1 << 24)) return fail(EG_ERR_ARG, "seq_init: %d pages", n_pages);
  Busy b(rt);
  if (!b.ok) return fail(EG_ERR_BUSY, "a decode call is in flight");
  CK(cudaSetDevice(rt->o.device));
  if ((s = seq_free(rt))) return s;
  if (!n_slots) return EG_OK;
  if ((s = seq_alloc(rt, n_slots, slot_ctx, n_pages))) seq_free(rt);  // no partial state
  return s;
}

static eg_status seq_alloc(eg_rt* rt, int n_slots, int slot_ctx, int n_pages) {
  eg_status s;
  const eg_config& c = rt->c;
  const int KVD = c.num_kv_heads * c.head_dim;
  // set first, so that seq_free releases whatever was allocated if this fails
  rt->seq_slots = n_slots;
  rt->seq_ctx = slot_ctx;
  rt->seq_pool_pages = n_pages;
  const size_t rows = n_pages ? (size_t)n_pages * 16 : (size_t)n_slots * slot_ctx;
  const size_t kvb = rows * KVD * (rt->o.kv_f16 ? 2 : 4);
  rt->seq_kc.assign(c.num_layers, nullptr);
  rt->seq_vc.assign(c.num_layers, nullptr);
  for (int i = 0; i < c.num_layers; i++) {
    DALLOC(rt->seq_kc[i], kvb, &rt->kv_bytes);
    DALLOC(rt->seq_vc[i], kvb, &rt->kv_bytes);
    CK(cudaMemsetAsync(rt->seq_kc[i], 0, kvb, rt->st));
    CK(cudaMemsetAsync(rt->seq_vc[i], 0, kvb, rt->st));
  }
  if ((s = batch_scratch(rt))) return s;
  int64_t* sb = &rt->scratch_bytes;
  DALLOC(rt->seq_pos, (size_t)n_slots * 4, sb);
  DALLOC(rt->seq_len, (size_t)n_slots * 4, sb);
  DALLOC(rt->seq_ids, (size_t)n_slots * slot_ctx * 4, sb);
  CK(cudaMemsetAsync(rt->seq_pos, 0, (size_t)n_slots * 4, rt->st));
  CK(cudaMemsetAsync(rt->seq_len, 0, (size_t)n_slots * 4, rt->st));
  CK(cudaMemsetAsync(rt->seq_ids, 0, (size_t)n_slots * slot_ctx * 4, rt->st));
  rt->h_seq_pos.assign(n_slots, 0);
  rt->h_seq_len.assign(n_slots, 0);
  if (n_pages) {
    rt->seq_max_pages = (slot_ctx + 15) / 16;
    DALLOC(rt->seq_page_table, (size_t)n_slots * rt->seq_max_pages * 4, sb);
    CK(cudaMemsetAsync(rt->seq_page_table, 0, (size_t)n_slots * rt->seq_max_pages * 4, rt->st));
    rt->h_pages.assign(n_slots, {});
    rt->free_pages.resize(n_pages);
    for (int i = 0; i < n_pages; i++) rt->free_pages[i] = (uint32_t)(n_pages - 1 - i);  // pop() = 0, 1, ...
  }
  CK(cudaStreamSynchronize(rt->st));
  return EG_OK;
}

EG_API eg_status eg_seq_init(eg_rt* rt, int n_slots, int slot_ctx) {
  return seq_setup(rt, n_slots, slot_ctx, 0);
}

EG_API eg_status eg_seq_init_paged(eg_rt* rt, int n_slots, int slot_ctx, int n_pages) {
  if (n_slots && n_pages < 1) return fail(EG_ERR_ARG, "seq_init_paged: need at least one page");
  return seq_setup(rt, n_slots, slot_ctx, n_pages);
}

// freeSeq: the slot's pages go back to the pool (most recent first).
static void release_pages(eg_rt* rt, int slot) {
  if (!rt->seq_pool_pages) return;
  auto& hp = rt->h_pages[slot];
  rt->free_pages.insert(rt->free_pages.end(), hp.begin(), hp.end());
  hp.clear();
}

// ensureBlocks: pages for positions [0, n_pos) of the slot; the table row is
// uploaded when it grew.  All or none: when the pool cannot cover the whole
// request, the pages taken by this call go back to the pool, so the slot's
// page list and its device table row always agree.  Fails (nothing
// launched) when the pool is short.
static eg_status ensure_pages(eg_rt* rt, int slot, int n_pos) {
  if (!rt->seq_pool_pages) return EG_OK;
  auto& hp = rt->h_pages[slot];
  const size_t need = (size_t)(n_pos + 15) / 16, had = hp.size();
  if (need > had && need - had > rt->free_pages.size())
    return fail(EG_ERR_OOM, "out of KV pages (%d in the pool, %zu free): slot %d needs %zu more",
                rt->seq_pool_pages, rt->free_pages.size(), slot, need - had);
  while (hp.size() < need) {
    hp.push_back(rt->free_pages.back());
    rt->free_pages.pop_back();
  }
  if (hp.size() != had)
    CK(cudaMemcpy(rt->seq_page_table + (size_t)slot * rt->seq_max_pages + had, hp.data() + had,
                  (hp.size() - had) * 4, cudaMemcpyHostToDevice));
  return EG_OK;
}

EG_API eg_status eg_seq_release(eg_rt* rt, int slot) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (slot < 0 || slot >= rt->seq_slots) return fail(EG_ERR_ARG, "slot %d out of range", slot);
  Busy b(rt);
  if (!b.ok) return fail(EG_ERR_BUSY, "a decode call is in flight");
  CK(cudaSetDevice(rt->o.device));
  CK(cudaStreamSynchronize(rt->st));
  release_pages(rt, slot);
  const int z = 0;
  CK(cudaMemcpy(rt->seq_len + slot, &z, 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(rt->seq_pos + slot, &z, 4, cudaMemcpyHostToDevice));
  rt->h_seq_pos[slot] = rt->h_seq_len[slot] = 0;
  return EG_OK;
}

EG_API eg_status eg_seq_pages(eg_rt* rt, int* free_pages, int* total_pages) {
  if (!rt) return fail(EG_ERR_ARG, "null runtime");
  if (free_pages) *free_pages = (int)rt->free_pages.size();
  if (total_pages) *total_pages = rt->seq_pool_pages;
  return EG_OK;
}

EG_API eg_status eg_seq_set_prompt(eg_rt* rt, int slot, const uint32_t* ids, int T) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (slot < 0 || slot >= rt->seq_slots)
    return fail(EG_ERR_ARG, "slot %d out of range (%d slots)", slot, rt->seq_slots);
  if (T < 1 || !ids) return fail(EG_ERR_ARG, "prompt of %d ids", T);
  if (T > rt->seq_ctx) return fail(EG_ERR_ARG, "prompt %d > slot ctx %d", T, rt->seq_ctx);
  for (int i = 0; i < T; i++)
    if (ids[i] >= (uint32_t)rt->c.vocab_size)
      return fail(EG_ERR_ARG, "token id %u >= vocab %d", ids[i], rt->c.vocab_size);
  Busy b(rt);
  if (!b.ok) return fail(EG_ERR_BUSY, "a decode call is in flight");
  CK(cudaSetDevice(rt->o.device));
  CK(cudaStreamSynchronize(rt->st));
  release_pages(rt, slot);  // a new sequence in this slot
  CK(cudaMemcpy(rt->seq_ids + (size_t)slot * rt->seq_ctx, ids, (size_t)T * 4,
                cudaMemcpyHostToDevice));
  const int pl[2] = {0, T};
  CK(cudaMemcpy(rt->seq_pos + slot, &pl[0], 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(rt->seq_len + slot, &pl[1], 4, cudaMemcpyHostToDevice));
  rt->h_seq_pos[slot] = 0;
  rt->h_seq_len[slot] = T;
  return EG_OK;
}

EG_API eg_status eg_seq_state(eg_rt* rt, int slot, int* pos, int* len) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (slot < 0 || slot >= rt->seq_slots) return fail(EG_ERR_ARG, "slot %d out of range", slot);
  if (pos) *pos = rt->h_seq_pos[slot];
  if (len) *len = rt->h_seq_len[slot];
  return EG_OK;
}

// Where a batched step's lanes live: the sequence table and, per layer, the
// K/V cache base (dense: slot s at s * kv_slot_bytes; paged: the pool).
struct BatchTarget {
  SeqTable sq;
  std::vector<void*> kc, vc;
  size_t kv_slot_bytes;
  const uint32_t* page_table;
  int max_pages;
};

static BatchTarget slots_target(eg_rt* rt, bool chunk) {
  const eg_config& c = rt->c;
  BatchTarget t;
  t.sq = SeqTable{rt->lane_slot, rt->seq_pos, rt->seq_len, rt->seq_ids, rt->seq_ctx,
                  (uint32_t)c.vocab_size, chunk ? 1 : 0};
  t.kc = rt->seq_kc;
  t.vc = rt->seq_vc;
  t.kv_slot_bytes = (size_t)rt->seq_ctx * c.num_kv_heads * c.head_dim * (rt->o.kv_f16 ? 2 : 4);
  t.page_table = rt->seq_page_table;
  t.max_pages = rt->seq_max_pages;
  return t;
}

// The single stream as slot 0 of a one-slot table (its cache is the dense
// [max_ctx][kv dim] layout, its position the decode state's).
static BatchTarget main_target(eg_rt* rt) {
  const eg_config& c = rt->c;
  BatchTarget t;
  t.sq = SeqTable{rt->lane_slot, &rt->state->pos, nullptr, rt->ids, rt->o.max_ctx,
                  (uint32_t)c.vocab_size, 1};
  for (auto& l : rt->L) {
    t.kc.push_back(l.kc);
    t.vc.push_back(l.vc);
  }
  t.kv_slot_bytes = 0;
  t.page_table = nullptr;
  t.max_pages = 0;
  return t;
}

// One batched step over lanes 0..n-1 (lane v = slot lane_slot[v]).  Chunk
// mode (chunked prefill): the lanes are consecutive positions of one slot;
// the K/V rows are appended before the attention and there is no LM head.
static int enqueue_batch_step(eg_rt* rt, int n, bool sample, int k, float temp,
                              const BatchTarget& tg) {
  const eg_config& c = rt->c;
  const int H = c.hidden_size, hd = c.head_dim, QD = c.num_heads * hd, KVD = c.num_kv_heads * hd;
  const int I = c.intermediate_size, NQKV = QD + 2 * KVD, V = c.vocab_size;
  cudaStream_t st = rt->st;
  int* err = reinterpret_cast<int*>(rt->fused_sync + 1);
  const bool lora = rt->active != nullptr;
  const int rank = lora ? rt->active->max_rank : 0;
  const LoraMod* lt = rt->lora_table;
  const int dstride = 3 * kMaxRank;
  const SeqTable& sq = tg.sq;
  const bool chunk = sq.chunk != 0;
  BatchPlanes xp = {};
  xp.xb = rt->b_xb;
  xp.xcor = rt->b_xcor;
  xp.xmul = rt->b_xmul;
  xp.xf = rt->b_xf;
  xp.gpr_max = rt->b_gpr;
  // 4 or more lanes: the int4 GEMVs on the tcgen05 tensor cores
  const bool tc = rt->o.use_tc_batch && n >= 4 && rt->L[0].qkv_a8;
  xp.xtc = tc ? rt->b_xtc : nullptr;
  xp.tc_tpad = (n + 3) / 4 * 4;
  int launches = 0;
  const bool pdl = rt->o.use_pdl != 0;
  auto gemv4 = [&](const unsigned char* w, const unsigned char* a8, const float* sc, int N, int K,
                   const BatchEpi& e) {
    if (tc)
      gemv_q4_tc(a8, sc, N, K, e.e.mode == EPI_SILU ? 2 : 1, n, xp, e, rt->b_tc_part, rt->b_tc_cnt, err, st,
                 pdl);
    else
      gemv_q4_batch(w, N, K, n, xp, e, err, st, pdl);
  };
  auto src = [&](int mode, const float* x, const float* g, int stride) {
    BatchSrc b = {};
    b.x.mode = mode;
    b.x.x = x;
    b.x.norm_g = g;
    b.x.eps = c.rms_norm_eps;
    b.x.f16 = rt->o.kv_f16;
    b.x.emb_w = rt->emb_w;
    b.x.emb_s = rt->emb_s;
    b.stride = stride;
    b.seq = sq;
    return b;
  };
  auto epi = [&](int mode, float* y, int N, int ystride, const float* bias, int m, int s1, int s2) {
    BatchEpi e = {};
    e.e.mode = mode;
    e.e.y = y;
    e.e.N = N;
    e.e.bias = bias;
    e.e.mods = lora ? lt + m : nullptr;
    e.e.lora_d = rt->b_lora_d;
    e.e.split1 = s1;
    e.e.split2 = s2;
    e.ystride = ystride;
    e.dstride = dstride;
    if (lora && tc) {  // the tcgen05 epilogue reads the LoRA B terms ahead of the GEMV
      const int rows = mode == EPI_SILU ? 2 * N : N;
      e.lora_pre = rt->b_lora_y;
      e.lstride = rows;
      lora_b_batch(e, rows, n, rt->b_lora_y, st, pdl);
      launches++;
    }  // the mma.sync GEMV computes them at each tile hand-off (lora_pre null, mods set)
    return e;
  };
  for (int i = 0; i < c.num_layers; i++) {
    const Layer& l = rt->L[i];
    BatchSrc xa = src(i == 0 ? X_EMBED_RMS : X_RMS, rt->b_hidden, l.in_norm, H);
    if (i == 0) xa.x.hidden_out = rt->b_hidden;
    // the LoRA A rows fold into the staging when the adapter is small
    if (!batch_stage_q4(xa, H, n, xp, st, pdl, lora ? lt + i * 7 + 0 : nullptr, 3, rank, rt->b_lora_d, dstride) &&
        lora) {
      BatchSrc xl = xa;
      xl.x.hidden_out = nullptr;
      lora_a_batch(xl, H, lt + i * 7 + 0, 3, rank, rt->b_lora_d, dstride, n, st, pdl);
      launches++;
    }
    gemv4(l.qkv_t, l.qkv_a8, l.qkv_sc, NQKV, H,
          epi(EPI_STORE, rt->b_qkv, NQKV, NQKV, c.attention_bias ? l.qkv_b : nullptr, i * 7 + 0, QD,
              QD + KVD));
    launches += 2;
    AttnArgs a = {};
    a.qkv = rt->b_qkv;
    a.kc = tg.kc[i];
    a.vc = tg.vc[i];
    a.cosT = rt->cosT;
    a.sinT = rt->sinT;
    a.nh = c.num_heads;
    a.nkv = c.num_kv_heads;
    a.max_splits = rt->b_max_splits;
    a.ctx_bound = tg.sq.slot_ctx;
    a.kv_f16 = rt->o.kv_f16;
    a.chunk = rt->o.attn_chunk;
    a.pm = rt->b_pm;
    a.pz = rt->b_pz;
    a.po = rt->b_po;
    a.out = rt->b_attn;
    a.counters = rt->b_attn_counters;
    AttnBatch ab;
    ab.seq = sq;
    ab.qkv_stride = NQKV;
    ab.out_stride = QD;
    ab.part_stride = c.num_heads * rt->b_max_splits;
    ab.kv_slot_bytes = tg.kv_slot_bytes;
    ab.page_table = tg.page_table;
    ab.max_pages = tg.max_pages;
    if (chunk) {  // every lane's row first, then attention reads them all (no early start)
      kv_append_batch(a, ab, n, st);
      attn_batch(a, ab, n, st, false);
      launches += 2;
    } else {
      attn_batch(a, ab, n, st, pdl);
      launches++;
    }
    BatchSrc xo = src(X_PLAIN, rt->b_attn, nullptr, QD);
    if (!batch_stage_q4(xo, QD, n, xp, st, pdl, lora ? lt + i * 7 + 3 : nullptr, 1, rank, rt->b_lora_d,
                        dstride) &&
        lora) {
      lora_a_batch(xo, QD, lt + i * 7 + 3, 1, rank, rt->b_lora_d, dstride, n, st, pdl);
      launches++;
    }
    gemv4(l.o_t, l.o_a8, l.o_sc, H, QD, epi(EPI_ADD, rt->b_hidden, H, H, nullptr, i * 7 + 3, H, H));
    launches += 2;
    BatchSrc xb = src(X_RMS, rt->b_hidden, l.post_norm, H);
    if (!batch_stage_q4(xb, H, n, xp, st, pdl, lora ? lt + i * 7 + 4 : nullptr, 2, rank, rt->b_lora_d,
                        dstride) &&
        lora) {
      lora_a_batch(xb, H, lt + i * 7 + 4, 2, rank, rt->b_lora_d, dstride, n, st, pdl);
      launches++;
    }
    gemv4(l.gu_t, l.gu_a8, l.gu_sc, I, H, epi(EPI_SILU, rt->b_tmp, I, I, nullptr, i * 7 + 4, I, I));
    launches += 2;
    BatchSrc xd = src(X_PLAIN, rt->b_tmp, nullptr, I);
    if (!batch_stage_q4(xd, I, n, xp, st, pdl, lora ? lt + i * 7 + 6 : nullptr, 1, rank, rt->b_lora_d,
                        dstride) &&
        lora) {
      lora_a_batch(xd, I, lt + i * 7 + 6, 1, rank, rt->b_lora_d, dstride, n, st, pdl);
      launches++;
    }
    gemv4(l.d_t, l.d_a8, l.d_sc, H, I, epi(EPI_ADD, rt->b_hidden, H, H, nullptr, i * 7 + 6, H, H));
    launches += 2;
  }
  if (chunk) {  // chunked prefill: no logits for these positions
    batch_advance(sq, rt->b_choice, n, rt->b_out, rt->b_step, st);
    return launches + 1;
  }
  BatchSrc xf = src(X_RMS, rt->b_hidden, rt->final_norm, H);
  batch_stage_q8(xf, H, n, xp, st, pdl);
  gemv_q8_batch(rt->emb_t, rt->emb_s, V, H, n, xp, rt->b_logits, V, err, st, pdl);
  launches += 2;
  if (!sample) {
    argmax_batch(rt->b_logits, V, n, rt->b_choice, rt->b_cand_v, rt->b_cand_i, st);
    launches += 2;
  } else {
    topk_batch(rt->b_logits, V, k, n, rt->b_topk_ids, rt->b_topk_vals, rt->b_cand_v,
               rt->b_cand_i, st);
    sample_batch(rt->b_topk_ids, rt->b_topk_vals, k, temp, rt->b_r, rt->b_step, n, rt->b_choice,
                 st);
    launches += 3;
  }
  batch_advance(sq, rt->b_choice, n, rt->b_out, rt->b_step, st);
  return launches + 1;
}

// Chunked prefill of `npos` positions of slot `slot` of the target, from
// its current position: steps of `chunk` consecutive positions (one weight
// pass each; the full-chunk step captured once as a graph), then the tail.
// The batch scratch must exist before `tg` was built (its sequence table
// points into it).
static eg_status run_chunks(eg_rt* rt, const BatchTarget& tg, int slot, int npos, int chunk) {
  if (npos <= 0) return EG_OK;
  if (!rt->b_hidden || tg.sq.lane_slot != rt->lane_slot)
    return fail(EG_ERR_STATE, "batched prefill: scratch not allocated");
  int lanes[kBatchMax];
  for (int& l : lanes) l = slot;
  CK(cudaMemcpyAsync(rt->lane_slot, lanes, sizeof lanes, cudaMemcpyHostToDevice, rt->st));
  const int full = npos / chunk, tail = npos % chunk;
  if (full >= 2 && rt->o.use_graphs) {
    cudaGraph_t g;
    cudaGraphExec_t ge = nullptr;
    CK(cudaStreamBeginCapture(rt->st, cudaStreamCaptureModeThreadLocal));
    enqueue_batch_step(rt, chunk, false, 1, 1.f, tg);
    cudaError_t e1 = cudaGetLastError();
    cudaError_t e2 = cudaStreamEndCapture(rt->st, &g);
    if (e1 != cudaSuccess) return fail(EG_ERR_CUDA, "prefill capture: %s", cudaGetErrorString(e1));
    if (e2 != cudaSuccess) return fail(EG_ERR_CUDA, "end capture: %s", cudaGetErrorString(e2));
    cudaError_t e3 = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e3 != cudaSuccess) return fail(EG_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e3));
    cudaError_t e4 = cudaSuccess;
    for (int t = 0; t < full && e4 == cudaSuccess; t++) e4 = cudaGraphLaunch(ge, rt->st);
    cudaError_t e5 = cudaStreamSynchronize(rt->st);
    cudaGraphExecDestroy(ge);
    if (e4 != cudaSuccess) return fail(EG_ERR_CUDA, "graph launch: %s", cudaGetErrorString(e4));
    if (e5 != cudaSuccess) return fail(EG_ERR_CUDA, "prefill chunks: %s", cudaGetErrorString(e5));
  } else {
    for (int t = 0; t < full; t++) enqueue_batch_step(rt, chunk, false, 1, 1.f, tg);
  }
  if (tail) enqueue_batch_step(rt, tail, false, 1, 1.f, tg);
  CK(cudaGetLastError());
  return EG_OK;
}

// The single stream's positions 0..npos-1 (its decode-state position is 0).
static eg_status prefill_main_chunks(eg_rt* rt, int npos, int chunk) {
  eg_status s = batch_scratch(rt);  // before the target captures its pointers
  if (s) return s;
  return run_chunks(rt, main_target(rt), 0, npos, chunk);
}

// Scratch of the whole-prompt prefill, for passes of up to `cap` positions.
static eg_status prefill_scratch(eg_rt* rt, int cap, bool lora) {
  const eg_config& c = rt->c;
  const int H = c.hidden_size, QD = c.num_heads * c.head_dim, KVD = c.num_kv_heads * c.head_dim;
  const int I = c.intermediate_size, NQKV = QD + 2 * KVD;
  int64_t* sb = &rt->scratch_bytes;
  if (!rt->p_hidden) {
    rt->p_cap = cap;
    rt->p_gpr = (std::max(std::max(H, QD), I) + 127) / 128;
    const size_t T = (size_t)cap, gpr = (size_t)rt->p_gpr, tiles = (T + 127) / 128;
    DALLOC(rt->p_hidden, T * H * 4, sb);
    DALLOC(rt->p_qkv, T * NQKV * 4, sb);
    DALLOC(rt->p_attn, T * QD * 4, sb);
    DALLOC(rt->p_tmp, T * I * 4, sb);
    DALLOC(rt->p_xb, T * gpr * 512, sb);
    DALLOC(rt->p_xcor, T * gpr * 8, sb);
    DALLOC(rt->p_xf, T * 4, sb);
    DALLOC(rt->p_xtc, gpr * 32 * 4 * 128, sb);
    DALLOC(rt->p_xh, tiles * gpr * 65536, sb);
    DALLOC(rt->p_part, gemv_q4_tc_part_bytes(), sb);
    DALLOC(rt->p_cnt, (size_t)gemv_q4_tc_max_octets() * 4, sb);
    CK(cudaMemsetAsync(rt->p_xtc, 0, gpr * 32 * 4 * 128, rt->st));
    CK(cudaMemsetAsync(rt->p_xh, 0, tiles * gpr * 65536, rt->st));
    CK(cudaMemsetAsync(rt->p_cnt, 0, (size_t)gemv_q4_tc_max_octets() * 4, rt->st));
  }
  if (lora && !rt->p_lora_y) {
    DALLOC(rt->p_lora_d, (size_t)rt->p_cap * 3 * kMaxRank * 4, sb);
    DALLOC(rt->p_lora_y, (size_t)rt->p_cap * std::max(std::max(NQKV, 2 * I), H) * 4, sb);
  }
  return EG_OK;
}

// One prefill pass over positions off .. off + n - 1 of the single stream
// (ids already on the device), prefillBatch's per-layer sequence
// (runtime.js:1967-2080): RMSNORM_T, GEMM4 q/k/v (+bias, LoRA), ROPE_T and the
// K/V rows, ATTN_PREFILL_BLOCK over keys 0 .. off + n - 1, GEMM4_ADD_T o,
// RMSNORM_T, GEMM4 gate/up + SILUMUL, GEMM4_ADD_T down.  Returns launches.
static int enqueue_prefill_pass(eg_rt* rt, int off, int n) {
  const eg_config& c = rt->c;
  const int H = c.hidden_size, hd = c.head_dim, QD = c.num_heads * hd, KVD = c.num_kv_heads * hd;
  const int I = c.intermediate_size, NQKV = QD + 2 * KVD;
  cudaStream_t st = rt->st;
  int* err = reinterpret_cast<int*>(rt->fused_sync + 1);
  const bool lora = rt->active != nullptr;
  const int rank = lora ? rt->active->max_rank : 0;
  const LoraMod* lt = rt->lora_table;
  const int dstride = 3 * kMaxRank;
  const int f16 = rt->o.kv_f16;
  BatchPlanes xp = {};
  xp.xb = rt->p_xb;
  xp.xcor = rt->p_xcor;
  xp.xf = rt->p_xf;
  xp.gpr_max = rt->p_gpr;
  // up to 32 rows: split-K gemv_q4_tc over digit planes; more: the f16 GEMM
  xp.xtc = n > 32 ? nullptr : rt->p_xtc;
  xp.tc_tpad = (n + 3) / 4 * 4;
  xp.xh = n > 32 ? rt->p_xh : nullptr;
  int launches = 0;
  auto src = [&](int mode, const float* x, const float* g, int stride) {
    BatchSrc b = {};
    b.x.mode = mode;
    b.x.x = x;
    b.x.norm_g = g;
    b.x.eps = c.rms_norm_eps;
    b.x.f16 = f16;
    b.stride = stride;
    return b;
  };
  auto gemm = [&](const unsigned char* a8, const unsigned char* a16, const float* sc, int N, int K, int R,
                  const BatchSrc& x, int nmods, int mode, float* y, int ystride, const float* bias, int m, int s1,
                  int s2) {
    if (!batch_stage_q4(x, K, n, xp, st, false, lora ? lt + m : nullptr, nmods, rank, rt->p_lora_d, dstride) &&
        lora) {
      lora_a_batch(x, K, lt + m, nmods, rank, rt->p_lora_d, dstride, n, st, false);
      launches++;
    }
    BatchEpi e = {};
    e.e.mode = mode;
    e.e.y = y;
    e.e.N = N;
    e.e.bias = bias;
    e.e.mods = lora ? lt + m : nullptr;
    e.e.lora_d = rt->p_lora_d;
    e.e.split1 = s1;
    e.e.split2 = s2;
    e.ystride = ystride;
    e.dstride = dstride;
    e.add_first = 1;
    e.silu_f16 = f16;
    if (lora) {
      const int rows = mode == EPI_SILU ? 2 * N : N;
      e.lora_pre = rt->p_lora_y;
      e.lstride = rows;
      lora_b_batch(e, rows, n, rt->p_lora_y, st, false);
      launches++;
    }
    if (n > 32)
      gemm_q4_prefill(a16, sc, N, K, R, n, xp, e, err, st);
    else
      gemv_q4_tc(a8, sc, N, K, R, n, xp, e, rt->p_part, rt->p_cnt, err, st, false);
    launches += 2;
  };
  prefill_embed(rt->ids + off, rt->emb_w, rt->emb_s, n, H, rt->p_hidden, st);
  launches++;
  for (int i = 0; i < c.num_layers; i++) {
    const Layer& l = rt->L[i];
    gemm(l.qkv_a8, l.qkv_a, l.qkv_sc, NQKV, H, 1, src(X_RMS, rt->p_hidden, l.in_norm, H), 3, EPI_STORE, rt->p_qkv, NQKV,
         c.attention_bias ? l.qkv_b : nullptr, i * 7 + 0, QD, QD + KVD);
    prefill_rope_append(rt->p_qkv, n, NQKV, c.num_heads, c.num_kv_heads, off, rt->cosT, rt->sinT, f16, l.kc, l.vc,
                        st);
    PrefillAttn pa = {};
    pa.qkv = rt->p_qkv;
    pa.qkv_stride = NQKV;
    pa.kc = l.kc;
    pa.vc = l.vc;
    pa.nh = c.num_heads;
    pa.nkv = c.num_kv_heads;
    pa.kv_f16 = f16;
    pa.T = n;
    pa.q_start = off;
    pa.ctx = off + n;
    pa.out = rt->p_attn;
    pa.out_stride = QD;
    attn_prefill(pa, st);
    launches += 2;
    gemm(l.o_a8, l.o_a, l.o_sc, H, QD, 1, src(X_PLAIN, rt->p_attn, nullptr, QD), 1, EPI_ADD, rt->p_hidden, H, nullptr, i * 7 + 3,
         H, H);
    gemm(l.gu_a8, l.gu_a, l.gu_sc, I, H, 2, src(X_RMS, rt->p_hidden, l.post_norm, H), 2, EPI_SILU, rt->p_tmp, I, nullptr, i * 7 + 4,
         I, I);
    gemm(l.d_a8, l.d_a, l.d_sc, H, I, 1, src(X_PLAIN, rt->p_tmp, nullptr, I), 1, EPI_ADD, rt->p_hidden, H, nullptr, i * 7 + 6, H,
         H);
  }
  return launches;
}

// prefillBatch through the tcgen05 passes: _prefillFull when the prompt fits
// one pass, else _prefillChunked; then the last row's final norm and LM head
// (runtime.js:2081-2084), and the decode state moves to position T.
static eg_status prefill_tc_run(eg_rt* rt, int T) {
  const eg_config& c = rt->c;
  const int H = c.hidden_size;
  const int cs = rt->o.prefill_chunk_size;
  const int pass = (cs > 0 && T > cs) ? cs : T;
  const int cap = cs > 0 ? std::min(cs, rt->o.max_prefill_t) : rt->o.max_prefill_t;
  eg_status s = prefill_scratch(rt, std::max(cap, pass), rt->active != nullptr);
  if (s) return s;
  if (pass > rt->p_cap) return fail(EG_ERR_STATE, "prefill pass of %d positions > scratch %d", pass, rt->p_cap);
  int last = 0;
  for (int off = 0; off < T; off += pass) {
    last = std::min(pass, T - off);
    enqueue_prefill_pass(rt, off, last);
  }
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(rt->hidden, rt->p_hidden + (size_t)(last - 1) * H, (size_t)H * 4, cudaMemcpyDeviceToDevice,
                     rt->st));
  XSrc xf = {};
  xf.mode = X_RMS;
  xf.x = rt->hidden;
  xf.norm_g = rt->final_norm;
  xf.eps = c.rms_norm_eps;
  xf.f16 = rt->o.kv_f16;
  gemv_q8(rt->emb_t, rt->emb_s, c.vocab_size, H, xf, rt->logits, nullptr, rt->st, false,
          GemvWork{reinterpret_cast<int*>(rt->fused_sync + 1)});
  CK(cudaGetLastError());
  return set_state(rt, T, 0, 0, nullptr);
}

EG_API eg_status eg_seq_prefill(eg_rt* rt, int slot) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (slot < 0 || slot >= rt->seq_slots) return fail(EG_ERR_ARG, "slot %d out of range", slot);
  const int pos = rt->h_seq_pos[slot], len = rt->h_seq_len[slot];
  if (len < 1) return fail(EG_ERR_STATE, "slot %d has no prompt", slot);
  const int npos = len - 1 - pos;  // the last prompt token is left to the next batch step
  if (npos <= 0) return EG_OK;
  Busy b(rt);
  if (!b.ok) return fail(EG_ERR_BUSY, "a decode call is in flight");
  CK(cudaSetDevice(rt->o.device));
  if ((s = ensure_pages(rt, slot, len - 1))) return s;
  if ((s = run_chunks(rt, slots_target(rt, true), slot, npos, kBatchMax))) return s;
  if ((s = sync(rt))) return s;
  rt->h_seq_pos[slot] = len - 1;
  return EG_OK;
}

static eg_status batch_run(eg_rt* rt, int nseq, const int* seq_ids, int steps, bool sample, int k,
                           float temp, const float* r, uint32_t* out) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (!rt->seq_slots) return fail(EG_ERR_STATE, "no sequence slots: call eg_seq_init first");
  if (nseq < 1 || nseq > kBatchMax || !seq_ids)
    return fail(EG_ERR_ARG, "batch of %d sequences (1..%d)", nseq, kBatchMax);
  if (steps < 0 || (steps && !out)) return fail(EG_ERR_ARG, "steps %d", steps);
  if (sample && steps && !r) return fail(EG_ERR_ARG, "sampling needs r[steps][nseq]");
  std::vector<int> seen(rt->seq_slots, 0);
  for (int j = 0; j < nseq; j++) {
    const int sl = seq_ids[j];
    if (sl < 0 || sl >= rt->seq_slots) return fail(EG_ERR_ARG, "slot %d out of range", sl);
    if (seen[sl]++) return fail(EG_ERR_ARG, "slot %d listed twice", sl);
    if (rt->h_seq_len[sl] < 1) return fail(EG_ERR_STATE, "slot %d has no prompt", sl);
    if (rt->h_seq_pos[sl] + steps > rt->seq_ctx - 1)
      return fail(EG_ERR_ARG, "slot %d: position %d + %d steps exceeds its ctx %d", sl,
                  rt->h_seq_pos[sl], steps, rt->seq_ctx);
  }
  if (!steps) return EG_OK;
  if (sample) {
    k = std::max(1, std::min(k, std::min(rt->o.max_sampling_top_k, rt->c.vocab_size)));
    for (int i = 0; i < steps * nseq; i++)
      if (!(r[i] >= 0.f)) return fail(EG_ERR_ARG, "r[%d] is negative or NaN", i);
  }
  Busy b(rt);
  if (!b.ok) return fail(EG_ERR_BUSY, "a decode call is in flight");
  CK(cudaSetDevice(rt->o.device));
  int64_t* sb = &rt->scratch_bytes;
  if (rt->b_out_cap < steps * nseq) {
    dfree(rt, (void**)&rt->b_out, 0, nullptr);
    DALLOC(rt->b_out, (size_t)steps * nseq * 4, sb);
    rt->b_out_cap = steps * nseq;
  }
  if (sample) {
    if (rt->b_r_cap < steps) {
      dfree(rt, (void**)&rt->b_r, 0, nullptr);
      DALLOC(rt->b_r, (size_t)steps * kBatchMax * 4, sb);
      rt->b_r_cap = steps;
    }
    std::vector<float> rp((size_t)steps * kBatchMax, 0.f);
    for (int t = 0; t < steps; t++)
      for (int j = 0; j < nseq; j++) rp[(size_t)t * kBatchMax + j] = std::min(r[t * nseq + j], 1.f);
    CK(cudaMemcpyAsync(rt->b_r, rp.data(), rp.size() * 4, cudaMemcpyHostToDevice, rt->st));
    CK(cudaStreamSynchronize(rt->st));
  }
  if (rt->seq_pool_pages) {  // pages for every position these steps write, all or none
    std::vector<size_t> had(nseq);
    for (int j = 0; j < nseq; j++) had[j] = rt->h_pages[seq_ids[j]].size();
    for (int j = 0; j < nseq; j++) {
      if ((s = ensure_pages(rt, seq_ids[j], rt->h_seq_pos[seq_ids[j]] + steps))) {
        for (int q = 0; q < nseq; q++) {
          auto& hp = rt->h_pages[seq_ids[q]];
          while (hp.size() > had[q]) {
            rt->free_pages.push_back(hp.back());
            hp.pop_back();
          }
        }
        return s;
      }
    }
  }
  int lanes[kBatchMax] = {0};
  for (int j = 0; j < nseq; j++) lanes[j] = seq_ids[j];
  CK(cudaMemcpyAsync(rt->lane_slot, lanes, sizeof lanes, cudaMemcpyHostToDevice, rt->st));
  CK(cudaMemsetAsync(rt->b_step, 0, 4, rt->st));
  if (rt->o.use_graphs) {
    cudaGraph_t g;
    cudaGraphExec_t ge = nullptr;
    CK(cudaStreamBeginCapture(rt->st, cudaStreamCaptureModeThreadLocal));
    rt->launches_per_step = enqueue_batch_step(rt, nseq, sample, k, temp, slots_target(rt, false));
    cudaError_t e1 = cudaGetLastError();
    cudaError_t e2 = cudaStreamEndCapture(rt->st, &g);
    if (e1 != cudaSuccess) return fail(EG_ERR_CUDA, "batch step capture: %s", cudaGetErrorString(e1));
    if (e2 != cudaSuccess) return fail(EG_ERR_CUDA, "end capture: %s", cudaGetErrorString(e2));
    cudaError_t e3 = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e3 != cudaSuccess) return fail(EG_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e3));
    cudaError_t e4 = cudaSuccess;
    for (int t = 0; t < steps && e4 == cudaSuccess; t++) e4 = cudaGraphLaunch(ge, rt->st);
    cudaError_t e5 = cudaStreamSynchronize(rt->st);
    cudaGraphExecDestroy(ge);
    if (e4 != cudaSuccess) return fail(EG_ERR_CUDA, "graph launch: %s", cudaGetErrorString(e4));
    if (e5 != cudaSuccess) return fail(EG_ERR_CUDA, "batch steps: %s", cudaGetErrorString(e5));
  } else {
    for (int t = 0; t < steps; t++)
      rt->launches_per_step = enqueue_batch_step(rt, nseq, sample, k, temp, slots_target(rt, false));
    CK(cudaGetLastError());
  }
  rt->seq_lanes_last = nseq;
  std::vector<uint32_t> h((size_t)steps * nseq);
  CK(cudaMemcpyAsync(h.data(), rt->b_out, h.size() * 4, cudaMemcpyDeviceToHost, rt->st));
  if ((s = sync(rt))) return s;
  memcpy(out, h.data(), h.size() * 4);
  for (int j = 0; j < nseq; j++) {
    const int sl = seq_ids[j];
    rt->h_seq_pos[sl] += steps;
    rt->h_seq_len[sl] = std::max(rt->h_seq_len[sl], rt->h_seq_pos[sl] + 1);
  }
  return EG_OK;
}

EG_API eg_status eg_batch_decode(eg_rt* rt, int nseq, const int* seq_ids, int steps,
                                 uint32_t* out) {
  return batch_run(rt, nseq, seq_ids, steps, false, 1, 1.f, nullptr, out);
}

EG_API eg_status eg_batch_sample(eg_rt* rt, int nseq, const int* seq_ids, int steps, int k,
                                 float temp, const float* r, uint32_t* out) {
  return batch_run(rt, nseq, seq_ids, steps, true, k, temp, r, out);
}

EG_API eg_status eg_batch_read_logits(eg_rt* rt, int lane, float* out) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (lane < 0 || lane >= rt->seq_lanes_last || !out)
    return fail(EG_ERR_ARG, "lane %d of the last batch (%d lanes)", lane, rt->seq_lanes_last);
  CK(cudaSetDevice(rt->o.device));
  CK(cudaMemcpyAsync(out, rt->b_logits + (size_t)lane * rt->c.vocab_size,
                     (size_t)rt->c.vocab_size * 4, cudaMemcpyDeviceToHost, rt->st));
  return sync(rt);
}

EG_API eg_status eg_generate(eg_rt* rt, const uint32_t* prompt, int n_prompt, int max_new,
                             int sample, float temp, const float* r_seq, uint32_t* out_ids) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (max_new <= 0) return EG_OK;
  if (!out_ids || (sample && !r_seq)) return fail(EG_ERR_ARG, "generate: null output / r_seq");
  if (n_prompt + max_new - 1 > rt->o.max_ctx)
    return fail(EG_ERR_ARG, "prompt %d + %d new tokens exceed maxCtx %d", n_prompt, max_new, rt->o.max_ctx);
  if ((s = eg_prefill(rt, prompt, n_prompt))) return s;
  if (!sample) {
    uint32_t first;
    if ((s = eg_argmax(rt, &first))) return s;
    out_ids[0] = first;
    int done = 1, pos = n_prompt;
    while (done < max_new) {
      int n = 0;
      if ((s = eg_decode_greedy(rt, pos, max_new - done, out_ids + done, &n))) return s;
      if (n <= 0) return fail(EG_ERR_STATE, "generate: context exhausted");
      done += n;
      pos += n;
    }
    return EG_OK;
  }
  CK(cudaSetDevice(rt->o.device));
  // sampled: GPU-resident loop, the sampled id is written straight into
  // s.amax (generate's writeBuffer, runtime.js:2494) and the id buffer.
  const float t = temp > 0 ? temp : 1.0f;
  int pos = n_prompt;
  for (int g = 0; g < max_new; g++) {
    if ((s = sample_dev(rt, t, r_seq[g], rt->amax))) return s;
    copy_u32(rt->amax, rt->out_ids + g, rt->st);
    if (g + 1 == max_new) break;
    if ((s = set_state(rt, pos, 1, 0, rt->amax))) return s;
    if ((s = run_tokens(rt, pos, 1, false, true))) return s;
    pos++;
  }
  CK(cudaMemcpyAsync(rt->h_small, rt->out_ids, (size_t)max_new * 4, cudaMemcpyDeviceToHost, rt->st));
  if ((s = sync(rt))) return s;
  memcpy(out_ids, rt->h_small, (size_t)max_new * 4);
  return EG_OK;
}

// ---------------------------------------------------------------- LoRA
EG_API eg_status eg_lora_orient(const float* A, int64_t a_rows, int64_t a_cols, const float* B,
                               int64_t b_rows, int64_t b_cols, int64_t in_dim, int64_t out_dim,
                               float* A_out, float* B_out, int* rank) {
  if (!A || !B || !A_out || !B_out || !rank) return fail(EG_ERR_ARG, "lora_orient: null argument");
  // rank = the smallest dimension (lora_gpu.js:101); A -> [r][in] unless it
  // already has r rows, B -> [r][out] likewise (lora_gpu.js:102-107)
  const int64_t r = std::min(std::min(a_rows, a_cols), std::min(b_rows, b_cols));
  if (r <= 0) return fail(EG_ERR_ARG, "lora_orient: empty A or B");
  const bool a_t = a_rows != r, b_t = b_rows != r;
  const int64_t a_in = a_t ? a_rows : a_cols, b_out = b_t ? b_rows : b_cols;
  if (a_in != in_dim || b_out != out_dim)
    return fail(EG_ERR_ARG, "lora_orient: A %lldx%lld / B %lldx%lld do not give [%lld][%lld] / [%lld][%lld]",
                (long long)a_rows, (long long)a_cols, (long long)b_rows, (long long)b_cols, (long long)r,
                (long long)in_dim, (long long)r, (long long)out_dim);
  for (int64_t i = 0; i < r; i++)
    for (int64_t k = 0; k < in_dim; k++) A_out[i * in_dim + k] = a_t ? A[k * r + i] : A[i * in_dim + k];
  for (int64_t i = 0; i < r; i++)
    for (int64_t j = 0; j < out_dim; j++) B_out[i * out_dim + j] = b_t ? B[j * r + i] : B[i * out_dim + j];
  *rank = (int)r;
  return EG_OK;
}

EG_API eg_status eg_lora_create(eg_rt* rt, int n, const eg_lora_module* mods, eg_lora** out) {
  if (!rt || !out || (n > 0 && !mods)) return fail(EG_ERR_ARG, "eg_lora_create: null argument");
  *out = nullptr;
  CK(cudaSetDevice(rt->o.device));
  const eg_config& c = rt->c;
  eg_lora* lo = new eg_lora();
  lo->table.assign((size_t)c.num_layers * 7, LoraMod{nullptr, nullptr, 0, 0.f});
  lo->shapes.assign((size_t)c.num_layers * 7 * 3, 0);
  auto bail = [&](eg_status st) {
    for (void* p : lo->allocs) cudaFree(p);
    delete lo;
    return st;
  };
  int matched = 0;
  for (int m = 0; m < n; m++) {
    const eg_lora_module& md = mods[m];
    int layer, p;
    if (!parse_key(md.key, c.num_layers, &layer, &p)) continue;
    if (!md.A || !md.B) continue;
    int64_t N, K;
    proj_shape(c, p, &N, &K);
    const int64_t r = std::min(std::min(md.a_rows, md.a_cols), std::min(md.b_rows, md.b_cols));
    if (r <= 0 || r > kMaxRank)
      return bail(fail(EG_ERR_ARG, "%s: rank %lld outside [1, %d]", md.key, (long long)r, kMaxRank));
    std::vector<float> A((size_t)r * K), B((size_t)r * N);
    int rr = 0;
    if (eg_lora_orient(md.A, md.a_rows, md.a_cols, md.B, md.b_rows, md.b_cols, K, N, A.data(), B.data(),
                       &rr) != EG_OK)
      return bail(fail(EG_ERR_ARG, "%s: A/B shapes do not match the %lldx%lld projection", md.key,
                       (long long)N, (long long)K));
    float *dA = nullptr, *dB = nullptr;
    if (cudaMalloc(&dA, A.size() * 4) != cudaSuccess || cudaMalloc(&dB, B.size() * 4) != cudaSuccess) {
      if (dA) cudaFree(dA);
      return bail(fail(EG_ERR_OOM, "LoRA allocation failed"));
    }
    lo->allocs.push_back(dA);
    lo->allocs.push_back(dB);
    if (cudaMemcpy(dA, A.data(), A.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dB, B.data(), B.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return bail(fail(EG_ERR_CUDA, "LoRA upload failed"));
    const size_t slot = (size_t)layer * 7 + p;
    lo->table[slot] = LoraMod{dA, dB, (int)r, md.scale};
    lo->shapes[slot * 3 + 0] = r;
    lo->shapes[slot * 3 + 1] = K;
    lo->shapes[slot * 3 + 2] = N;
    lo->max_rank = std::max(lo->max_rank, (int)r);
    matched++;
  }
  if (!matched) return bail(fail(EG_ERR_ARG, "no LoRA modules matched layers.*.{self_attn,mlp}.*_proj"));
  *out = lo;
  return EG_OK;
}

EG_API eg_status eg_lora_destroy(eg_rt* rt, eg_lora* lora) {
  if (!lora) return EG_OK;
  if (rt && rt->active == lora) eg_clear_lora(rt);
  if (rt) cudaStreamSynchronize(rt->st);
  for (void* p : lora->allocs) cudaFree(p);
  delete lora;
  return EG_OK;
}

EG_API eg_status eg_lora_update(eg_rt* rt, eg_lora* lora, const char* key, const float* A, const float* B) {
  if (!rt || !lora) return fail(EG_ERR_ARG, "null argument");
  int layer, p;
  if (!parse_key(key, rt->c.num_layers, &layer, &p)) return fail(EG_ERR_ARG, "bad module key %s", key ? key : "");
  const size_t slot = (size_t)layer * 7 + p;
  const LoraMod& m = lora->table[slot];
  if (m.rank <= 0) return fail(EG_ERR_ARG, "module %s not in adapter", key);
  CK(cudaSetDevice(rt->o.device));
  const int64_t r = lora->shapes[slot * 3], K = lora->shapes[slot * 3 + 1], N = lora->shapes[slot * 3 + 2];
  if (A) CK(cudaMemcpyAsync((void*)m.A, A, (size_t)r * K * 4, cudaMemcpyHostToDevice, rt->st));
  if (B) CK(cudaMemcpyAsync((void*)m.B, B, (size_t)r * N * 4, cudaMemcpyHostToDevice, rt->st));
  return sync(rt);
}

static eg_status push_table(eg_rt* rt) {
  const size_t n = (size_t)rt->c.num_layers * 7;
  if (!rt->active) return EG_OK;
  CK(cudaMemcpyAsync(rt->lora_table, rt->active->table.data(), n * sizeof(LoraMod),
                     cudaMemcpyHostToDevice, rt->st));
  return sync(rt);
}

EG_API eg_status eg_set_lora(eg_rt* rt, eg_lora* lora) {
  eg_status s = need_ready(rt);
  if (s) return s;
  CK(cudaSetDevice(rt->o.device));
  rt->active = lora;
  return push_table(rt);
}
EG_API eg_status eg_clear_lora(eg_rt* rt) {
  if (!rt) return fail(EG_ERR_ARG, "null runtime");
  rt->active = nullptr;
  return EG_OK;
}
EG_API eg_status eg_invalidate_lora(eg_rt* rt) {
  eg_status s = need_ready(rt);
  if (s) return s;
  CK(cudaSetDevice(rt->o.device));
  return push_table(rt);
}

// ---------------------------------------------------------------- observability
EG_API eg_status eg_profile_token(eg_rt* rt, uint32_t id, int pos, double* us, int* n_cat) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (pos < 0 || pos >= rt->o.max_ctx || id >= (uint32_t)rt->c.vocab_size)
    return fail(EG_ERR_ARG, "profile_token: bad id/pos");
  CK(cudaSetDevice(rt->o.device));
  if ((s = set_state(rt, pos, 1, id, nullptr))) return s;
  std::vector<cudaEvent_t> marks;
  std::vector<int> cats;
  cudaEvent_t start;
  CK(cudaEventCreate(&start));
  CK(cudaEventRecord(start, rt->st));
  StepOpts so{false, rt->active != nullptr, false, rt->active ? rt->active->max_rank : 0, &marks,
              step_long(rt, pos)};
  enqueue_step(rt, so, &cats);
  CK(cudaGetLastError());
  if ((s = sync(rt))) return s;
  double acc[6] = {0, 0, 0, 0, 0, 0};
  cudaEvent_t prev = start;
  for (size_t i = 0; i < marks.size(); i++) {
    float ms = 0;
    cudaEventElapsedTime(&ms, prev, marks[i]);
    acc[cats[i]] += ms * 1000.0;
    prev = marks[i];
  }
  for (auto e : marks) cudaEventDestroy(e);
  cudaEventDestroy(start);
  if (us)
    for (int i = 0; i < 6; i++) us[i] = acc[i];
  if (n_cat) *n_cat = 6;
  return EG_OK;
}

EG_API eg_status eg_profile_fused(eg_rt* rt, int start_pos, uint64_t* out_ns, int n_max, int* n_out) {
  eg_status s = need_ready(rt);
  if (s) return s;
  if (!fused_ok(rt)) return fail(EG_ERR_STATE, "fused decode not available (LoRA active or disabled)");
  if (start_pos < 0 || start_pos >= rt->o.max_ctx) return fail(EG_ERR_ARG, "bad start_pos");
  const int nph = 2 * (rt->c.num_layers * 5 + 1);
  if (!out_ns || n_max < nph) return fail(EG_ERR_ARG, "need room for %d timestamps", nph);
  CK(cudaSetDevice(rt->o.device));
  unsigned long long* d = nullptr;
  CK(cudaMalloc(&d, nph * 8));
  CK(cudaMemsetAsync(d, 0, nph * 8, rt->st));
  if ((s = set_state(rt, start_pos, 1, 0, rt->amax))) { cudaFree(d); return s; }
  s = run_fused(rt, start_pos, 1, true, true, d);
  if (!s) s = sync(rt);
  if (!s && cudaMemcpy(out_ns, d, nph * 8, cudaMemcpyDeviceToHost) != cudaSuccess)
    s = fail(EG_ERR_CUDA, "profile readback failed");
  cudaFree(d);
  if (n_out) *n_out = nph;
  return s;
}

EG_API eg_status eg_memory_footprint(eg_rt* rt, int64_t* kv, int64_t* w, int64_t* scratch) {
  if (!rt) return fail(EG_ERR_ARG, "null runtime");
  if (kv) *kv = rt->kv_bytes;
  if (w) *w = rt->weight_bytes;
  if (scratch) *scratch = rt->scratch_bytes;
  return EG_OK;
}

EG_API int eg_launches_per_step(eg_rt* rt) { return rt ? rt->launches_per_step : 0; }

// ---------------------------------------------------------------- single ops
#define OPSTREAM reinterpret_cast<cudaStream_t>(stream)

EG_API eg_status eg_op_gemv_q4(const float* x, const uint32_t* w, const float* scale, const float* bias,
                               int N, int K, int group, float* y, int accumulate, void* stream) {
  if (!x || !w || !scale || !y || N <= 0 || K <= 0) return fail(EG_ERR_ARG, "gemv_q4: bad argument");
  if (reinterpret_cast<uintptr_t>(w) & 15) return fail(EG_ERR_ARG, "gemv_q4: w must be 16-byte aligned");
  if (group != 128 || K % 128 || K > 12288)
    return fail(EG_ERR_ARG, "gemv_q4: group must be 128, K %% 128 == 0, K <= 12288");
  XSrc xs = {};
  xs.mode = X_PLAIN;
  xs.x = x;
  Epi e = {};
  e.mode = accumulate ? EPI_ADD : EPI_STORE;
  e.y = y;
  e.bias = accumulate ? nullptr : bias;
  e.N = N;
  e.split1 = e.split2 = N;
  if (accumulate && bias) return fail(EG_ERR_ARG, "gemv_q4: bias with accumulate is not supported");
  GemvWork wk;
  const unsigned char* ws = nullptr;
  eg_status s = op_gemv_work(N, K, 1, w, scale, &ws, &wk, OPSTREAM);
  if (s) return s;
  gemv_q4(ws, N, K, xs, e, OPSTREAM, false, wk);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_q4_stream_bytes(int N, int K, int R, uint64_t* bytes) {
  if (!bytes || N <= 0 || K <= 0 || K % 128 || K > 12288 || (R != 1 && R != 2))
    return fail(EG_ERR_ARG, "q4_stream_bytes: need K %% 128 == 0, K <= 12288, R = 1 or 2");
  *bytes = q4_stream_bytes(N, K, R);
  return EG_OK;
}

EG_API eg_status eg_op_q4_to_stream(const uint32_t* w, const float* scale, int N, int K, int R, void* out,
                                    void* stream) {
  if (!w || !scale || !out || N <= 0 || K <= 0 || K % 128 || K > 12288 || (R != 1 && R != 2))
    return fail(EG_ERR_ARG, "q4_to_stream: bad argument");
  if (reinterpret_cast<uintptr_t>(out) & 15) return fail(EG_ERR_ARG, "q4_to_stream: out must be 16-byte aligned");
  q4_to_stream(w, scale, N, K, R, static_cast<unsigned char*>(out), OPSTREAM);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_gemv_q4_stream(const float* x, const void* ws, const float* bias, int N, int K,
                                      float* y, int* err, int pdl, void* stream) {
  if (!x || !ws || !y || !err || N <= 0 || K <= 0 || K % 128 || K > 12288)
    return fail(EG_ERR_ARG, "gemv_q4_stream: bad argument");
  if (reinterpret_cast<uintptr_t>(ws) & 15) return fail(EG_ERR_ARG, "gemv_q4_stream: ws must be 16-byte aligned");
  XSrc xs = {};
  xs.mode = X_PLAIN;
  xs.x = x;
  Epi e = {};
  e.mode = EPI_STORE;
  e.y = y;
  e.bias = bias;
  e.N = N;
  e.split1 = e.split2 = N;
  GemvWork wk;
  wk.err = err;
  gemv_q4(static_cast<const unsigned char*>(ws), N, K, xs, e, OPSTREAM, pdl != 0, wk);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_q4_tc_bytes(int N, int K, int R, uint64_t* bytes) {
  if (!bytes || N <= 0 || K <= 0 || K % 128 || K > 12288 || (R != 1 && R != 2))
    return fail(EG_ERR_ARG, "q4_tc_bytes: need K %% 128 == 0, K <= 12288, R = 1 or 2");
  *bytes = q4_tc_bytes(N, K, R);
  return EG_OK;
}

EG_API eg_status eg_op_q4_stream_to_tc(const void* ws, int N, int K, int R, void* out, void* stream) {
  if (!ws || !out || N <= 0 || K <= 0 || K % 128 || K > 12288 || (R != 1 && R != 2))
    return fail(EG_ERR_ARG, "q4_stream_to_tc: bad argument");
  if ((reinterpret_cast<uintptr_t>(ws) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(EG_ERR_ARG, "q4_stream_to_tc: 16-byte aligned buffers required");
  q4_stream_to_tc(static_cast<const unsigned char*>(ws), N, K, R, static_cast<unsigned char*>(out), OPSTREAM);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_gemm_q4_stream(const float* x, int T, const void* ws, const float* bias, int N,
                                      int K, float* y, int accumulate, int use_tc, void* stream) {
  if (!x || !ws || !y || T < 1 || N <= 0 || K <= 0 || K % 128 || K > 12288)
    return fail(EG_ERR_ARG, "gemm_q4_stream: bad argument");
  if (T > (use_tc ? kPrefillMaxT : kBatchMax))
    return fail(EG_ERR_ARG, "gemm_q4_stream: at most %d tokens per call", use_tc ? kPrefillMaxT : kBatchMax);
  if (accumulate && bias) return fail(EG_ERR_ARG, "gemm_q4_stream: bias with accumulate is not supported");
  if (reinterpret_cast<uintptr_t>(ws) & 15) return fail(EG_ERR_ARG, "gemm_q4_stream: ws must be 16-byte aligned");
  const int gpr = K / 128, tpad = T > 32 ? 32 : (T + 3) / 4 * 4;
  const size_t xb = (size_t)T * gpr * 512, xc = ((size_t)T * gpr * 8 + 255) / 256 * 256,
               xtc = T > 32 && use_tc ? (size_t)(T + 127) / 128 * gpr * 65536 : (size_t)gpr * 4 * tpad * 128;
  const size_t cnt = (size_t)gemv_q4_tc_max_octets() * 4, part = gemv_q4_tc_part_bytes();
  const size_t xfb = ((size_t)T * 4 + 255) / 256 * 256;  // one exponent per token
  // [err | xb | xcor | xf | xtc | counters | partials], every piece 256-byte aligned
  // more than 32 rows: the whole-prompt GEMM over A images built here from ws
  // tcgen05: the int8 A images and row scales (and for more than 32 rows the
  // f16 A images) built here from the tc-layout ws
  const size_t a8 = use_tc ? q4_a8_bytes(N, K, 1) + q4_a16_bytes(N, K, 1) * (T > 32) : 0,
               s8 = use_tc ? q4_row_scale_bytes(N, K, 1) : 0;
  const size_t o_xb = 256, o_xc = o_xb + xb, o_xf = o_xc + xc, o_tc = o_xf + xfb, o_cnt = o_tc + xtc,
               o_part = o_cnt + cnt, o_a8 = o_part + part, o_s8 = o_a8 + a8;
  void* scr = nullptr;
  eg_status s = op_scratch(o_s8 + s8, &scr);
  if (s) return s;
  char* b = static_cast<char*>(scr);
  int* err = reinterpret_cast<int*>(b);
  BatchPlanes xp = {};
  xp.xb = b + o_xb;
  xp.xcor = reinterpret_cast<int*>(b + o_xc);
  xp.xf = reinterpret_cast<int*>(b + o_xf);
  xp.gpr_max = gpr;
  xp.xtc = use_tc && T <= 32 ? b + o_tc : nullptr;
  xp.xh = use_tc && T > 32 ? b + o_tc : nullptr;  // the f16 operand of the whole-prompt GEMM
  xp.tc_tpad = tpad;
  unsigned* counters = reinterpret_cast<unsigned*>(b + o_cnt);
  float* prt = reinterpret_cast<float*>(b + o_part);
  CK(cudaMemsetAsync(err, 0, 4, OPSTREAM));
  if (use_tc) CK(cudaMemsetAsync(counters, 0, cnt, OPSTREAM));
  BatchSrc src = {};
  src.x.mode = X_PLAIN;
  src.x.x = x;
  src.stride = K;
  batch_stage_q4(src, K, T, xp, OPSTREAM, false);
  BatchEpi be = {};
  be.e.mode = accumulate ? EPI_ADD : EPI_STORE;
  be.e.y = y;
  be.e.N = N;
  be.e.bias = bias;
  be.e.split1 = be.e.split2 = N;
  be.ystride = N;
  if (use_tc) {
    const unsigned char* wc = static_cast<const unsigned char*>(ws);
    unsigned char* ia8 = reinterpret_cast<unsigned char*>(b + o_a8);
    unsigned char* ia16 = ia8 + q4_a8_bytes(N, K, 1);
    float* isc = reinterpret_cast<float*>(b + o_s8);
    q4_tc_to_a8(wc, N, K, 1, ia8, isc, OPSTREAM);
    if (T > 32) {
      q4_tc_to_a16(wc, N, K, 1, ia16, OPSTREAM);
      gemm_q4_prefill(ia16, isc, N, K, 1, T, xp, be, err, OPSTREAM);
    } else {
      gemv_q4_tc(ia8, isc, N, K, 1, T, xp, be, prt, counters, err, OPSTREAM, false);
    }
  } else
    gemv_q4_batch(static_cast<const unsigned char*>(ws), N, K, T, xp, be, err, OPSTREAM, false);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_gate_up_silu(const float* x, const uint32_t* w, const float* scale, int N, int K,
                                    float* y, void* stream) {
  if (!x || !w || !scale || !y || N <= 0 || K <= 0 || K % 128 || K > 12288)
    return fail(EG_ERR_ARG, "gate_up_silu: need K %% 128 == 0, K <= 12288");
  if (reinterpret_cast<uintptr_t>(w) & 15) return fail(EG_ERR_ARG, "gate_up_silu: w must be 16-byte aligned");
  XSrc xs = {};
  xs.mode = X_PLAIN;
  xs.x = x;
  Epi e = {};
  e.mode = EPI_SILU;
  e.y = y;
  e.N = N;
  GemvWork wk;
  const unsigned char* ws = nullptr;
  eg_status s = op_gemv_work(N, K, 2, w, scale, &ws, &wk, OPSTREAM);
  if (s) return s;
  gemv_q4(ws, N, K, xs, e, OPSTREAM, false, wk);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_gemv_q8(const float* x, const uint32_t* w, const float* scale, int N, int K, float* y,
                               void* stream) {
  if (!x || !w || !scale || !y || N <= 0 || K <= 0 || K % 64 || K > 12288)
    return fail(EG_ERR_ARG, "gemv_q8: K must be a multiple of 64, <= 12288");
  XSrc xs = {};
  xs.mode = X_PLAIN;
  xs.x = x;
  // the single-op entry takes int8 rows; convert them to the stream layout
  void* scr = nullptr;
  eg_status s = op_scratch(256 + q8_stream_bytes(N, K), &scr);
  if (s) return s;
  char* b = static_cast<char*>(scr);
  CK(cudaMemsetAsync(b, 0, 4, OPSTREAM));
  unsigned char* t = reinterpret_cast<unsigned char*>(b + 256);
  q8_to_stream(w, N, K, t, OPSTREAM);
  gemv_q8(t, scale, N, K, xs, y, nullptr, OPSTREAM, false, GemvWork{reinterpret_cast<int*>(b)});
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_rmsnorm(const float* x, const float* g, int K, float eps, int f16, float* y, void* stream) {
  if (!x || !g || !y || K <= 0) return fail(EG_ERR_ARG, "rmsnorm: bad argument");
  rmsnorm(x, g, K, eps, f16, y, OPSTREAM);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_rope_qk(float* q, float* k, int nq, int nkv, int pos, const float* cos_t,
                               const float* sin_t, int f16, void* stream) {
  if (!q || !k || !cos_t || !sin_t || nq < 0 || nkv < 0 || pos < 0) return fail(EG_ERR_ARG, "rope_qk: bad argument");
  rope_qk(q, k, nq, nkv, pos, cos_t, sin_t, f16, OPSTREAM);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_attn_prefill(float* qkv, int T, void* k_cache, void* v_cache, const float* cos_t,
                                    const float* sin_t, int nh, int nkv, int q_start, int max_ctx, int kv_f16,
                                    float* out, void* stream) {
  if (!qkv || !k_cache || !v_cache || !cos_t || !sin_t || !out) return fail(EG_ERR_ARG, "attn_prefill: null argument");
  if (nh <= 0 || nh > 64 || nkv <= 0 || nh % nkv || T < 1 || q_start < 0 || q_start + T > max_ctx)
    return fail(EG_ERR_ARG, "attn_prefill: bad heads or rows");
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(k_cache) |
       reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(EG_ERR_ARG, "attn_prefill: 16-byte aligned buffers required");
  const int stride = (nh + 2 * nkv) * 128;
  prefill_rope_append(qkv, T, stride, nh, nkv, q_start, cos_t, sin_t, kv_f16, k_cache, v_cache, OPSTREAM);
  PrefillAttn a = {};
  a.qkv = qkv;
  a.qkv_stride = stride;
  a.kc = k_cache;
  a.vc = v_cache;
  a.nh = nh;
  a.nkv = nkv;
  a.kv_f16 = kv_f16;
  a.T = T;
  a.q_start = q_start;
  a.ctx = q_start + T;
  a.out = out;
  a.out_stride = nh * 128;
  attn_prefill(a, OPSTREAM);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_attn_decode(const float* qkv, void* k_cache, void* v_cache, const float* cos_t,
                                   const float* sin_t, int nh, int nkv, int pos, int max_ctx, int kv_f16,
                                   int chunk, float* out, void* stream) {
  if (!qkv || !k_cache || !v_cache || !cos_t || !sin_t || !out) return fail(EG_ERR_ARG, "attn_decode: null argument");
  if (nh <= 0 || nh > 64 || nkv <= 0 || nh % nkv || nh / nkv > 8 || pos < 0 || pos >= max_ctx)
    return fail(EG_ERR_ARG, "attn_decode: bad heads/pos");
  if (chunk < 0 || chunk > 128 || chunk % 16)
    return fail(EG_ERR_ARG, "attn_decode: chunk must be 0 or a multiple of 16 up to 128");
  const int ms = attn_max_splits(max_ctx);
  void* scr = nullptr;
  const size_t part = (size_t)nh * ms * (128 + 2) * 4;
  eg_status s = op_scratch(part + 64 * 4, &scr);
  if (s) return s;
  unsigned* counters = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(scr) + part);
  CK(cudaMemsetAsync(counters, 0, nh * 4, OPSTREAM));
  AttnArgs a = {};
  a.qkv = qkv;
  a.kc = k_cache;
  a.vc = v_cache;
  a.cosT = cos_t;
  a.sinT = sin_t;
  a.pos = nullptr;
  a.fixed_pos = pos;
  a.nh = nh;
  a.nkv = nkv;
  a.max_splits = ms;
  a.ctx_bound = pos + 1;
  a.kv_f16 = kv_f16;
  a.chunk = chunk;
  a.pm = reinterpret_cast<float*>(scr);
  a.pz = a.pm + (size_t)nh * ms;
  a.po = a.pz + (size_t)nh * ms;
  a.out = out;
  a.counters = counters;
  attn_decode(a, OPSTREAM, false, attn_long(a, pos));
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_embed(const uint32_t* w, const float* scale, const uint32_t* id, int H, float* out,
                             void* stream) {
  if (!w || !scale || !id || !out || H <= 0 || H % 4) return fail(EG_ERR_ARG, "embed: bad argument");
  embed_rows(w, scale, id, H, out, OPSTREAM);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_lora_a(const float* x, const float* A, int K, int rank, float* d, void* stream) {
  if (!x || !A || !d || K <= 0 || rank <= 0 || rank > kMaxRank) return fail(EG_ERR_ARG, "lora_a: bad argument");
  void* scr = nullptr;
  eg_status s = op_scratch(sizeof(LoraMod) + kMaxRank * 4, &scr);
  if (s) return s;
  LoraMod m{A, nullptr, rank, 1.f};
  CK(cudaMemcpyAsync(scr, &m, sizeof m, cudaMemcpyHostToDevice, OPSTREAM));
  float* dd = reinterpret_cast<float*>(reinterpret_cast<char*>(scr) + 256);
  XSrc xs = {};
  xs.mode = X_PLAIN;
  xs.x = x;
  lora_a(xs, K, reinterpret_cast<const LoraMod*>(scr), 1, rank, dd, OPSTREAM, false);
  CK(cudaMemcpyAsync(d, dd, (size_t)rank * 4, cudaMemcpyDeviceToDevice, OPSTREAM));
  CK(cudaStreamSynchronize(OPSTREAM));
  return EG_OK;
}

EG_API eg_status eg_op_argmax(const float* logits, int n, uint32_t* out, void* stream) {
  if (!logits || !out || n <= 0) return fail(EG_ERR_ARG, "argmax: bad argument");
  void* scr = nullptr;
  eg_status s = op_scratch((size_t)kCandMax * 8, &scr);
  if (s) return s;
  argmax(logits, n, out, reinterpret_cast<float*>(scr),
         reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(scr) + kCandMax * 4), OPSTREAM);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_topk(const float* logits, int n, int k, uint32_t* ids, float* vals, void* stream) {
  if (!logits || !ids || !vals || n <= 0 || k < 1 || k > 64) return fail(EG_ERR_ARG, "topk: need 1 <= k <= 64");
  if (n > 148 * 2048) return fail(EG_ERR_ARG, "topk: n too large");
  void* scr = nullptr;
  const size_t nc = (size_t)kCandMax * 64;
  eg_status s = op_scratch(nc * 8, &scr);
  if (s) return s;
  topk(logits, n, k, ids, vals, reinterpret_cast<float*>(scr),
       reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(scr) + nc * 4), OPSTREAM);
  CK(cudaGetLastError());
  return EG_OK;
}

EG_API eg_status eg_op_sample_topk(const uint32_t* ids, const float* vals, int k, float temp, float r,
                                   uint32_t* out, void* stream) {
  if (!ids || !vals || !out || k < 0 || k > 64) return fail(EG_ERR_ARG, "sample_topk: need 0 <= k <= 64");
  sample_topk(ids, vals, k, temp, r, out, nullptr, OPSTREAM);
  CK(cudaGetLastError());
  return EG_OK;
}

}  // extern "C"
