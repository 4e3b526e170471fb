// eg_noalloc.cu -- decode attention for callers that must not allocate.
//
// eg_op_attn_decode keeps its split-K partials in library scratch that it
// grows with cudaMalloc on first use (and cudaFree + cudaMalloc when a larger
// call arrives).  Some callers cannot allow that at call time: a host
// framework whose caching allocator has reserved the device memory up front
// (a fresh cudaMalloc can fail, or force that allocator to release cached
// blocks), and latency-critical serving loops where cudaMalloc/cudaFree's
// implicit device-wide synchronisation is not acceptable.  This file gives
// them the same kernel with its scratch in a fixed, file-scope device array
// that is loaded with the library, so the entry point itself allocates
// nothing.
#include <mutex>

#include "eg_host.h"
#include "eg_kernels.h"
#include "emberglass.h"

namespace {

// Scratch capacity: 4096 (head, split) slots of 130 floats (split max, split
// sum, 128-wide partial output) plus 64 per-head arrival counters:
// 2,130,176 bytes, held by every GPU that loads the library until exit.
constexpr int kSlots = 4096;
constexpr size_t kPartialBytes = (size_t)kSlots * (128 + 2) * sizeof(float);
constexpr size_t kScratchBytes = kPartialBytes + 64 * sizeof(unsigned);

static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

// In host code g_attn_scratch names a host-side stand-in, not device memory.
// Its device address is looked up once per device, with that device current,
// and cached here.
std::mutex g_mu;
void* g_scratch_ptr[64] = {};

eg_status scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return eg::fail(EG_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return eg::fail(EG_ERR_ARG, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p)
      return eg::fail(EG_ERR_CUDA, "cudaGetSymbolAddress(attention scratch): %s",
                      cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return EG_OK;
}

}  // namespace

extern "C" {

// Same inputs, outputs and results as eg_op_attn_decode; scratch comes from
// the static array above.  Limits: nh * ceil((pos+1) / keys) must not exceed
// 4096, where keys = chunk, or 128 (the fixed default chunk) when chunk = 0;
// nh <= 64.
// Every call shares the one array: calls that overlap on the GPU (concurrent
// streams, or several host threads on one device) race on it.  The first
// call on a device resolves the array's device address; make that first call
// before any stream capture.
EG_API eg_status eg_op_attn_decode_noalloc(const float* qkv, void* k_cache, void* v_cache,
                                           const float* cos_t, const float* sin_t, int nh,
                                           int nkv, int pos, int max_ctx, int kv_f16, int chunk,
                                           float* out, void* stream) {
  if (!qkv || !k_cache || !v_cache || !cos_t || !sin_t || !out)
    return eg::fail(EG_ERR_ARG, "attn_decode_noalloc: null argument");
  if (nh <= 0 || nh > 64 || nkv <= 0 || nh % nkv || nh / nkv > 8 || pos < 0 || pos >= max_ctx)
    return eg::fail(EG_ERR_ARG, "attn_decode_noalloc: bad heads/pos");
  if (chunk < 0 || chunk > eg::kAttnDefaultChunk || chunk % 16)
    return eg::fail(EG_ERR_ARG, "attn_decode_noalloc: chunk must be 0 or a multiple of 16 up to 128");
  const int ctx = pos + 1;
  const int keys = chunk > 0 ? chunk : eg::kAttnDefaultChunk;
  const int splits = (ctx + keys - 1) / keys;
  if ((long long)nh * splits > kSlots)
    return eg::fail(EG_ERR_ARG,
                    "attn_decode_noalloc: %d heads x %d splits (pos %d, chunk %d) exceed the "
                    "%d-slot static scratch; pass a larger chunk or use eg_op_attn_decode",
                    nh, splits, pos, chunk, kSlots);
  void* base = nullptr;
  eg_status s = scratch_for_current_device(&base);
  if (s) return s;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float* f = reinterpret_cast<float*>(base);
  unsigned* counters = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(base) + kPartialBytes);
  // the arrival counters must start at zero; the array keeps the last call's contents
  cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)nh * sizeof(unsigned), st);
  if (e != cudaSuccess) return eg::fail(EG_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  eg::AttnArgs a = {};
  a.qkv = qkv;
  a.kc = k_cache;
  a.vc = v_cache;
  a.cosT = cos_t;
  a.sinT = sin_t;
  a.pos = nullptr;
  a.fixed_pos = pos;
  a.nh = nh;
  a.nkv = nkv;
  a.max_splits = splits;
  a.ctx_bound = ctx;
  a.kv_f16 = kv_f16;
  a.chunk = chunk;
  a.pm = f;
  a.pz = f + (size_t)nh * splits;
  a.po = f + 2 * (size_t)nh * splits;
  a.out = out;
  a.counters = counters;
  eg::attn_decode(a, st, false, eg::attn_long(a, pos));
  e = cudaGetLastError();
  if (e != cudaSuccess) return eg::fail(EG_ERR_CUDA, "attn_decode_noalloc: %s", cudaGetErrorString(e));
  return EG_OK;
}

}  // extern "C"
