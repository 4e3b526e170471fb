"""Single-op entry points (the reference's exported WGSL kernels,
src/qwgpu/kernels.js) on device tensors.  Arguments are torch CUDA tensors
(or anything with data_ptr()); calls are asynchronous on `stream`
(torch.cuda.Stream, raw handle, or None for the current torch stream)."""
from __future__ import annotations

from . import _lib as L


def _st(stream):
    if stream is None:
        try:
            import torch
            return torch.cuda.current_stream().cuda_stream
        except Exception:
            return None
    return L.stream_ptr(stream)


def gemv_q4(x, w, scale, N, K, y, bias=None, accumulate=False, group=128, stream=None):
    L.check(L.lib().eg_op_gemv_q4(L.ptr(x), L.ptr(w), L.ptr(scale), L.ptr(bias), N, K, group,
                                  L.ptr(y), int(accumulate), _st(stream)))


def q4_stream_bytes(N, K, R=1):
    """Bytes of the device stream layout of an int4 matrix (R = 2: [gate;up])."""
    import ctypes as C
    n = C.c_uint64(0)
    L.check(L.lib().eg_op_q4_stream_bytes(N, K, R, C.byref(n)))
    return int(n.value)


def q4_to_stream(w, scale, N, K, out, R=1, stream=None):
    """Write the stream layout of a reference-layout int4 matrix into `out`
    (a uint8 device buffer of q4_stream_bytes(N, K, R) bytes), once."""
    L.check(L.lib().eg_op_q4_to_stream(L.ptr(w), L.ptr(scale), N, K, R, L.ptr(out), _st(stream)))


def gemv_q4_stream(x, ws, N, K, y, err, bias=None, pdl=False, stream=None):
    """GEMV4 over a matrix already in the stream layout: no conversion, no
    allocation.  err: int32 device word, zero before the call."""
    L.check(L.lib().eg_op_gemv_q4_stream(L.ptr(x), L.ptr(ws), L.ptr(bias), N, K, L.ptr(y), L.ptr(err),
                                         int(pdl), _st(stream)))


def q4_tc_bytes(N, K, R=1):
    """Bytes of the tensor-core (octet-major) layout of an int4 matrix."""
    import ctypes as C
    n = C.c_uint64(0)
    L.check(L.lib().eg_op_q4_tc_bytes(N, K, R, C.byref(n)))
    return int(n.value)


def q4_stream_to_tc(ws, N, K, out, R=1, stream=None):
    """Regroup a stream-layout matrix into the tensor-core layout, once."""
    L.check(L.lib().eg_op_q4_stream_to_tc(L.ptr(ws), N, K, R, L.ptr(out), _st(stream)))


def gemm_q4_stream(x, T, ws, N, K, y, bias=None, accumulate=False, use_tc=True, stream=None):
    """GEMM4 / GEMM4_ADD_T over a stream-layout matrix: y[t] (+)= W x[t]."""
    L.check(L.lib().eg_op_gemm_q4_stream(L.ptr(x), T, L.ptr(ws), L.ptr(bias), N, K, L.ptr(y),
                                         int(accumulate), int(use_tc), _st(stream)))


def gate_up_silu(x, w, scale, N, K, y, stream=None):
    L.check(L.lib().eg_op_gate_up_silu(L.ptr(x), L.ptr(w), L.ptr(scale), N, K, L.ptr(y), _st(stream)))


def gemv_q8(x, w, scale, N, K, y, stream=None):
    L.check(L.lib().eg_op_gemv_q8(L.ptr(x), L.ptr(w), L.ptr(scale), N, K, L.ptr(y), _st(stream)))


def rmsnorm(x, g, K, eps, f16, y, stream=None):
    L.check(L.lib().eg_op_rmsnorm(L.ptr(x), L.ptr(g), K, eps, int(f16), L.ptr(y), _st(stream)))


def rope_qk(q, k, nq, nkv, pos, cos_t, sin_t, f16, stream=None):
    L.check(L.lib().eg_op_rope_qk(L.ptr(q), L.ptr(k), nq, nkv, pos, L.ptr(cos_t), L.ptr(sin_t),
                                  int(f16), _st(stream)))


def attn_prefill(qkv, T, k_cache, v_cache, cos_t, sin_t, nh, nkv, q_start, max_ctx, kv_f16, out, stream=None):
    """ROPE_T + K/V rows + ATTN_PREFILL_BLOCK of one prefill pass (qkv rotated in place)."""
    L.check(L.lib().eg_op_attn_prefill(L.ptr(qkv), T, L.ptr(k_cache), L.ptr(v_cache), L.ptr(cos_t),
                                       L.ptr(sin_t), nh, nkv, q_start, max_ctx, int(kv_f16), L.ptr(out),
                                       _st(stream)))


def attn_decode(qkv, k_cache, v_cache, cos_t, sin_t, nh, nkv, pos, max_ctx, kv_f16, out, chunk=0,
                stream=None):
    L.check(L.lib().eg_op_attn_decode(L.ptr(qkv), L.ptr(k_cache), L.ptr(v_cache), L.ptr(cos_t),
                                      L.ptr(sin_t), nh, nkv, pos, max_ctx, int(kv_f16), chunk,
                                      L.ptr(out), _st(stream)))


def embed(w, scale, id_dev, H, out, stream=None):
    L.check(L.lib().eg_op_embed(L.ptr(w), L.ptr(scale), L.ptr(id_dev), H, L.ptr(out), _st(stream)))


def lora_a(x, A, K, rank, d, stream=None):
    L.check(L.lib().eg_op_lora_a(L.ptr(x), L.ptr(A), K, rank, L.ptr(d), _st(stream)))


def argmax(logits, n, out, stream=None):
    L.check(L.lib().eg_op_argmax(L.ptr(logits), n, L.ptr(out), _st(stream)))


def topk(logits, n, k, ids, vals, stream=None):
    L.check(L.lib().eg_op_topk(L.ptr(logits), n, k, L.ptr(ids), L.ptr(vals), _st(stream)))


def sample_topk(ids, vals, k, temp, r, out, stream=None):
    L.check(L.lib().eg_op_sample_topk(L.ptr(ids), L.ptr(vals), k, temp, r, L.ptr(out), _st(stream)))
