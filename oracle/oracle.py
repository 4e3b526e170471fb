"""ctypes binding for the CPU oracle (test infrastructure only).

The oracle restates the Emberglass reference decode path in C (oracle.c).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may use
this module; the product library never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def build() -> str:
    """Compile oracle.c into _build/liboracle.so (make; no-op when fresh)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        _lib = C.CDLL(_SO)
        _declare(_lib)
    return _lib


f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")


class OrcCfg(C.Structure):
    _fields_ = [
        ("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
        ("head_dim", C.c_int), ("inter", C.c_int), ("vocab", C.c_int), ("eps", C.c_float),
        ("theta", C.c_double),
    ]


def _declare(L):
    vp, i, f, d, u64, i64, u32 = C.c_void_p, C.c_int, C.c_float, C.c_double, C.c_uint64, C.c_int64, C.c_uint32
    sig = {
        "orc_stream_at": (u64, [u64, u64]),
        "orc_fill_normal": (None, [f32p, i64, u64, d, i64]),
        "orc_fill_uniform": (None, [f32p, i64, u64]),
        "orc_fill_ids": (None, [u32p, i64, u64, u32]),
        "orc_quantize_int4_group": (i, [f32p, i, i, i, u32p, f32p]),
        "orc_quantize_int8_rows": (i, [f32p, i, i, u32p, f32p]),
        "orc_dequant_int4": (None, [u32p, f32p, i, i, i, f32p]),
        "orc_gemv_q4": (None, [f32p, u32p, f32p, vp, vp, vp, i, f, i, i, i, i, f32p]),
        "orc_gemv_q8": (None, [f32p, u32p, f32p, vp, i, i, f32p]),
        "orc_gate_up_silu": (None, [f32p, u32p, f32p, vp, vp, i, f, vp, vp, i, f, i, i, i, f32p]),
        "orc_lora_a": (None, [f32p, f32p, i, i, f32p]),
        "orc_rmsnorm": (None, [f32p, f32p, i, f, i, f32p]),
        "orc_rope_tables": (None, [i, i, d, f32p, f32p]),
        "orc_rope_qk": (None, [f32p, f32p, i, i, i, i, f32p, f32p, i]),
        "orc_embed": (None, [u32p, f32p, u32, i, f32p]),
        "orc_attention": (None, [f32p, f32p, f32p, i, i, i, i, i, i, f32p]),
        "orc_gemm4": (None, [f32p, i, u32p, f32p, vp, i, i, i, f32p]),
        "orc_lora_batch_delta": (None, [f32p, i, f32p, f32p, i, f, i, i, f32p]),
        "orc_silu_mul": (None, [f32p, f32p, i64, i]),
        "orc_rope_t": (None, [f32p, i, i, i, i, f32p, f32p, i]),
        "orc_attn_prefill": (None, [f32p, f32p, f32p, i, i, i, i, i, i, f32p]),
        "orc_model_prefill": (i, [vp, u32p, i, i, vp]),
        "orc_argmax": (u32, [f32p, i]),
        "orc_topk": (None, [f32p, i, i, u32p, f32p]),
        "orc_sample_topk": (u32, [u32p, f32p, i, f, f]),
        "orc_tensor_seed": (u64, [u64, i]),
        "orc_model_create": (vp, [C.POINTER(OrcCfg), i, i, u64, d]),
        "orc_model_set_chunk": (None, [vp, i]),
        "orc_set_sum_order": (None, [i]),
        "orc_model_tensor": (vp, [vp, i, i]),
        "orc_model_lora_synth": (None, [vp, u64, i, f, d, d]),
        "orc_model_lora_clear": (None, [vp]),
        "orc_model_step": (i, [vp, u32, i, vp]),
        "orc_model_hidden": (vp, [vp]),
        "orc_model_logits": (vp, [vp]),
        "orc_model_generate": (i, [vp, u32p, i, i, u32p, vp]),
        "orc_model_free": (None, [vp]),
        "orc_num_threads": (i, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- inputs
def normal(n: int, seed: int, std: float = 1.0, start: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_fill_normal(out, n, seed, std, start)
    return out


def uniform(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_fill_uniform(out, n, seed)
    return out


def token_ids(n: int, seed: int, vocab: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().orc_fill_ids(out, n, seed, vocab)
    return out


def stream_at(seed: int, k: int) -> int:
    return lib().orc_stream_at(seed, k)


# ---------------------------------------------------------------- quantisers
def quantize_int4_group(W: np.ndarray, group: int = 128):
    W = np.ascontiguousarray(W, np.float32)
    N, K = W.shape
    packed = np.empty(N * K // 8, np.uint32)
    scale = np.empty(N * (K // group), np.float32)
    if lib().orc_quantize_int4_group(W, N, K, group, packed, scale) != 0:
        raise ValueError("bad int4 quantiser shape")
    return packed, scale


def quantize_int8_rows(W: np.ndarray):
    W = np.ascontiguousarray(W, np.float32)
    N, K = W.shape
    packed = np.empty(N * K // 4, np.uint32)
    scale = np.empty(N, np.float32)
    if lib().orc_quantize_int8_rows(W, N, K, packed, scale) != 0:
        raise ValueError("bad int8 quantiser shape")
    return packed, scale


def dequant_int4(packed, scale, N, K, group=128):
    out = np.empty(N * K, np.float32)
    lib().orc_dequant_int4(packed, scale, N, K, group, out)
    return out.reshape(N, K)


# ---------------------------------------------------------------- ops
def gemv_q4(x, packed, scale, N, K, bias=None, lora_d=None, lora_b=None, rank=0, lora_scale=0.0,
            y=None, add=False):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(N, np.float32) if y is None else y
    lib().orc_gemv_q4(x, packed, scale, _ptr(bias), _ptr(lora_d), _ptr(lora_b), rank, lora_scale,
                      N, K, K // 128, int(add), out)
    return out


def gemv_q8(x, packed, scale, N, K, bias=None):
    out = np.empty(N, np.float32)
    lib().orc_gemv_q8(np.ascontiguousarray(x, np.float32), packed, scale, _ptr(bias), N, K, out)
    return out


def gate_up_silu(x, packed, scale, N, K, gD=None, gB=None, gRank=0, gScale=0.0, uD=None, uB=None,
                 uRank=0, uScale=0.0):
    out = np.empty(N, np.float32)
    lib().orc_gate_up_silu(np.ascontiguousarray(x, np.float32), packed, scale, _ptr(gD), _ptr(gB),
                           gRank, gScale, _ptr(uD), _ptr(uB), uRank, uScale, N, K, K // 128, out)
    return out


def lora_a(x, A, K, rank):
    d = np.empty(rank, np.float32)
    lib().orc_lora_a(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(A, np.float32), K,
                     rank, d)
    return d


def rmsnorm(x, g, eps=1e-6, f16=False):
    y = np.empty_like(x, dtype=np.float32)
    lib().orc_rmsnorm(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(g, np.float32),
                      x.size, eps, int(f16), y)
    return y


def rope_tables(max_ctx, hd=128, theta=1e6):
    c = np.empty(max_ctx * hd, np.float32)
    s = np.empty(max_ctx * hd, np.float32)
    lib().orc_rope_tables(max_ctx, hd, theta, c, s)
    return c, s


def rope_qk(q, k, nq, nkv, hd, pos, cosT, sinT, f16=False):
    q = np.array(q, np.float32)
    k = np.array(k, np.float32)
    lib().orc_rope_qk(q, k, nq, nkv, hd, pos, cosT, sinT, int(f16))
    return q, k


def embed(w, scale, tok, H):
    out = np.empty(H, np.float32)
    lib().orc_embed(w, scale, tok, H, out)
    return out


def attention(q, kc, vc, nh, nkv, ctx, hd, chunk=128, f16=False):
    out = np.empty(nh * hd, np.float32)
    lib().orc_attention(np.ascontiguousarray(q, np.float32), np.ascontiguousarray(kc, np.float32),
                        np.ascontiguousarray(vc, np.float32), nh, nkv, ctx, hd, chunk, int(f16), out)
    return out


def gemm4(X, packed, scale, N, K, bias=None, Y=None, add=False):
    """GEMM4 / GEMM4_ADD_T over T rows of X (kernels.js:389-473)."""
    X = np.ascontiguousarray(X, np.float32)
    T = X.size // K
    out = np.zeros((T, N), np.float32) if Y is None else Y
    lib().orc_gemm4(X, T, packed, scale, _ptr(bias), N, K, int(add), out)
    return out


def rope_t(x, T, nh, hd, pos0, cosT, sinT, f16=False):
    x = np.array(x, np.float32)
    lib().orc_rope_t(x, T, nh, hd, pos0, cosT, sinT, int(f16))
    return x


def attn_prefill(q, kc, vc, nh, nkv, hd, T, q_start, ctx):
    """ATTN_PREFILL_BLOCK (kernels.js:684-770): rows q_start .. q_start+T-1."""
    out = np.empty(T * nh * hd, np.float32)
    lib().orc_attn_prefill(np.ascontiguousarray(q, np.float32), np.ascontiguousarray(kc, np.float32),
                           np.ascontiguousarray(vc, np.float32), nh, nkv, hd, T, q_start, ctx, out)
    return out


def argmax(logits) -> int:
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_argmax(logits, logits.size))


def topk(logits, k):
    logits = np.ascontiguousarray(logits, np.float32)
    ids = np.zeros(k, np.uint32)
    vals = np.zeros(k, np.float32)
    lib().orc_topk(logits, logits.size, k, ids, vals)
    return ids, vals


def sample_topk(ids, vals, k, temp, r) -> int:
    return int(lib().orc_sample_topk(np.ascontiguousarray(ids, np.uint32),
                                     np.ascontiguousarray(vals, np.float32), k, temp, r))


def threads() -> int:
    return lib().orc_num_threads()


# ---------------------------------------------------------------- model
class OracleModel:
    """Synthetic Qwen2.5-shaped model stepped on the CPU (runtime.js:1466-1571)."""

    def __init__(self, cfg: dict, max_ctx: int, f16: bool, seed: int, std: float = 0.02):
        self.cfg = cfg
        c = OrcCfg(cfg["hiddenSize"], cfg["numLayers"], cfg["numHeads"], cfg["numKVHeads"],
                   cfg["headDim"], cfg["intermediateSize"], cfg["vocabSize"], cfg["rmsNormEps"],
                   cfg["ropeTheta"])
        self._h = lib().orc_model_create(C.byref(c), max_ctx, int(f16), seed, std)
        if not self._h:
            raise MemoryError("oracle model allocation failed")
        self.vocab = cfg["vocabSize"]

    def close(self):
        if self._h:
            lib().orc_model_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def set_chunk(self, chunk: int):
        lib().orc_model_set_chunk(self._h, chunk)

    def lora_synth(self, seed, rank=8, scale=2.0, stdA=0.02, stdB=0.01):
        lib().orc_model_lora_synth(self._h, seed, rank, scale, stdA, stdB)

    def lora_clear(self):
        lib().orc_model_lora_clear(self._h)

    def step(self, tok: int, pos: int) -> np.ndarray:
        out = np.empty(self.vocab, np.float32)
        if lib().orc_model_step(self._h, tok, pos, out.ctypes.data_as(C.c_void_p)) != 0:
            raise ValueError("oracle step: bad token or position")
        return out

    def prefill(self, ids, chunk: int = 0) -> np.ndarray:
        """prefillBatch(ids) (runtime.js:1936-2087); returns the last row's logits."""
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.empty(self.vocab, np.float32)
        if lib().orc_model_prefill(self._h, ids, ids.size, chunk, out.ctypes.data_as(C.c_void_p)) != 0:
            raise ValueError("oracle prefill: bad token or length")
        return out

    def logits(self) -> np.ndarray:
        p = lib().orc_model_logits(self._h)
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), (self.vocab,)).copy()

    def hidden(self) -> np.ndarray:
        p = lib().orc_model_hidden(self._h)
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), (self.cfg["hiddenSize"],)).copy()

    def generate(self, prompt, n_gen: int, prefill: bool = False, chunk: int = 0):
        """Greedy continuation (decodeBatch, runtime.js:1776-1793); the prompt
        through the token loop, or with prefill=True through prefillBatch."""
        prompt = np.ascontiguousarray(prompt, np.uint32)
        if prefill:
            logits = self.prefill(prompt, chunk)
            ids = np.zeros(n_gen, np.uint32)
            margins = np.zeros(n_gen, np.float32)
            for g in range(n_gen):
                top2 = np.partition(logits, -2)[-2:]
                ids[g] = argmax(logits)
                margins[g] = top2[1] - top2[0]
                if g + 1 < n_gen:
                    logits = self.step(int(ids[g]), prompt.size + g)
            return ids, margins
        ids = np.zeros(n_gen, np.uint32)
        margins = np.zeros(n_gen, np.float32)
        rc = lib().orc_model_generate(self._h, prompt, prompt.size, n_gen, ids,
                                      margins.ctypes.data_as(C.c_void_p))
        if rc != 0:
            raise ValueError("oracle generate: context overflow")
        return ids, margins

    def tensor(self, layer: int, which: int, count: int, dtype):
        p = lib().orc_model_tensor(self._h, layer, which)
        ct = C.c_uint32 if dtype == np.uint32 else C.c_float
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(ct)), (count,)).copy()
