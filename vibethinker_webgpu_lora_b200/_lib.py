"""ctypes binding of libemberglass_cuda.so (include/emberglass.h).

The shared library is the product: there is no CPU fallback.  Importing this
module does not need a GPU; calling into the runtime does, and every status
other than EG_OK raises EmberglassError with the library's message.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libemberglass_cuda.so")

EG_OK, EG_ERR_ARG, EG_ERR_CUDA, EG_ERR_STATE, EG_ERR_OOM, EG_ERR_BUSY, EG_ERR_DEVICE = range(7)


class EmberglassError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


class EgConfig(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_int), ("num_layers", C.c_int), ("num_heads", C.c_int),
        ("num_kv_heads", C.c_int), ("head_dim", C.c_int), ("intermediate_size", C.c_int),
        ("vocab_size", C.c_int), ("rms_norm_eps", C.c_float), ("rope_theta", C.c_double),
        ("tie_word_embeddings", C.c_int), ("attention_bias", C.c_int),
    ]


class EgOptions(C.Structure):
    _fields_ = [
        ("device", C.c_int), ("max_ctx", C.c_int), ("max_prefill_t", C.c_int), ("kv_f16", C.c_int),
        ("decode_batch_capacity", C.c_int), ("sampling_top_k", C.c_int),
        ("max_sampling_top_k", C.c_int), ("attn_chunk", C.c_int), ("use_graphs", C.c_int),
        ("use_pdl", C.c_int), ("use_fused", C.c_int), ("prefill_chunk", C.c_int),
        ("use_tc_batch", C.c_int), ("prefill_tc", C.c_int), ("prefill_chunk_size", C.c_int),
        ("use_l2_prefetch", C.c_int),
    ]


class EgLoraModule(C.Structure):
    _fields_ = [
        ("key", C.c_char_p), ("A", C.c_void_p), ("a_rows", C.c_int64), ("a_cols", C.c_int64),
        ("B", C.c_void_p), ("b_rows", C.c_int64), ("b_cols", C.c_int64), ("scale", C.c_float),
    ]


vp, i32, f32, f64, u32, u64, i64 = (C.c_void_p, C.c_int, C.c_float, C.c_double, C.c_uint32,
                                    C.c_uint64, C.c_int64)
_SIGS = {
    "eg_last_error": (C.c_char_p, []),
    "eg_version": (C.c_char_p, []),
    "eg_default_config": (None, [C.POINTER(EgConfig)]),
    "eg_default_options": (None, [C.POINTER(EgOptions)]),
    "eg_create": (i32, [C.POINTER(EgConfig), C.POINTER(EgOptions), C.POINTER(vp)]),
    "eg_destroy": (i32, [vp]),
    "eg_quantize_int4_group": (i32, [vp, i32, i32, i32, vp, vp]),
    "eg_quantize_int8_rows": (i32, [vp, i32, i32, vp, vp]),
    "eg_upload_tensor": (i32, [vp, C.c_char_p, vp, vp, i32]),
    "eg_upload_quantized": (i32, [vp, C.c_char_p, i32, vp, vp, vp, i32]),
    "eg_build_synthetic": (i32, [vp, u64, f64]),
    "eg_finalize": (i32, [vp]),
    "eg_token": (i32, [vp, u32, i32]),
    "eg_decode_greedy": (i32, [vp, i32, i32, vp, C.POINTER(i32)]),
    "eg_prefill": (i32, [vp, vp, i32]),
    "eg_decode_greedy_async": (i32, [vp, i32, i32, C.POINTER(i32)]),
    "eg_read_ids": (i32, [vp, vp, i32]),
    "eg_stream": (vp, [vp]),
    "eg_sync": (i32, [vp]),
    "eg_argmax": (i32, [vp, C.POINTER(u32)]),
    "eg_topk": (i32, [vp, i32, vp, vp, C.POINTER(i32)]),
    "eg_sample": (i32, [vp, f32, f32, C.POINTER(u32)]),
    "eg_read_logits": (i32, [vp, vp]),
    "eg_read_hidden": (i32, [vp, vp]),
    "eg_generate": (i32, [vp, vp, i32, i32, i32, f32, vp, vp]),
    "eg_lora_create": (i32, [vp, i32, vp, C.POINTER(vp)]),
    "eg_lora_orient": (i32, [vp, i64, i64, vp, i64, i64, i64, i64, vp, vp, C.POINTER(i32)]),
    "eg_lora_destroy": (i32, [vp, vp]),
    "eg_lora_update": (i32, [vp, vp, C.c_char_p, vp, vp]),
    "eg_set_lora": (i32, [vp, vp]),
    "eg_clear_lora": (i32, [vp]),
    "eg_invalidate_lora": (i32, [vp]),
    "eg_profile_token": (i32, [vp, u32, i32, vp, C.POINTER(i32)]),
    "eg_profile_fused": (i32, [vp, i32, vp, i32, C.POINTER(i32)]),
    "eg_memory_footprint": (i32, [vp, C.POINTER(i64), C.POINTER(i64), C.POINTER(i64)]),
    "eg_lm_head_shard": (i32, [vp, vp, i32, i32, vp, vp, vp, vp]),
    "eg_load_safetensors": (i32, [vp, C.c_char_p, C.POINTER(i32)]),
    "eg_safetensors_tensor": (i32, [C.c_char_p, C.c_char_p, vp, i64, vp, C.POINTER(i32)]),
    "eg_seq_init": (i32, [vp, i32, i32]),
    "eg_seq_init_paged": (i32, [vp, i32, i32, i32]),
    "eg_seq_release": (i32, [vp, i32]),
    "eg_seq_prefill": (i32, [vp, i32]),
    "eg_seq_pages": (i32, [vp, C.POINTER(i32), C.POINTER(i32)]),
    "eg_seq_set_prompt": (i32, [vp, i32, vp, i32]),
    "eg_seq_state": (i32, [vp, i32, vp, vp]),
    "eg_batch_decode": (i32, [vp, i32, vp, i32, vp]),
    "eg_batch_sample": (i32, [vp, i32, vp, i32, i32, f32, vp, vp]),
    "eg_batch_read_logits": (i32, [vp, i32, vp]),
    "eg_launches_per_step": (i32, [vp]),
    "eg_op_gemv_q4": (i32, [vp, vp, vp, vp, i32, i32, i32, vp, i32, vp]),
    "eg_op_q4_stream_bytes": (i32, [i32, i32, i32, C.POINTER(u64)]),
    "eg_op_q4_to_stream": (i32, [vp, vp, i32, i32, i32, vp, vp]),
    "eg_op_gemv_q4_stream": (i32, [vp, vp, vp, i32, i32, vp, vp, i32, vp]),
    "eg_op_gemm_q4_stream": (i32, [vp, i32, vp, vp, i32, i32, vp, i32, i32, vp]),
    "eg_op_q4_tc_bytes": (i32, [i32, i32, i32, C.POINTER(u64)]),
    "eg_op_q4_stream_to_tc": (i32, [vp, i32, i32, i32, vp, vp]),
    "eg_op_gate_up_silu": (i32, [vp, vp, vp, i32, i32, vp, vp]),
    "eg_op_gemv_q8": (i32, [vp, vp, vp, i32, i32, vp, vp]),
    "eg_op_rmsnorm": (i32, [vp, vp, i32, f32, i32, vp, vp]),
    "eg_op_rope_qk": (i32, [vp, vp, i32, i32, i32, vp, vp, i32, vp]),
    "eg_op_attn_decode": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp]),
    "eg_op_attn_prefill": (i32, [vp, i32, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, vp]),
    "eg_op_attn_decode_noalloc": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp]),
    "eg_op_embed": (i32, [vp, vp, vp, i32, vp, vp]),
    "eg_op_lora_a": (i32, [vp, vp, i32, i32, vp, vp]),
    "eg_op_argmax": (i32, [vp, i32, vp, vp]),
    "eg_op_topk": (i32, [vp, i32, i32, vp, vp, vp]),
    "eg_op_sample_topk": (i32, [vp, vp, i32, f32, f32, vp, vp]),
    "eg_synth_normal": (None, [vp, i64, u64, f64, i64]),
    "eg_synth_stream_at": (u64, [u64, u64]),
}

_lib = None


def lib():
    """Load the CUDA library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run __graft_entry__.build() "
                              "(python vibethinker_webgpu_lora_b200/build.py)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def declared_symbols() -> list[str]:
    return list(_SIGS)


def check(status: int):
    if status != EG_OK:
        msg = lib().eg_last_error().decode(errors="replace")
        raise EmberglassError(status, msg)


def ptr(a) -> int | None:
    """Address of a numpy array or torch tensor (None passes NULL)."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def stream_ptr(stream) -> int | None:
    if stream is None:
        return None
    return getattr(stream, "cuda_stream", stream)
