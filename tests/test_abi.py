"""The C-ABI library loads and exports every entry point include/emberglass.h
declares; host-side functions (quantisers, generator, argument checks) run
without a GPU."""
import ctypes as C
import json
import os
import re
import struct
import subprocess

import numpy as np
import pytest

import vibethinker_webgpu_lora_b200 as E
from vibethinker_webgpu_lora_b200 import _lib as L
from vibethinker_webgpu_lora_b200.lora import moduleKeyFromTensorName, _read_safetensors
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "emberglass.h")


def header_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"EG_API\s+[\w\s\*]+?\b(eg_\w+)\s*\(", txt)))


def test_exports_every_declared_symbol():
    syms = header_symbols()
    assert len(syms) >= 40
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (eg_\w+)", out))
    missing = [s for s in syms if s not in exported]
    assert not missing, missing
    lib = L.lib()
    for s in syms:
        assert hasattr(lib, s)
    # every header symbol has a ctypes signature in the binding
    assert set(syms) <= set(L.declared_symbols())


def test_quantizers_bit_exact_vs_oracle():
    W = O.normal(300 * 512, 0xE6B00001, 0.02).reshape(300, 512)
    W[3, :128] = 0.0  # all-zero group -> scale 1
    p, s, gpr = E.quantizeInt4Group(W)
    p2, s2 = O.quantize_int4_group(W)
    assert gpr == 4 and np.array_equal(p, p2) and np.array_equal(s, s2)
    assert s[3 * 4] == 1.0
    q, qs = E.quantizeInt8RowMajor(W)
    q2, qs2 = O.quantize_int8_rows(W)
    assert np.array_equal(q, q2) and np.array_equal(qs, qs2)


def test_quantizer_rejects_bad_shapes():
    with pytest.raises(E.EmberglassError, match="group"):
        E.quantizeInt4Group(np.zeros((2, 100), np.float32))
    with pytest.raises(E.EmberglassError, match="K % 4"):
        E.quantizeInt8RowMajor(np.zeros((2, 6), np.float32))


def test_generator_matches_oracle():
    from vibethinker_webgpu_lora_b200.quantize import synth_normal
    for seed, start in [(1, 0), (0xE6B00000, 12345), (2**63 + 5, 7)]:
        assert np.array_equal(synth_normal(4096, seed, 0.02, start), O.normal(4096, seed, 0.02, start))
    lib = L.lib()
    for k in (0, 1, 99):
        assert lib.eg_synth_stream_at(42, k) == O.stream_at(42, k)


def test_create_without_gpu_or_bad_config_fails_cleanly():
    cfg = dict(E.QWEN25_3B)
    cfg["headDim"] = 64
    with pytest.raises(E.EmberglassError, match="head_dim"):
        E.QwenB200(cfg)
    cfg = dict(E.QWEN25_3B)
    cfg["tieWordEmbeddings"] = False
    with pytest.raises(E.EmberglassError, match="tied"):
        E.QwenB200(cfg)


def test_ops_reject_bad_arguments():
    lib = L.lib()
    assert lib.eg_op_gemv_q4(None, None, None, None, 1, 128, 128, None, 0, None) == L.EG_ERR_ARG
    assert b"gemv_q4" in lib.eg_last_error()
    assert lib.eg_op_topk(1, 10, 65, 1, 1, None) == L.EG_ERR_ARG
    assert lib.eg_token(None, 0, 0) == L.EG_ERR_ARG


def test_module_keys():
    assert moduleKeyFromTensorName(
        "base_model.model.model.layers.3.self_attn.q_proj.lora_A.weight") == "layers.3.self_attn.q_proj"
    assert moduleKeyFromTensorName("model.layers.10.mlp.down_proj.lora_b") == "layers.10.mlp.down_proj"
    assert moduleKeyFromTensorName("model.layers.1.mlp.gate.lora_a") == "layers.1.mlp.gate_proj"
    assert moduleKeyFromTensorName("model.embed_tokens.weight") is None


def test_safetensors_reader(tmp_path):
    a = np.arange(6, dtype=np.float32).reshape(2, 3)
    b16 = (np.arange(4, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    hdr = {"x.lora_A.weight": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 24]},
           "x.lora_B.weight": {"dtype": "BF16", "shape": [4], "data_offsets": [24, 32]}}
    h = json.dumps(hdr).encode()
    p = tmp_path / "a.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + a.tobytes() + b16.tobytes())
    t = _read_safetensors(str(p))
    assert np.array_equal(t["x.lora_A.weight"], a)
    assert np.array_equal(t["x.lora_B.weight"], np.arange(4, dtype=np.float32))


def test_default_options_match_the_header_and_python_struct():
    """eg_default_options fills every field of the Python mirror of
    eg_options (the struct sizes agree: the last field is written), with the
    defaults the header documents."""
    o = L.EgOptions()
    for name, _ in L.EgOptions._fields_:
        setattr(o, name, -7)
    L.lib().eg_default_options(C.byref(o))
    got = {name: getattr(o, name) for name, _ in L.EgOptions._fields_}
    assert -7 not in got.values()
    assert got["max_ctx"] == 8192 and got["kv_f16"] == 1 and got["use_graphs"] == 1
    assert got["use_pdl"] == 1 and got["use_fused"] == 0 and got["prefill_chunk"] == 16
    assert got["use_tc_batch"] == 0
    assert got["prefill_tc"] == 1 and got["prefill_chunk_size"] == 0 and got["use_l2_prefetch"] == 1
    hdr = open(HEADER).read()
    fields = hdr[:hdr.index("} eg_options;")].rsplit("typedef struct {", 1)[1]
    names = re.findall(r"\bint\s+(\w+);", fields)
    assert names == [n for n, _ in L.EgOptions._fields_]
