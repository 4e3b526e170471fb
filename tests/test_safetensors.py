"""Streaming safetensors loader (eg_load_safetensors / eg_safetensors_tensor),
following src/qwgpu/safetensors_loader.js:20-126: index-json sharding,
header parsing, BF16 / F16 / F32 decoding to f32 (bit-exact: BF16 is the
upper half of an f32, F16 converts exactly), unsupported dtypes and broken
files raise.  CPU tests use the host-only decode entry; the GPU test builds a
model from a sharded directory and compares it with direct uploads."""
import json
import struct

import numpy as np
import pytest

import vibethinker_webgpu_lora_b200 as E

def bf16_bits(a):
    """Truncate f32 to bf16 (the upper 16 bits)."""
    return (np.ascontiguousarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def write_st(path, tensors, metadata=None):
    """tensors: name -> (dtype, array already in that dtype's storage)."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, (dt, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def test_decode_bf16_f16_f32(tmp_path):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((7, 33)).astype(np.float32) * 3
    h = np.array([0.0, -0.0, 1.0, -2.5, 65504.0, 6e-8, -5.96e-8, 1e-5, np.inf, -np.inf, np.nan],
                 np.float16)
    p = str(tmp_path / "m.safetensors")
    write_st(p, {"a.bf16": ("BF16", bf16_bits(x)), "b.f16": ("F16", h), "c.f32": ("F32", x)},
             metadata={"format": "pt"})
    got = E.readSafetensorsTensor(p, "a.bf16")
    want = (bf16_bits(x).astype(np.uint32) << 16).view(np.float32)
    assert got.shape == (7, 33) and np.array_equal(got.view(np.uint32), want.view(np.uint32))
    got = E.readSafetensorsTensor(p, "b.f16")
    want = h.astype(np.float32)
    assert np.array_equal(got[~np.isnan(want)].view(np.uint32), want[~np.isnan(want)].view(np.uint32))
    assert np.isnan(got[-1])
    assert np.array_equal(E.readSafetensorsTensor(p, "c.f32"), x)


def test_all_f16_values_exact(tmp_path):
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    p = str(tmp_path / "h.safetensors")
    write_st(p, {"h": ("F16", allh)})
    got = E.readSafetensorsTensor(p, "h")
    want = allh.astype(np.float32)
    ok = ~np.isnan(want)
    assert np.array_equal(got[ok].view(np.uint32), want[ok].view(np.uint32))
    assert np.isnan(got[~ok]).all()


def test_sharded_directory_and_escaped_names(tmp_path):
    rng = np.random.default_rng(2)
    a = rng.standard_normal((4, 8)).astype(np.float32)
    b = rng.standard_normal((16,)).astype(np.float32)
    write_st(str(tmp_path / "s1.safetensors"), {"w.é\"q": ("F32", a)})
    write_st(str(tmp_path / "s2.safetensors"), {"v": ("F32", b)})
    with open(tmp_path / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {"total_size": 0},
                   "weight_map": {"w.é\"q": "s1.safetensors", "v": "s2.safetensors"}}, f)
    assert np.array_equal(E.readSafetensorsTensor(str(tmp_path), "w.é\"q"), a)
    assert np.array_equal(E.readSafetensorsTensor(str(tmp_path), "v"), b)
    # a directory without an index falls back to model.safetensors
    d2 = tmp_path / "single"
    d2.mkdir()
    write_st(str(d2 / "model.safetensors"), {"v": ("F32", b)})
    assert np.array_equal(E.readSafetensorsTensor(str(d2), "v"), b)


def _raw(path, header_bytes, data=b"", hlen=None):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header_bytes) if hlen is None else hlen))
        f.write(header_bytes)
        f.write(data)


@pytest.mark.parametrize("case", ["dtype", "hlen", "json", "offsets", "bytes", "dims", "missing",
                                  "nofile"])
def test_broken_files_raise(tmp_path, case):
    p = str(tmp_path / "x.safetensors")
    ok = json.dumps({"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}).encode()
    if case == "dtype":
        _raw(p, json.dumps({"t": {"dtype": "I8", "shape": [2], "data_offsets": [0, 2]}}).encode(), b"ab")
    elif case == "hlen":
        _raw(p, ok, b"\0" * 8, hlen=1 << 40)
    elif case == "json":
        _raw(p, b'{"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]', b"\0" * 8)
    elif case == "offsets":
        _raw(p, json.dumps({"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 800]}}).encode(),
             b"\0" * 8)
    elif case == "bytes":
        _raw(p, json.dumps({"t": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}).encode(),
             b"\0" * 8)
    elif case == "dims":
        _raw(p, json.dumps({"t": {"dtype": "F32", "shape": [1] * 9, "data_offsets": [0, 4]}}).encode(),
             b"\0" * 4)
    elif case == "missing":
        _raw(p, ok, b"\0" * 8)
        with pytest.raises(E.EmberglassError, match="not found"):
            E.readSafetensorsTensor(p, "nope")
        return
    else:
        p = str(tmp_path / "absent.safetensors")
    with pytest.raises(E.EmberglassError):
        E.readSafetensorsTensor(p, "t")


def model_tensors(cfg, seed=3):
    """Every schema tensor of `cfg` (HF names), N(0, 0.02) matrices / biases,
    norms near 1, rounded through bf16 as a checkpoint would store them."""
    rng = np.random.default_rng(seed)
    H, I, V = cfg["hiddenSize"], cfg["intermediateSize"], cfg["vocabSize"]
    QD, KVD = cfg["numHeads"] * cfg["headDim"], cfg["numKVHeads"] * cfg["headDim"]
    t = {"model.embed_tokens.weight": (V, H), "model.norm.weight": (H,)}
    for i in range(cfg["numLayers"]):
        p = f"model.layers.{i}."
        t.update({p + "input_layernorm.weight": (H,), p + "post_attention_layernorm.weight": (H,),
                  p + "self_attn.q_proj.weight": (QD, H), p + "self_attn.k_proj.weight": (KVD, H),
                  p + "self_attn.v_proj.weight": (KVD, H), p + "self_attn.o_proj.weight": (H, QD),
                  p + "mlp.gate_proj.weight": (I, H), p + "mlp.up_proj.weight": (I, H),
                  p + "mlp.down_proj.weight": (H, I), p + "self_attn.q_proj.bias": (QD,),
                  p + "self_attn.k_proj.bias": (KVD,), p + "self_attn.v_proj.bias": (KVD,)})
    out = {}
    for name, shape in t.items():
        a = rng.standard_normal(shape).astype(np.float32) * 0.02
        if name.endswith("norm.weight"):
            a = 1.0 + a
        out[name] = bf16_bits(a)
    return out


@pytest.mark.gpu
def test_model_from_sharded_bf16_equals_direct_upload(cuda, tmp_path):
    from vibethinker_webgpu_lora_b200.config import small_config
    cfg = small_config(layers=2, vocab=3000)
    ts = model_tensors(cfg)
    names = sorted(ts)
    half = len(names) // 2
    write_st(str(tmp_path / "a.safetensors"), {n: ("BF16", ts[n]) for n in names[:half]})
    write_st(str(tmp_path / "b.safetensors"),
             {**{n: ("BF16", ts[n]) for n in names[half:]},
              "lm_head.weight": ("BF16", ts["model.embed_tokens.weight"])})  # tied: skipped
    with open(tmp_path / "model.safetensors.index.json", "w") as f:
        wm = {n: "a.safetensors" for n in names[:half]}
        wm.update({n: "b.safetensors" for n in names[half:]})
        wm["lm_head.weight"] = "b.safetensors"
        json.dump({"weight_map": wm}, f)
    f32 = {n: (v.astype(np.uint32) << 16).view(np.float32) for n, v in ts.items()}
    rt_a = E.QwenB200(cfg, dict(maxCtx=32)).build(f32)
    rt_b = E.QwenB200(cfg, dict(maxCtx=32)).build(str(tmp_path))
    assert rt_b.tensorsVisited == len(names) + 1
    for t, tok in enumerate([5, 17, 2999, 0]):
        rt_a.token(tok, t)
        rt_b.token(tok, t)
        assert np.array_equal(rt_a.readLogits(), rt_b.readLogits())


@pytest.mark.gpu
def test_model_load_errors(cuda, tmp_path):
    from vibethinker_webgpu_lora_b200.config import small_config
    cfg = small_config(layers=1, vocab=2048)
    ts = model_tensors(cfg)
    p = str(tmp_path / "m.safetensors")
    bad = dict(ts)
    bad["model.norm.weight"] = bad["model.norm.weight"][:-1]  # shape mismatch
    write_st(p, {n: ("BF16", v) for n, v in bad.items()})
    with pytest.raises(E.EmberglassError, match="shape mismatch"):
        E.QwenB200(cfg, dict(maxCtx=32)).build(p)
    part = {n: ("BF16", v) for n, v in ts.items() if "mlp.down_proj" not in n}
    write_st(p, part)
    with pytest.raises(E.EmberglassError, match="missing"):
        E.QwenB200(cfg, dict(maxCtx=32)).build(p)
