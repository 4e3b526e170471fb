"""loadLoraAdapter's host side on CPU (src/lora_gpu.js:65-113): adapter
files written here in the PEFT and MLX conventions, the scale chain
(lora_parameters.scale, lora_alpha / r, alpha / r, default 2.0), the rank
taken from the smallest dimension, the [r][in] / [r][out] orientation the
library stores (eg_lora_orient), and the reference's error texts."""
import json
import struct

import numpy as np
import pytest

import vibethinker_webgpu_lora_b200 as E

R, HID, KV = 8, 2048, 256


def write_safetensors(path, tensors):
    header, blobs, off = {}, [], 0
    for name, (arr, dt) in tensors.items():
        if dt == "BF16":
            raw = (np.ascontiguousarray(arr, np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
        else:
            raw = np.ascontiguousarray(arr, np.float32).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def bf16(a):  # the value a BF16 file holds
    return ((np.asarray(a, np.float32).view(np.uint32) >> 16) << 16).view(np.float32)


def rng(seed, *shape):
    return np.random.default_rng(seed).normal(0, 0.02, shape).astype(np.float32)


def test_peft_adapter(tmp_path):
    # PEFT: lora_A [r][in], lora_B [out][r]; scale = lora_alpha / r
    A_q, B_q = rng(1, R, HID), rng(2, HID, R)
    A_k, B_k = rng(3, R, HID), rng(4, KV, R)
    st = tmp_path / "adapter_model.safetensors"
    write_safetensors(st, {
        "base_model.model.model.layers.0.self_attn.q_proj.lora_A.weight": (A_q, "F32"),
        "base_model.model.model.layers.0.self_attn.q_proj.lora_B.weight": (B_q, "F32"),
        "base_model.model.model.layers.3.self_attn.k_proj.lora_A.weight": (A_k, "BF16"),
        "base_model.model.model.layers.3.self_attn.k_proj.lora_B.weight": (B_k, "BF16"),
        "base_model.model.model.layers.0.mlp.gate_proj.lora_A.weight": (rng(5, R, HID), "F32"),
        "base_model.model.lm_head.weight": (rng(6, 4, 4), "F32"),  # not a LoRA tensor
    })
    cfg = tmp_path / "adapter_config.json"
    cfg.write_text(json.dumps({"r": 8, "lora_alpha": 16}))
    name, mods = E.parseLoraAdapter([str(st), str(cfg)])
    assert name == "adapter_model"
    # gate_proj has only A: skipped, as the reference skips modules missing A or B
    assert sorted(mods) == ["layers.0.self_attn.q_proj", "layers.3.self_attn.k_proj"]
    assert all(m["scale"] == 2.0 for m in mods.values())
    a, b, r = E.orientLora(mods["layers.0.self_attn.q_proj"]["A"], mods["layers.0.self_attn.q_proj"]["B"], HID, HID)
    assert r == R and np.array_equal(a, A_q) and np.array_equal(b, B_q.T)
    a, b, r = E.orientLora(mods["layers.3.self_attn.k_proj"]["A"], mods["layers.3.self_attn.k_proj"]["B"], HID, KV)
    assert r == R and np.array_equal(a, bf16(A_k)) and np.array_equal(b, bf16(B_k).T)


def test_mlx_adapter(tmp_path):
    # MLX: lora_a [in][r], lora_b [r][out]; scale = lora_parameters.scale
    A, B = rng(7, HID, 4), rng(8, 4, 11008)
    st = tmp_path / "adapters.safetensors"
    write_safetensors(st, {"model.layers.2.mlp.up_proj.lora_a": (A, "F32"),
                           "model.layers.2.mlp.up_proj.lora_b": (B, "F32")})
    cfg = tmp_path / "adapter_config.json"
    cfg.write_text(json.dumps({"lora_parameters": {"rank": 4, "scale": 20.0}, "lora_alpha": 99}))
    name, mods = E.parseLoraAdapter([str(cfg), str(st)])
    assert name == "adapters" and list(mods) == ["layers.2.mlp.up_proj"]
    assert mods["layers.2.mlp.up_proj"]["scale"] == 20.0  # lora_parameters.scale wins
    a, b, r = E.orientLora(A, B, HID, 11008)
    assert r == 4 and np.array_equal(a, A.T) and np.array_equal(b, B)


@pytest.mark.parametrize("conf,scale", [
    ({"rank": 4, "alpha": 8}, 2.0),               # alpha / rank
    ({"lora_rank": 8, "alpha": 32}, 4.0),         # lora_rank
    ({"lora_alpha": 24}, 1.5),                    # rank defaults to 16
    ({"lora_parameters": {"rank": 8}, "lora_alpha": 4}, 0.5),
    ({"r": 8}, 2.0),                              # no scale given: 2.0
    (None, 2.0),                                  # no config file: 2.0
])
def test_scale_chain(tmp_path, conf, scale):
    st = tmp_path / "a.safetensors"
    write_safetensors(st, {"layers.1.self_attn.o_proj.lora_A.weight": (rng(9, R, HID), "F32"),
                           "layers.1.self_attn.o_proj.lora_B.weight": (rng(10, HID, R), "F32")})
    files = [str(st)]
    if conf is not None:
        (tmp_path / "config.json").write_text(json.dumps(conf))
        files.append(str(tmp_path / "config.json"))
    _, mods = E.parseLoraAdapter(files)
    assert mods["layers.1.self_attn.o_proj"]["scale"] == scale


def test_errors(tmp_path):
    with pytest.raises(ValueError, match="no .safetensors in adapter files"):
        E.parseLoraAdapter([str(tmp_path / "adapter_config.json")])
    st = tmp_path / "x.safetensors"
    write_safetensors(st, {"model.embed_tokens.lora_A.weight": (rng(11, R, 16), "F32")})
    with pytest.raises(ValueError, match=r"no LoRA modules matched layers\.\*\.\{self_attn,mlp\}\.\*_proj"):
        E.parseLoraAdapter([str(st)])
    # shapes that cannot be a rank-r update of a 2048 x 2048 projection
    with pytest.raises(E.EmberglassError, match="lora_orient"):
        E.orientLora(rng(12, R, 1024), rng(13, HID, R), HID, HID)


def test_module_keys():
    k = E.moduleKeyFromTensorName
    assert k("base_model.model.model.layers.12.mlp.down_proj.lora_B.weight") == "layers.12.mlp.down_proj"
    assert k("model.layers.0.self_attn.v_proj.lora_a") == "layers.0.self_attn.v_proj"
    assert k("model.norm.weight") is None
