"""LoRA adapters: loadLoraAdapter (src/lora_gpu.js:65-113) over the C ABI.

Parses a PEFT/MLX adapter (.safetensors + adapter_config.json), maps tensor
names to module keys with moduleKeyFromTensorName (model_schema.js:130-134),
derives the scale exactly as the reference (lora_parameters.scale, else
lora_alpha / r, else alpha / r, else 2.0), and hands A/B to the library,
which stores A as [rank][in] and B as [rank][out] on the device.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import re
import struct

import numpy as np

from . import _lib as L
from .quantize import synth_normal

PROJ_KEYS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
             "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")

_KEY_RE = re.compile(r"layers\.(\d+)\.(self_attn|mlp)\.([a-z_]+?)(_proj)?\.(lora_[ABab])", re.I)


def moduleKeyFromTensorName(name: str):
    m = _KEY_RE.search(name)
    if not m:
        return None
    return f"layers.{m.group(1)}.{m.group(2)}.{re.sub(r'_proj$', '', m.group(3))}_proj"


class LoraAdapter:
    """{name, modules: {key: {rank, scale}}} plus the device handle."""

    def __init__(self, rt, name: str, modules: dict):
        self.rt = rt
        self.name = name
        keep = []
        arr = (L.EgLoraModule * len(modules))()
        for i, (key, m) in enumerate(modules.items()):
            A = np.ascontiguousarray(m["A"], np.float32)
            B = np.ascontiguousarray(m["B"], np.float32)
            keep += [A, B]
            k = key.encode()
            keep.append(k)
            arr[i] = L.EgLoraModule(k, A.ctypes.data, A.shape[0], A.shape[1], B.ctypes.data,
                                    B.shape[0], B.shape[1], float(m["scale"]))
        h = C.c_void_p()
        L.check(L.lib().eg_lora_create(rt.handle, len(modules), arr, C.byref(h)))
        self.handle = h
        self.modules = {k: {"rank": int(min(*np.shape(m["A"]), *np.shape(m["B"]))),
                            "scale": float(m["scale"])} for k, m in modules.items()}

    def update(self, key: str, A: np.ndarray | None = None, B: np.ndarray | None = None):
        """Overwrite one module's A ([r][in]) / B ([r][out]) in place; call
        rt.invalidateLora() afterwards, as the reference does after an
        optimizer step (runtime.js:727-734)."""
        a = None if A is None else np.ascontiguousarray(A, np.float32)
        b = None if B is None else np.ascontiguousarray(B, np.float32)
        L.check(L.lib().eg_lora_update(self.rt.handle, self.handle, key.encode(),
                                       None if a is None else a.ctypes.data,
                                       None if b is None else b.ctypes.data))

    def destroy(self):
        if self.handle:
            L.lib().eg_lora_destroy(self.rt.handle, self.handle)
            self.handle = None


def _read_safetensors(path: str) -> dict:
    with open(path, "rb") as f:
        buf = f.read()
    (hl,) = struct.unpack("<Q", buf[:8])
    header = json.loads(buf[8:8 + hl].decode())
    base = 8 + hl
    out = {}
    for name, t in header.items():
        if name == "__metadata__":
            continue
        s, e = t["data_offsets"]
        raw = buf[base + s: base + e]
        dt = t["dtype"].upper()
        if dt == "BF16":
            u16 = np.frombuffer(raw, np.uint16).astype(np.uint32) << 16
            arr = u16.view(np.float32)
        elif dt == "F16":
            arr = np.frombuffer(raw, np.float16).astype(np.float32)
        else:
            arr = np.frombuffer(raw, np.float32).copy()
        out[name] = arr.reshape(t["shape"])
    return out


def parseLoraAdapter(files: list[str]) -> tuple[str, dict]:
    """The host half of loadLoraAdapterGPU (lora_gpu.js:65-113): the adapter
    name and {module key: {A, B, scale}} with A / B as the file holds them.
    Scale: lora_parameters.scale (MLX), else lora_alpha / rank (PEFT), else
    alpha / rank, else 2.0; rank from r / rank / lora_rank /
    lora_parameters.rank, 16 when absent (lora_gpu.js:68-80)."""
    st = [f for f in files if f.endswith(".safetensors")]
    if not st:
        raise ValueError("no .safetensors in adapter files")
    conf = [f for f in files if re.search(r"adapter_config\.json|config\.json", os.path.basename(f))]
    rank_cfg, scale_cfg = 16, None
    if conf:
        with open(conf[0]) as f:
            c = json.load(f)
        lp = c.get("lora_parameters") or {}
        for k in ("r", "rank", "lora_rank"):
            if c.get(k) is not None:
                rank_cfg = c[k]
                break
        else:
            if lp.get("rank") is not None:
                rank_cfg = lp["rank"]
        if lp.get("scale") is not None:
            scale_cfg = lp["scale"]
        elif c.get("lora_alpha") is not None:
            scale_cfg = c["lora_alpha"] / rank_cfg
        elif c.get("alpha") is not None:
            scale_cfg = c["alpha"] / rank_cfg
    tensors = _read_safetensors(st[0])
    groups: dict = {}
    for name, arr in tensors.items():
        if not re.search(r"lora_[abAB]", name):
            continue
        key = moduleKeyFromTensorName(name)
        if not key:
            continue
        groups.setdefault(key, {})["A" if re.search(r"lora_a", name, re.I) else "B"] = arr
    scale = scale_cfg if scale_cfg is not None else 2.0
    modules = {k: {"A": g["A"], "B": g["B"], "scale": scale} for k, g in groups.items()
               if "A" in g and "B" in g}
    if not modules:
        raise ValueError("no LoRA modules matched layers.*.{self_attn,mlp}.*_proj")
    return os.path.basename(st[0]).rsplit(".safetensors", 1)[0], modules


def orientLora(A: np.ndarray, B: np.ndarray, in_dim: int, out_dim: int):
    """(A [r][in], B [r][out], r) as the library stores them (eg_lora_orient,
    lora_gpu.js:100-107)."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    r = int(min(*A.shape, *B.shape))
    a = np.empty((r, in_dim), np.float32)
    b = np.empty((r, out_dim), np.float32)
    rr = C.c_int(0)
    L.check(L.lib().eg_lora_orient(A.ctypes.data, A.shape[0], A.shape[1], B.ctypes.data, B.shape[0],
                                   B.shape[1], in_dim, out_dim, a.ctypes.data, b.ctypes.data, C.byref(rr)))
    return a, b, rr.value


def loadLoraAdapter(rt, files: list[str], cfg: dict | None = None) -> LoraAdapter:
    """loadLoraAdapterGPU(dev, files, cfg) (lora_gpu.js:65-113)."""
    name, modules = parseLoraAdapter(files)
    return LoraAdapter(rt, name, modules)


def synthetic_modules(cfg: dict, seed: int, rank: int = 8, alpha: float = 16.0,
                      std_a: float = 0.02, std_b: float = 0.01) -> dict:
    """Adapter on q,k,v,o,gate,up,down of every layer: module 7i+p draws
    A ~ N(0, std_a) [rank][in] from stream 2(7i+p) of `seed` and
    B ~ N(0, std_b) [rank][out] from stream 2(7i+p)+1; scale = alpha/rank."""
    lib = L.lib()
    H, I = cfg["hiddenSize"], cfg["intermediateSize"]
    QD, KVD = cfg["numHeads"] * cfg["headDim"], cfg["numKVHeads"] * cfg["headDim"]
    dims = [(QD, H), (KVD, H), (KVD, H), (H, QD), (I, H), (I, H), (H, I)]
    mods = {}
    for i in range(cfg["numLayers"]):
        for p, (N, K) in enumerate(dims):
            m = 7 * i + p
            A = synth_normal(rank * K, lib.eg_synth_stream_at(seed, 2 * m), std_a).reshape(rank, K)
            B = synth_normal(rank * N, lib.eg_synth_stream_at(seed, 2 * m + 1), std_b).reshape(rank, N)
            mods[f"layers.{i}.{PROJ_KEYS[p]}"] = {"A": A, "B": B, "scale": alpha / rank}
    return mods


def synthetic_adapter(rt, seed: int, rank: int = 8, alpha: float = 16.0, name: str = "synthetic"):
    return LoraAdapter(rt, name, synthetic_modules(rt.cfg, seed, rank, alpha))
