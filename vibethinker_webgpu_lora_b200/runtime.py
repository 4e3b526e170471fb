"""QwenB200: the host-side runtime with the reference's `QwenWGPU` surface
(src/qwgpu/runtime.js:84-2571), driving libemberglass_cuda through its C ABI.

Method names, argument meaning and error behaviour follow the reference
(camelCase kept so reference-style harnesses read the same); all device work
happens in the CUDA library.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib as L
from .config import QWEN25_3B

PROFILE_CATEGORIES = ("embed+qkv", "attn", "o", "gate_up", "down", "lm_head")


def _cfg_struct(cfg: dict) -> L.EgConfig:
    return L.EgConfig(cfg["hiddenSize"], cfg["numLayers"], cfg["numHeads"], cfg["numKVHeads"],
                      cfg["headDim"], cfg["intermediateSize"], cfg["vocabSize"], cfg["rmsNormEps"],
                      cfg["ropeTheta"], int(cfg.get("tieWordEmbeddings", True)),
                      int(cfg.get("attentionBias", True)))


class QwenB200:
    """new QwenWGPU(device, cfg, opts) (runtime.js:87).

    opts: maxCtx, maxPrefillT, decodeBatchSize (capacity of one decodeBatch
    call), samplingTopK, maxSamplingTopK, useF16 (f16 KV cache + the
    reference's f16 staging numerics, default True), attnChunk, useGraphs,
    usePdl, useFused (persistent fused decode), device.
    """

    def __init__(self, cfg: dict | None = None, opts: dict | None = None):
        self.cfg = dict(cfg or QWEN25_3B)
        opts = dict(opts or {})
        o = L.EgOptions()
        L.lib().eg_default_options(C.byref(o))
        o.device = int(opts.get("device", 0))
        o.max_ctx = int(opts.get("maxCtx", 8192))
        o.max_prefill_t = int(opts.get("maxPrefillT", 0))
        o.kv_f16 = int(bool(opts.get("useF16", True)))
        o.decode_batch_capacity = int(opts.get("decodeBatchSize", 32))
        o.sampling_top_k = int(opts.get("samplingTopK", 40))
        o.max_sampling_top_k = int(opts.get("maxSamplingTopK", 64))
        o.attn_chunk = int(opts.get("attnChunk", 0))
        o.use_graphs = int(bool(opts.get("useGraphs", True)))
        o.use_pdl = int(bool(opts.get("usePdl", True)))
        o.use_fused = int(bool(opts.get("useFused", False)))
        o.prefill_chunk = int(opts.get("prefillChunk", 16))
        o.use_tc_batch = int(bool(opts.get("useTcBatch", False)))
        o.prefill_tc = int(bool(opts.get("prefillTc", True)))
        o.prefill_chunk_size = int(opts.get("prefillChunkSize", 0))
        o.use_l2_prefetch = int(bool(opts.get("useL2Prefetch", True)))
        self.opts = o
        h = C.c_void_p()
        L.check(L.lib().eg_create(C.byref(_cfg_struct(self.cfg)), C.byref(o), C.byref(h)))
        self._h = h
        self.lora = None
        self.maxCtx = o.max_ctx

    # ------------------------------------------------------------ lifecycle
    def close(self):
        if getattr(self, "_h", None):
            L.lib().eg_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def usingF16(self) -> bool:
        return bool(self.opts.kv_f16)

    # ------------------------------------------------------------ weights
    def build(self, source="synthetic", seed: int = 0xE6B00000, std: float = 0.02):
        """build(source) (runtime.js:326): 'synthetic' = seeded N(0, std)
        weights; a path = a safetensors model (file, or a directory with
        model.safetensors.index.json / model.safetensors), streamed tensor by
        tensor by the library's loader; or a mapping / iterable of (HF name,
        f32 array)."""
        lib = L.lib()
        if source == "synthetic":
            L.check(lib.eg_build_synthetic(self._h, seed, std))
        elif isinstance(source, (str, os.PathLike)):
            n = C.c_int(0)
            L.check(lib.eg_load_safetensors(self._h, os.fsencode(source), C.byref(n)))
            self.tensorsVisited = n.value
        else:
            items = source.items() if hasattr(source, "items") else source
            for name, arr in items:
                self.uploadTensor(name, arr)
        L.check(lib.eg_finalize(self._h))
        return self

    def uploadTensor(self, name: str, arr: np.ndarray):
        a = np.ascontiguousarray(arr, np.float32)
        shape = (C.c_int64 * a.ndim)(*a.shape)
        L.check(L.lib().eg_upload_tensor(self._h, name.encode(), a.ctypes.data, shape, a.ndim))

    def uploadQuantized(self, name: str, kind: int, packed: np.ndarray, scale: np.ndarray, shape):
        p = np.ascontiguousarray(packed, np.uint32)
        s = np.ascontiguousarray(scale, np.float32)
        sh = (C.c_int64 * len(shape))(*shape)
        L.check(L.lib().eg_upload_quantized(self._h, name.encode(), kind, p.ctypes.data,
                                            s.ctypes.data, sh, len(shape)))

    def finalize(self):
        L.check(L.lib().eg_finalize(self._h))

    # ------------------------------------------------------------ decode
    def token(self, id: int, pos: int):
        """token(id, pos) (runtime.js:1735-1741)."""
        L.check(L.lib().eg_token(self._h, int(id), int(pos)))

    step = token

    def decodeBatch(self, startPos: int, K: int) -> list[int]:
        """decodeBatch(startPos, K) (runtime.js:1776-1793)."""
        out = np.zeros(max(int(K), 1), np.uint32)
        n = C.c_int(0)
        L.check(L.lib().eg_decode_greedy(self._h, int(startPos), int(K), out.ctypes.data, C.byref(n)))
        return out[: n.value].tolist()

    decodeGreedyBatch = decodeBatch

    def decodeBatchAsync(self, startPos: int, K: int) -> int:
        """Enqueue K chained greedy tokens without reading them back."""
        n = C.c_int(0)
        L.check(L.lib().eg_decode_greedy_async(self._h, int(startPos), int(K), C.byref(n)))
        return n.value

    def readIds(self, n: int) -> list[int]:
        out = np.zeros(max(int(n), 1), np.uint32)
        L.check(L.lib().eg_read_ids(self._h, out.ctypes.data, int(n)))
        return out[: int(n)].tolist()

    def sync(self):
        L.check(L.lib().eg_sync(self._h))

    @property
    def stream(self) -> int:
        return L.lib().eg_stream(self._h)

    def prefillBatch(self, ids):
        """prefillBatch(ids) (runtime.js:1936-1945)."""
        a = np.ascontiguousarray(ids, np.uint32)
        L.check(L.lib().eg_prefill(self._h, a.ctypes.data, int(a.size)))

    def argmaxLogits(self) -> int:
        v = C.c_uint32(0)
        L.check(L.lib().eg_argmax(self._h, C.byref(v)))
        return int(v.value)

    def topKLogits(self, k: int | None = None):
        k = self.opts.sampling_top_k if k is None else int(k)
        ids = np.zeros(64, np.uint32)
        vals = np.zeros(64, np.float32)
        kk = C.c_int(0)
        L.check(L.lib().eg_topk(self._h, k, ids.ctypes.data, vals.ctypes.data, C.byref(kk)))
        return [{"id": int(ids[i]), "logit": float(vals[i])} for i in range(kk.value)]

    def sampleToken(self, temp: float = 1.0, r: float | None = None) -> int:
        if r is None:
            r = float(np.random.random())
        v = C.c_uint32(0)
        L.check(L.lib().eg_sample(self._h, float(temp), float(r), C.byref(v)))
        return int(v.value)

    def readLogits(self) -> np.ndarray:
        out = np.empty(self.cfg["vocabSize"], np.float32)
        L.check(L.lib().eg_read_logits(self._h, out.ctypes.data))
        return out

    def readHidden(self) -> np.ndarray:
        out = np.empty(self.cfg["hiddenSize"], np.float32)
        L.check(L.lib().eg_read_hidden(self._h, out.ctypes.data))
        return out

    def generate(self, promptIds, maxNewTokens: int = 32, opts: dict | None = None) -> list[int]:
        """generate(ids, n, {sample, temp, rSeq}) (runtime.js:2481-2516)."""
        opts = opts or {}
        p = np.ascontiguousarray(promptIds, np.uint32)
        n = int(maxNewTokens)
        out = np.zeros(max(n, 1), np.uint32)
        sample = bool(opts.get("sample", False))
        r = None
        if sample:
            r = np.ascontiguousarray(opts.get("rSeq", np.random.random(n)), np.float32)
        L.check(L.lib().eg_generate(self._h, p.ctypes.data, int(p.size), n, int(sample),
                                    float(opts.get("temp", 1.0)),
                                    None if r is None else r.ctypes.data, out.ctypes.data))
        ids = out[:n].tolist()
        cb = opts.get("onToken")
        if cb:
            for t in ids:
                cb(t)
        return ids

    # ------------------------------------------------------------ multi-sequence
    def seqInit(self, nSlots: int, slotCtx: int):
        """Allocate nSlots independent sequences of slotCtx positions each."""
        L.check(L.lib().eg_seq_init(self._h, int(nSlots), int(slotCtx)))

    def seqInitPaged(self, nSlots: int, slotCtx: int, nPages: int):
        """Slots sharing a pool of nPages 16-position KV pages per layer
        (PagedAttentionManager, runtime.js:2573-2616)."""
        L.check(L.lib().eg_seq_init_paged(self._h, int(nSlots), int(slotCtx), int(nPages)))

    def seqRelease(self, slot: int):
        """freeSeq: empty the slot, its pages back to the pool."""
        L.check(L.lib().eg_seq_release(self._h, int(slot)))

    def seqPages(self) -> tuple[int, int]:
        """(free pages, pool pages)."""
        f, t = C.c_int(0), C.c_int(0)
        L.check(L.lib().eg_seq_pages(self._h, C.byref(f), C.byref(t)))
        return f.value, t.value

    def seqSetPrompt(self, slot: int, ids):
        """Load a slot's prompt; its position returns to 0."""
        p = np.ascontiguousarray(ids, np.uint32)
        L.check(L.lib().eg_seq_set_prompt(self._h, int(slot), p.ctypes.data, int(p.size)))

    def seqPrefill(self, slot: int):
        """Run the slot's prompt up to its last token in batched chunks."""
        L.check(L.lib().eg_seq_prefill(self._h, int(slot)))

    def seqState(self, slot: int) -> tuple[int, int]:
        """(position, known ids) of a slot."""
        pos, n = C.c_int(0), C.c_int(0)
        L.check(L.lib().eg_seq_state(self._h, int(slot), C.byref(pos), C.byref(n)))
        return pos.value, n.value

    def batchDecode(self, slots, steps: int) -> np.ndarray:
        """`steps` batched greedy steps over `slots` (<= 16): [steps][len(slots)]
        tokens at each slot's new position (prompt tokens while prefilling)."""
        sl = np.ascontiguousarray(slots, np.int32)
        out = np.zeros((max(int(steps), 1), sl.size), np.uint32)
        L.check(L.lib().eg_batch_decode(self._h, int(sl.size), sl.ctypes.data, int(steps),
                                        out.ctypes.data))
        return out[:int(steps)]

    def batchSample(self, slots, steps: int, k: int, temp: float, r) -> np.ndarray:
        """As batchDecode with top-k sampling; r[steps][len(slots)] uniforms."""
        sl = np.ascontiguousarray(slots, np.int32)
        rr = np.ascontiguousarray(r, np.float32).reshape(int(steps), sl.size)
        out = np.zeros((max(int(steps), 1), sl.size), np.uint32)
        L.check(L.lib().eg_batch_sample(self._h, int(sl.size), sl.ctypes.data, int(steps), int(k),
                                        float(temp), rr.ctypes.data, out.ctypes.data))
        return out[:int(steps)]

    def batchLogits(self, lane: int) -> np.ndarray:
        """Logits of lane `lane` of the last batch call after its last step."""
        out = np.empty(self.cfg["vocabSize"], np.float32)
        L.check(L.lib().eg_batch_read_logits(self._h, int(lane), out.ctypes.data))
        return out

    # ------------------------------------------------------------ LoRA
    def setLora(self, adapter):
        """setLora(adapter) (runtime.js:717-721)."""
        L.check(L.lib().eg_set_lora(self._h, adapter.handle))
        self.lora = adapter

    def clearLora(self):
        L.check(L.lib().eg_clear_lora(self._h))
        self.lora = None

    def invalidateLora(self):
        L.check(L.lib().eg_invalidate_lora(self._h))

    # ------------------------------------------------------------ observability
    def profToken(self, id: int, pos: int) -> dict:
        us = (C.c_double * 6)()
        n = C.c_int(0)
        L.check(L.lib().eg_profile_token(self._h, int(id), int(pos), us, C.byref(n)))
        return {PROFILE_CATEGORIES[i]: us[i] for i in range(n.value)}

    def profFused(self, startPos: int) -> dict:
        """Per-phase microseconds of one fused greedy step: 'work' = phase
        start to the last CTA's end of work, 'wait' = from there to the next
        phase's start (barrier + skew), summed by phase kind."""
        n = 2 * (5 * self.cfg["numLayers"] + 1)
        buf = np.zeros(n, np.uint64)
        nn = C.c_int(0)
        L.check(L.lib().eg_profile_fused(self._h, int(startPos), buf.ctypes.data, n, C.byref(nn)))
        t = buf.astype(np.int64)
        kinds = ["qkv", "attn", "o", "gate_up", "down"]
        out = {f"{k}_{w}": 0.0 for k in kinds + ["lm_head"] for w in ("work", "wait")}
        nph = n // 2
        for p in range(nph):
            k = "lm_head" if p == nph - 1 else kinds[p % 5]
            out[f"{k}_work"] += (t[2 * p + 1] - t[2 * p]) / 1000
            if p + 1 < nph:
                out[f"{k}_wait"] += (t[2 * p + 2] - t[2 * p + 1]) / 1000
        out["total"] = (t[-1] - t[0]) / 1000
        return out

    def memoryFootprintBytes(self) -> dict:
        kv, w, s = C.c_int64(), C.c_int64(), C.c_int64()
        L.check(L.lib().eg_memory_footprint(self._h, C.byref(kv), C.byref(w), C.byref(s)))
        return {"kvBytes": kv.value, "packedBytes": w.value, "decodeScratchBytes": s.value}

    def estimateKvCacheBytes(self) -> int:
        c = self.cfg
        return c["numLayers"] * 2 * c["numKVHeads"] * self.maxCtx * c["headDim"] * (
            2 if self.usingF16() else 4)

    @property
    def lastDispatchCount(self) -> int:
        return L.lib().eg_launches_per_step(self._h)


def readSafetensorsTensor(path, name: str) -> np.ndarray:
    """One tensor of a safetensors file / model directory decoded to f32 by
    the library's loader (BF16 / F16 / F32, safetensors_loader.js:20-54)."""
    shape = (C.c_int64 * 8)()
    nd = C.c_int(0)
    p, n = os.fsencode(path), name.encode()
    L.check(L.lib().eg_safetensors_tensor(p, n, None, 0, shape, C.byref(nd)))
    dims = tuple(shape[i] for i in range(nd.value))
    out = np.empty(dims, np.float32)
    L.check(L.lib().eg_safetensors_tensor(p, n, out.ctypes.data, out.size, shape, C.byref(nd)))
    return out
