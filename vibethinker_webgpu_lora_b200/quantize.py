"""Host quantisers of the reference (src/qwgpu/quantize.js), bit-exact,
implemented in libemberglass_cuda (eg_quantize_*)."""
from __future__ import annotations

import numpy as np

from . import _lib as L


def quantizeInt4Group(W: np.ndarray, group: int = 128):
    """quantizeInt4Group(f32, outDim, inDim, group) (quantize.js:81-111).
    Returns (packed u32[N*K/8], scale f32[N*K/group], groupsPerRow)."""
    W = np.ascontiguousarray(W, np.float32)
    N, K = W.shape
    packed = np.empty(N * K // 8, np.uint32)
    scale = np.empty(N * (K // group), np.float32)
    L.check(L.lib().eg_quantize_int4_group(W.ctypes.data, N, K, group, packed.ctypes.data,
                                           scale.ctypes.data))
    return packed, scale, K // group


def quantizeInt8RowMajor(W: np.ndarray):
    """quantizeInt8RowMajor(f32, outDim, inDim) (quantize.js:28-57)."""
    W = np.ascontiguousarray(W, np.float32)
    N, K = W.shape
    packed = np.empty(N * K // 4, np.uint32)
    scale = np.empty(N, np.float32)
    L.check(L.lib().eg_quantize_int8_rows(W.ctypes.data, N, K, packed.ctypes.data, scale.ctypes.data))
    return packed, scale


def synth_normal(n: int, seed: int, std: float = 1.0, start: int = 0) -> np.ndarray:
    """The seeded N(0, std) stream the synthetic model build draws from."""
    out = np.empty(n, np.float32)
    L.lib().eg_synth_normal(out.ctypes.data, n, seed, std, start)
    return out
