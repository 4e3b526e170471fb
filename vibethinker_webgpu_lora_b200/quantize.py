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


def _splitmix_at(seed: int, n: int) -> np.ndarray:
    """Outputs 0..n-1 of the counter-form SplitMix64 stream starting at
    `seed` (the synthetic-input generator of the model build)."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (np.arange(1, n + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15))
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def synth_ids(n: int, seed: int, vocab: int) -> np.ndarray:
    """n uniform token ids (SplitMix64 output mod vocab)."""
    return (_splitmix_at(seed, n) % np.uint64(vocab)).astype(np.uint32)


def synth_uniform(n: int, seed: int) -> np.ndarray:
    """n uniforms in [0, 1) from the top 53 bits, rounded to f32."""
    return ((_splitmix_at(seed, n) >> np.uint64(11)).astype(np.float64) * 2.0 ** -53).astype(np.float32)
