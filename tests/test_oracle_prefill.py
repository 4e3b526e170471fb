"""The oracle's restatement of prefillBatch (runtime.js:1936-2087) on the CPU.

The reference checks its batched prefill against the token loop
(test/prefill_diff.js:88-103: same argmax, same greedy continuation); these
tests hold the oracle's GEMM4 / ROPE_T / ATTN_PREFILL_BLOCK / SILUMUL
restatements to the decode-step restatements, which are pinned separately.
"""
import numpy as np

from oracle import oracle as O
from vibethinker_webgpu_lora_b200.config import small_config

SEED = 0xE6B00000


def test_gemm4_reference_case():
    """test/gemm_test.js:21-60 through GEMM4's own arithmetic (dequantise the
    word, then the eight products): maxAbs < 1e-2 against the f64 dequant."""
    T, K, N = 40, 2048, 517
    A = ((np.sin(np.arange(T * K) * 0.3) + np.cos(np.arange(T * K) * 0.7)) * 0.5).astype(np.float32)
    W = (np.sin(np.arange(N * K) * 0.11) * 0.4).astype(np.float32).reshape(N, K)
    bias = (np.cos(np.arange(N)) * 0.1).astype(np.float32)
    packed, scale = O.quantize_int4_group(W)
    deq = O.dequant_int4(packed, scale, N, K)
    A = A.reshape(T, K)
    ref = bias[None, :].astype(np.float64) + A.astype(np.float64) @ deq.astype(np.float64).T
    got = O.gemm4(A, packed, scale, N, K, bias=bias)
    assert np.abs(got - ref).max() < 1e-2
    # GEMM4_ADD_T adds onto Y
    y0 = O.normal(T * N, 3).reshape(T, N)
    y = y0.copy()
    O.gemm4(A, packed, scale, N, K, bias=bias, Y=y, add=True)
    assert np.abs(y - (y0 + got)).max() < 1e-5


def test_attn_prefill_equals_decode_attention():
    """ATTN_PREFILL_BLOCK's online softmax over 128-key blocks and the decode
    split-K attention are the same function: every row agrees to f32
    rounding, for a whole prompt and for a later chunk (q_start > 0)."""
    nh, nkv, hd, ctx = 16, 2, 128, 300
    q = O.normal(ctx * nh * hd, 31)
    kc = O.normal(ctx * nkv * hd, 32)
    vc = O.normal(ctx * nkv * hd, 33)
    full = O.attn_prefill(q, kc, vc, nh, nkv, hd, ctx, 0, ctx).reshape(ctx, nh * hd)
    for t in (0, 1, 127, 128, 200, 299):
        ref = O.attention(q[t * nh * hd:(t + 1) * nh * hd], kc, vc, nh, nkv, t + 1, hd)
        assert np.abs(full[t] - ref).max() < 2e-5
    q0 = 140
    part = O.attn_prefill(q[q0 * nh * hd:], kc, vc, nh, nkv, hd, ctx - q0, q0, ctx).reshape(-1, nh * hd)
    assert np.abs(part - full[q0:]).max() < 1e-6


def test_silu_mul_f16():
    g = O.normal(1000, 41, 3.0)
    u = O.normal(1000, 42)
    a = g.copy()
    O.lib().orc_silu_mul(a, u, a.size, 0)
    ref = (g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64)))) * u
    assert np.abs(a - ref).max() < 1e-5
    b = g.copy()
    O.lib().orc_silu_mul(b, u, b.size, 1)
    sg = (g / (1 + np.exp(-g))).astype(np.float32)
    want = (sg.astype(np.float16) * u.astype(np.float16)).astype(np.float32)
    assert np.array_equal(b, want)


def test_prefill_matches_token_loop_f32():
    """prefill_diff.js:88-103 on the oracle: the whole-prompt pass and the
    chunked pass (_prefillChunked) agree with the token loop's logits to f32
    rounding, and the greedy continuation after either is the same stream."""
    cfg = small_config(layers=2, vocab=3000, inter=512)
    prompt = O.token_ids(150, 7, cfg["vocabSize"])
    a = O.OracleModel(cfg, 256, False, SEED)
    for t, tok in enumerate(prompt):
        ref = a.step(int(tok), t)
    ids_a, _ = a.generate(prompt, 1)  # argmax of the loop's last logits
    b = O.OracleModel(cfg, 256, False, SEED)
    got = b.prefill(prompt)
    assert np.abs(got - ref).max() < 2e-3
    assert O.argmax(got) == O.argmax(ref) == int(ids_a[0])
    c = O.OracleModel(cfg, 256, False, SEED)
    got_c = c.prefill(prompt, chunk=64)
    assert np.abs(got_c - got).max() < 2e-3
    # decode continues from position T on the prefilled cache
    tok = O.argmax(got)
    step_b = b.step(tok, len(prompt))
    step_a = a.step(tok, len(prompt))
    assert np.abs(step_b - step_a).max() < 2e-3
