"""Pins the CPU oracle (oracle/oracle.c) against the reference's own known
answers and hand-derived quantiser cases.  No GPU."""
import json
import math
import os

import numpy as np

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    with open(os.path.join(GOLD, name)) as f:
        return json.load(f)


def test_argmax_topk_ties_reference_case():
    g = _load("reference_known_answers.json")["topk_argmax_ties"]
    logits = np.full(g["n"], g["fill"], np.float32)
    for i, v in g["set"].items():
        logits[int(i)] = v
    assert O.argmax(logits) == g["expect_argmax"]
    ids, vals = O.topk(logits, 3)
    assert ids[0] == g["expect_top1"]
    assert list(ids) == [1, 256, 129]  # value desc, ties to the lower index
    picked = O.sample_topk(np.array(g["sample_ids"], np.uint32), np.array(g["sample_vals"], np.float32),
                           len(g["sample_ids"]), g["sample_temp"], g["sample_r"])
    assert picked == g["expect_sample"]


def test_sampler_edges():
    ids = np.array([5, 6, 7], np.uint32)
    vals = np.array([1.0, 1.0, 1.0], np.float32)
    assert O.sample_topk(ids, vals, 3, 1.0, 0.0) == 5      # r <= P_0
    assert O.sample_topk(ids, vals, 3, 1.0, 1.0) == 7      # r = 1 -> last (prefix may round below 1)
    assert O.sample_topk(ids, vals, 0, 1.0, 0.5) == 0      # k = 0
    # temperature <= 0 means 1 (kernels.js:823)
    v2 = np.array([3.0, 1.0, 0.0], np.float32)
    assert O.sample_topk(ids, v2, 3, 0.0, 0.95) == O.sample_topk(ids, v2, 3, 1.0, 0.95)
    # exp overflow without max subtraction: sum is inf -> invSum 0 -> prefix all 0 -> chosen = first j with r<=0
    big = np.array([100.0, 99.0], np.float32)
    assert O.sample_topk(ids[:2], big, 2, 1.0, 0.5) == 6


def test_argmax_nan_and_floor():
    x = np.array([np.nan, -2e30, -1e30, -1e30], np.float32)
    assert O.argmax(x) == 2          # NaN never wins, < -1e30 never taken, ties -> lowest
    x = np.array([np.nan, np.nan], np.float32)
    assert O.argmax(x) == 0xFFFFFFFF


def test_quantizer_hand_cases():
    q = _load("quantizer_cases.json")
    for case in q["int4"]:
        row = np.zeros(case["pad_to"], np.float32)
        row[: len(case["row"])] = case["row"]
        packed, scale = O.quantize_int4_group(row[None, :])
        assert scale[0] == np.float32(case["scale"])
        nib = [(int(packed[0]) >> (4 * j)) & 0xF for j in range(8)]
        got = [n - 16 if n > 7 else n for n in nib]
        assert got == case["q"], (case, got)
    for case in q["int8"]:
        row = np.array(case["row"], np.float32)
        packed, scale = O.quantize_int8_rows(row[None, :])
        got = packed.view(np.int8).tolist()
        assert got == case["q"]
        assert scale[0] == np.float32(case["scale"])


def test_gemm_test_reference_case():
    """test/gemm_test.js: int4-quantised GEMM vs a CPU dequant reference with
    JS-double accumulation, maxAbs < 1e-2 (T=40, K=2048, N=517)."""
    g = _load("reference_known_answers.json")["gemm_test"]
    T, K, N = g["T"], g["K"], g["N"]
    A = ((np.sin(np.arange(T * K) * 0.3) + np.cos(np.arange(T * K) * 0.7)) * 0.5).astype(np.float32)
    W = (np.sin(np.arange(N * K) * 0.11) * 0.4).astype(np.float32).reshape(N, K)
    bias = (np.cos(np.arange(N)) * 0.1).astype(np.float32)
    packed, scale = O.quantize_int4_group(W)
    deq = O.dequant_int4(packed, scale, N, K)
    A = A.reshape(T, K)
    ref = bias[None, :].astype(np.float64) + A.astype(np.float64) @ deq.astype(np.float64).T
    got = np.stack([O.gemv_q4(A[t], packed, scale, N, K, bias=bias) for t in range(T)])
    assert np.abs(got - ref).max() < g["max_abs"]


def test_rope_tables_and_pair():
    c, s = O.rope_tables(4, 128, 1e6)
    assert c[0] == 1.0 and s[0] == 0.0
    assert c[128 + 1] == np.float32(math.cos(1 / 1e6 ** (2 / 128)))
    q = O.normal(16 * 128, 11)
    k = O.normal(2 * 128, 12)
    q2, k2 = O.rope_qk(q, k, 16, 2, 128, 0, c, s)
    assert np.array_equal(q2, q) and np.array_equal(k2, k)  # pos 0 is the identity
    q3, _ = O.rope_qk(q, k, 16, 2, 128, 3, c, s)
    lo, hi = q[0], q[64]
    assert q3[0] == np.float32(np.float32(lo * c[3 * 128]) + np.float32(-hi * s[3 * 128]))


def test_attention_split_invariance():
    """Split-K merge is exact math: chunk size only changes rounding."""
    ctx, nh, nkv = 300, 16, 2
    q = O.normal(nh * 128, 21)
    kc = O.normal(ctx * nkv * 128, 22)
    vc = O.normal(ctx * nkv * 128, 23)
    a = O.attention(q, kc, vc, nh, nkv, ctx, 128, 128)
    b = O.attention(q, kc, vc, nh, nkv, ctx, 128, 16)
    # f64 reference
    Q = q.reshape(nh, 128).astype(np.float64)
    Kc = kc.reshape(ctx, nkv, 128).astype(np.float64)
    Vc = vc.reshape(ctx, nkv, 128).astype(np.float64)
    ref = np.zeros((nh, 128))
    for h in range(nh):
        kvh = h // (nh // nkv)
        sc = Kc[:, kvh] @ Q[h] / math.sqrt(128)
        p = np.exp(sc - sc.max())
        ref[h] = p @ Vc[:, kvh] / p.sum()
    assert np.abs(a - ref.ravel()).max() < 1e-5
    assert np.abs(b - ref.ravel()).max() < 1e-5


def test_f16_rounding_paths():
    x = O.normal(2048, 31) * 3
    g = np.ones(2048, np.float32)
    y32 = O.rmsnorm(x, g, 1e-6, False)
    y16 = O.rmsnorm(x, g, 1e-6, True)
    assert np.array_equal(y16, y16.astype(np.float16).astype(np.float32))
    assert np.abs(y16 - y32).max() < 4e-3


def test_generator_is_counter_based():
    a = O.normal(1000, 77, 0.02)
    b = O.normal(500, 77, 0.02, start=500)
    assert np.array_equal(a[500:], b)
    assert abs(float(a.std()) - 0.02) < 0.002
