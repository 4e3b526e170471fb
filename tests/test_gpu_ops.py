"""Single-op parity: every CUDA kernel entry point against the CPU oracle on
the same seeded inputs.  Tolerances: logits/activations max-abs <= 1e-2 and
mean-rel <= 1e-3 (the reference f32 path bar), much tighter where the op is
short; index outputs (argmax, top-k ids, sampled id) bit-exact."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from vibethinker_webgpu_lora_b200 import kernels as K

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def close(got, ref, max_abs, mean_rel=1e-3):
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    assert d.max() <= max_abs, f"max abs {d.max()}"
    rel = d.mean() / max(np.abs(ref).mean(), 1e-12)  # mean relative error
    assert rel <= mean_rel, f"mean rel {rel}"


@pytest.mark.parametrize("N,Kd,seed", [(2048, 2048, 1), (517, 2048, 2), (2560, 2048, 3),
                                       (2048, 11008, 4), (16, 128, 5), (1, 256, 6)])
def test_gemv_q4(cuda, N, Kd, seed):
    W = O.normal(N * Kd, 0xE6B00001 + seed, 0.02).reshape(N, Kd)
    x = O.normal(Kd, 0xE6B00002 + seed, 1.0)
    bias = O.normal(N, 0xE6B00003 + seed, 0.02)
    p, s = O.quantize_int4_group(W)
    ref = O.gemv_q4(x, p, s, N, Kd, bias=bias)
    y = torch.zeros(N, device=cuda)
    K.gemv_q4(dev(x), dev(p), dev(s), N, Kd, y, bias=dev(bias))
    close(host(y), ref, 2e-4, 1e-4)
    # accumulate (GEMV4_ADD): y += W x
    y0 = O.normal(N, 9, 1.0)
    yt = dev(y0)
    K.gemv_q4(dev(x), dev(p), dev(s), N, Kd, yt, accumulate=True)
    ref2 = O.gemv_q4(x, p, s, N, Kd, y=y0.copy(), add=True)
    close(host(yt), ref2, 2e-4, 1e-4)


def test_gemv_q4_large_activations(cuda):
    """|x| beyond the f16 range goes through the power-of-two prescale."""
    N, Kd = 64, 2048
    W = O.normal(N * Kd, 41, 0.02).reshape(N, Kd)
    x = O.normal(Kd, 42, 1.0) * 3e5
    p, s = O.quantize_int4_group(W)
    ref = O.gemv_q4(x, p, s, N, Kd)
    y = torch.zeros(N, device=cuda)
    K.gemv_q4(dev(x), dev(p), dev(s), N, Kd, y)
    got = host(y)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


def test_gate_up_silu(cuda):
    N, Kd = 11008, 2048
    W = O.normal(2 * N * Kd, 51, 0.02).reshape(2 * N, Kd)
    x = O.normal(Kd, 52, 1.0)
    p, s = O.quantize_int4_group(W)
    ref = O.gate_up_silu(x, p, s, N, Kd)
    y = torch.zeros(N, device=cuda)
    K.gate_up_silu(dev(x), dev(p), dev(s), N, Kd, y)
    close(host(y), ref, 1e-4, 1e-3)


@pytest.mark.parametrize("N", [151936, 1000, 17])
def test_gemv_q8(cuda, N):
    Kd = 2048
    W = O.normal(N * Kd, 61, 0.02).reshape(N, Kd)
    x = O.normal(Kd, 62, 1.0)
    p, s = O.quantize_int8_rows(W)
    ref = O.gemv_q8(x, p, s, N, Kd)
    y = torch.zeros(N, device=cuda)
    K.gemv_q8(dev(x), dev(p), dev(s), N, Kd, y)
    close(host(y), ref, 1e-4, 1e-4)


@pytest.mark.parametrize("f16", [0, 1])
def test_rmsnorm(cuda, f16):
    x = O.normal(2048, 71, 2.0)
    g = O.normal(2048, 72, 0.1) + 1
    ref = O.rmsnorm(x, g, 1e-6, bool(f16))
    y = torch.zeros(2048, device=cuda)
    K.rmsnorm(dev(x), dev(g), 2048, 1e-6, f16, y)
    got = host(y)
    # rsqrt differs from a correctly rounded 1/sqrt by <= 2 ulp
    tol = 2e-3 if f16 else 1e-5
    assert np.abs(got - ref).max() <= tol * np.abs(ref).max()


@pytest.mark.parametrize("f16", [0, 1])
def test_rope_qk(cuda, f16):
    c, s = O.rope_tables(512, 128, 1e6)
    q = O.normal(2048, 81, 1.0)
    k = O.normal(256, 82, 1.0)
    for pos in (0, 1, 77, 511):
        rq, rk = O.rope_qk(q, k, 16, 2, 128, pos, c, s, bool(f16))
        tq, tk = dev(q), dev(k)
        K.rope_qk(tq, tk, 16, 2, pos, dev(c), dev(s), f16)
        assert np.array_equal(host(tq), rq) and np.array_equal(host(tk), rk)


def test_gemv_q4_stream_upload_once(cuda):
    """The upload-once GEMV (stream layout written once, then GEMV calls with
    no conversion) equals the per-call entry bit for bit, and the oracle
    within the GEMV bars; calls with PDL give the same bits."""
    N = Kd = 2048
    W = O.normal(N * Kd, 0xE6B00001, 0.02).reshape(N, Kd)
    x = O.normal(Kd, 0xE6B00002, 1.0)
    p, s = O.quantize_int4_group(W)
    ref = O.gemv_q4(x, p, s, N, Kd)
    y0 = torch.zeros(N, device=cuda)
    K.gemv_q4(dev(x), dev(p), dev(s), N, Kd, y0)
    ws = torch.zeros(K.q4_stream_bytes(N, Kd), dtype=torch.uint8, device=cuda)
    K.q4_to_stream(dev(p), dev(s), N, Kd, ws)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    xd = dev(x)
    for pdl in (False, True, True):
        y = torch.full((N,), float("nan"), device=cuda)
        K.gemv_q4_stream(xd, ws, N, Kd, y, err, pdl=pdl)
        assert torch.equal(y, y0)
    assert int(host(err)[0]) == 0
    close(host(y0), ref, 2e-4, 1e-4)


@pytest.mark.parametrize("N,Kd,T", [(2560, 2048, 16), (517, 2048, 5), (2048, 11008, 32), (128, 128, 4),
                                    (2560, 2048, 33), (517, 384, 100), (2048, 2048, 300)])
def test_gemm4_tc_and_mma_vs_oracle(cuda, N, Kd, T):
    """GEMM4 / GEMM4_ADD_T (kernels.js:389-473): T token vectors through one
    weight pass, on the tcgen05 path (tc layout) and, for T <= 16, the
    integer mma.sync path (stream layout), each row against the oracle's
    GEMV of that token; full octets, a partial last octet (N = 517) and
    split-K octets all occur.  More than 32 tokens run the whole-prompt mode
    (32-token tiles, every CTA on whole octets), ragged last tiles included."""
    W = O.normal(N * Kd, 0xE6B00101 + N, 0.02).reshape(N, Kd)
    X = O.normal(T * Kd, 0xE6B00102 + T, 1.0).reshape(T, Kd)
    bias = O.normal(N, 0xE6B00103, 0.02)
    p, s = O.quantize_int4_group(W)
    ref = np.stack([O.gemv_q4(X[t], p, s, N, Kd, bias=bias) for t in range(T)])
    ws = torch.zeros(K.q4_stream_bytes(N, Kd), dtype=torch.uint8, device=cuda)
    K.q4_to_stream(dev(p), dev(s), N, Kd, ws)
    wc = torch.zeros(K.q4_tc_bytes(N, Kd), dtype=torch.uint8, device=cuda)
    K.q4_stream_to_tc(ws, N, Kd, wc)
    paths = [True] + ([False] if T <= 16 else [])
    for tc in paths:
        y = torch.full((T, N), float("nan"), device=cuda)
        K.gemm_q4_stream(dev(X), T, wc if tc else ws, N, Kd, y, bias=dev(bias), use_tc=tc)
        close(host(y), ref, 2e-4, 1e-4)
        y0 = O.normal(T * N, 7, 1.0).reshape(T, N)
        ya = dev(y0)
        K.gemm_q4_stream(dev(X), T, wc if tc else ws, N, Kd, ya, accumulate=True, use_tc=tc)
        close(host(ya), y0 + (ref - bias), 2e-4, 1e-4)


@pytest.mark.parametrize("f16", [0, 1])
@pytest.mark.parametrize("pos,chunk", [(0, 0), (16, 0), (127, 0), (128, 0), (300, 0), (1000, 16),
                                       (4095, 0), (4095, 64), (7799, 0)])
def test_attn_decode(cuda, f16, pos, chunk):
    _attn_case(cuda, f16, pos, chunk, 16, 2, 8192 if pos >= 4096 else 4096)


@pytest.mark.parametrize("nh,nkv", [(32, 8), (16, 16), (12, 2), (24, 3)])
def test_attn_decode_gqa_shapes(cuda, nh, nkv):
    """Query groups of 4, 1, 6 and 8 heads per KV head (items of up to 4
    query heads each: partial items included)."""
    for f16, pos in [(1, 300), (0, 1000)]:
        _attn_case(cuda, f16, pos, 0, nh, nkv, 1024)


def _attn_case(cuda, f16, pos, chunk, nh, nkv, max_ctx):
    hd = 128
    c, s = O.rope_tables(max_ctx, hd, 1e6)
    ctx = pos + 1
    kc = O.normal(max_ctx * nkv * hd, 91, 1.0)
    vc = O.normal(max_ctx * nkv * hd, 92, 1.0)
    if f16:  # an f16 cache holds f16-representable values
        kc = kc.astype(np.float16).astype(np.float32)
        vc = vc.astype(np.float16).astype(np.float32)
    qkv = O.normal(nh * hd + 2 * nkv * hd, 93 + pos, 1.0)
    q, k = O.rope_qk(qkv[: nh * hd], qkv[nh * hd: nh * hd + nkv * hd], nh, nkv, hd, pos, c, s, bool(f16))
    v = qkv[nh * hd + nkv * hd:]
    kref = kc.copy().reshape(max_ctx, nkv * hd)
    vref = vc.copy().reshape(max_ctx, nkv * hd)
    kref[pos] = k
    vref[pos] = v
    # same chunking on both sides (0 = the reference's CHUNK of 128)
    ref = O.attention(q, kref[:ctx].ravel(), vref[:ctx].ravel(), nh, nkv, ctx, hd, chunk or 128, bool(f16))
    dt = torch.float16 if f16 else torch.float32
    tk = torch.from_numpy(kc).to(dt).cuda()
    tv = torch.from_numpy(vc).to(dt).cuda()
    out = torch.zeros(nh * hd, device=cuda)
    K.attn_decode(dev(qkv), tk, tv, dev(c), dev(s), nh, nkv, pos, max_ctx, f16, out, chunk=chunk)
    # The f16 variant rounds each chunk's partial output through f16 at the
    # reference's points; an f32 summation-order difference can still move
    # a value across an f16 rounding boundary (one f16 ulp, rare), hence the
    # max-abs bar; the mean stays at f32 noise.
    close(host(out), ref, 2e-5 if not f16 else 2e-3, 2e-6 if not f16 else 2e-5)
    # the new k/v row landed in the cache (f16-rounded in the f16 cache)
    krow = host(tk.float()).reshape(max_ctx, nkv * hd)[pos]
    vrow = host(tv.float()).reshape(max_ctx, nkv * hd)[pos]
    assert np.array_equal(krow, k.astype(np.float16).astype(np.float32) if f16 else k)
    assert np.array_equal(vrow, v.astype(np.float16).astype(np.float32) if f16 else v)


@pytest.mark.parametrize("f16,T,q_start,nh,nkv", [(1, 200, 0, 16, 2), (0, 200, 0, 16, 2), (1, 64, 300, 16, 2),
                                                 (0, 33, 129, 16, 2), (1, 100, 0, 32, 8), (0, 50, 10, 12, 2),
                                                 (1, 1, 0, 16, 16), (1, 517, 0, 16, 2)])
def test_attn_prefill(cuda, f16, T, q_start, nh, nkv):
    """ROPE_T + K/V rows + ATTN_PREFILL_BLOCK of one pass (kernels.js:588-618,
    684-770) against the oracle: whole prompts and later chunks (q_start > 0
    over earlier cache rows), ragged row tiles, GQA groups of 8, 4, 6 and 1.
    The tensor-core products carry f16 hi/lo splits of every f32 operand, so
    the bar is f32 noise."""
    hd, max_ctx = 128, 1024
    c, s = O.rope_tables(max_ctx, hd, 1e6)
    W = nh + 2 * nkv
    kc = O.normal(max_ctx * nkv * hd, 71, 1.0)
    vc = O.normal(max_ctx * nkv * hd, 72, 1.0)
    if f16:
        kc = kc.astype(np.float16).astype(np.float32)
        vc = vc.astype(np.float16).astype(np.float32)
    qkv = O.normal(T * W * hd, 73 + T, 1.0).reshape(T, W * hd)
    q = O.rope_t(qkv[:, : nh * hd].ravel(), T, nh, hd, q_start, c, s, bool(f16)).reshape(T, nh * hd)
    k = O.rope_t(qkv[:, nh * hd: (nh + nkv) * hd].ravel(), T, nkv, hd, q_start, c, s, bool(f16))
    v = qkv[:, (nh + nkv) * hd:]
    rnd = (lambda a: a.astype(np.float16).astype(np.float32)) if f16 else (lambda a: a)
    kref = kc.copy().reshape(max_ctx, nkv * hd)
    vref = vc.copy().reshape(max_ctx, nkv * hd)
    kref[q_start:q_start + T] = rnd(k.reshape(T, nkv * hd))
    vref[q_start:q_start + T] = rnd(v)
    ctx = q_start + T
    ref = O.attn_prefill(q, kref[:ctx].ravel(), vref[:ctx].ravel(), nh, nkv, hd, T, q_start, ctx)
    dt = torch.float16 if f16 else torch.float32
    tk = torch.from_numpy(kc).to(dt).cuda()
    tv = torch.from_numpy(vc).to(dt).cuda()
    tq = dev(qkv)
    out = torch.full((T, nh * hd), float("nan"), device=cuda)
    K.attn_prefill(tq, T, tk, tv, dev(c), dev(s), nh, nkv, q_start, max_ctx, f16, out)
    close(host(out).ravel(), ref, 3e-5, 3e-6)
    assert np.array_equal(host(tq)[:, : nh * hd], q)  # q rotated in place
    assert np.array_equal(host(tk.float()).reshape(max_ctx, -1), kref)
    assert np.array_equal(host(tv.float()).reshape(max_ctx, -1), vref)


def test_argmax_topk_ties_reference_case(cuda):
    logits = np.full(300, -5, np.float32)
    logits[1] = 7
    logits[256] = 7
    logits[129] = 6
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    K.argmax(dev(logits), 300, out)
    assert int(host(out)[0]) == 1
    ids = torch.zeros(3, dtype=torch.int32, device=cuda)
    vals = torch.zeros(3, device=cuda)
    K.topk(dev(logits), 300, 3, ids, vals)
    assert host(ids).tolist() == [1, 256, 129]
    sid = torch.tensor([10, 20, 30, 40], dtype=torch.int32, device=cuda)
    sv = torch.tensor([4.0, 3.0, 2.0, 1.0], device=cuda)
    K.sample_topk(sid, sv, 4, 1.0, 0.9, out)
    assert int(host(out)[0]) == 30


@pytest.mark.parametrize("n,k,seed", [(151936, 40, 1), (151936, 64, 2), (151936, 1, 3), (1000, 64, 4),
                                      (70, 64, 5)])
def test_topk_vs_oracle(cuda, n, k, seed):
    logits = O.normal(n, 100 + seed, 1.0)
    logits[::97] = logits[5]  # many exact ties
    rid, rv = O.topk(logits, k)
    ids = torch.zeros(k, dtype=torch.int32, device=cuda)
    vals = torch.zeros(k, device=cuda)
    K.topk(dev(logits), n, k, ids, vals)
    assert host(ids).astype(np.uint32).tolist() == rid.tolist()
    assert np.array_equal(host(vals), rv)
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    K.argmax(dev(logits), n, out)
    assert int(host(out)[0]) == O.argmax(logits)


def test_sample_vs_oracle(cuda):
    for seed in range(20):
        vals = np.sort(O.normal(40, 200 + seed, 2.0))[::-1].copy()
        ids = np.arange(1000, 1040, dtype=np.uint32)
        r = float(O.uniform(1, 300 + seed)[0])
        ref = O.sample_topk(ids, vals, 40, 0.7, r)
        out = torch.zeros(1, dtype=torch.int32, device=cuda)
        K.sample_topk(dev(ids.astype(np.int32)), dev(vals), 40, 0.7, r, out)
        assert int(host(out)[0]) == ref


def test_embed_and_lora_a(cuda):
    V, H = 1000, 2048
    W = O.normal(V * H, 301, 0.02).reshape(V, H)
    p, s = O.quantize_int8_rows(W)
    idt = torch.tensor([777], dtype=torch.int32, device=cuda)
    out = torch.zeros(H, device=cuda)
    K.embed(dev(p), dev(s), idt, H, out)
    assert np.array_equal(host(out), O.embed(p, s, 777, H))
    A = O.normal(8 * H, 302, 0.02)
    x = O.normal(H, 303, 1.0)
    d = torch.zeros(8, device=cuda)
    K.lora_a(dev(x), dev(A), H, 8, d)
    close(host(d), O.lora_a(x, A, H, 8), 1e-5, 1e-4)
