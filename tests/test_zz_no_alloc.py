"""The allocation-free attention entry point (eg_op_attn_decode_noalloc),
called through the C ABI, must give the allocating entry point's results.

It exists for callers that cannot allocate device memory at call time: a
host framework whose caching allocator has already reserved the GPU's memory
(a new cudaMalloc could fail or make that allocator release its cache), and
latency-critical loops that cannot accept cudaMalloc's implicit
synchronisation.  This file is collected last so that a failing run that stops
at the first failure has already run every other test."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from vibethinker_webgpu_lora_b200 import _lib as L
from vibethinker_webgpu_lora_b200 import kernels as K

pytestmark = pytest.mark.gpu

NH, NKV, HD, MAX_CTX = 16, 2, 128, 4096


def _inputs(pos, f16):
    c, s = O.rope_tables(MAX_CTX, HD, 1e6)
    kc = O.normal(MAX_CTX * NKV * HD, 501, 1.0)
    vc = O.normal(MAX_CTX * NKV * HD, 502, 1.0)
    qkv = O.normal(NH * HD + 2 * NKV * HD, 503 + pos, 1.0)
    dt = torch.float16 if f16 else torch.float32
    mk = lambda a: torch.from_numpy(a).to(dt).cuda()  # noqa: E731
    return (torch.from_numpy(qkv).cuda(), mk(kc), mk(vc), mk(kc), mk(vc),
            torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda())


def _noalloc(qkv, kc, vc, c, s, pos, f16, out, chunk=0, nh=NH, nkv=NKV, stream=None):
    st = stream if stream is not None else torch.cuda.current_stream()
    return L.lib().eg_op_attn_decode_noalloc(
        qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(), c.data_ptr(), s.data_ptr(), nh, nkv, pos,
        MAX_CTX, int(f16), chunk, out.data_ptr(), st.cuda_stream)


def _compare(ref, got, f16):
    torch.cuda.synchronize()
    r, g = ref.cpu().numpy().astype(np.float64), got.cpu().numpy().astype(np.float64)
    d = np.abs(g - r)
    # same kernel, same inputs: only the scratch differs, so the results agree
    # far inside the attention tolerance of tests/test_gpu_ops.py
    assert d.max() <= (2e-3 if f16 else 2e-5)
    assert d.mean() / np.abs(r).mean() <= (2e-5 if f16 else 2e-6)


@pytest.mark.parametrize("f16", [1, 0])
def test_noalloc_matches_allocating_entry_two_calls(cuda, f16):
    # two calls in a row: the second reuses the static scratch the first left behind
    for pos, chunk in [(700, 0), (1500, 32)]:
        qkv, kc1, vc1, kc2, vc2, c, s = _inputs(pos, f16)
        ref = torch.zeros(NH * HD, device=cuda)
        K.attn_decode(qkv, kc1, vc1, c, s, NH, NKV, pos, MAX_CTX, f16, ref, chunk=chunk)
        got = torch.full((NH * HD,), float("nan"), device=cuda)
        assert _noalloc(qkv, kc2, vc2, c, s, pos, f16, got, chunk) == L.EG_OK, L.lib().eg_last_error()
        _compare(ref, got, f16)
        row = slice(pos * NKV * HD, (pos + 1) * NKV * HD)  # the appended KV row
        assert torch.equal(kc1[row], kc2[row]) and torch.equal(vc1[row], vc2[row])


def test_noalloc_limits_and_largest_call(cuda):
    """The size check counts the splits the kernel really makes (128 keys
    when chunk = 0): 32 query heads over 8 KV heads at pos 4095 take 32 x 32
    slots and are accepted; the largest accepted call (16 heads x 256
    splits of 16 keys = all 4096 slots) matches the allocating entry, on a
    stream other than the current one; one more slot is refused."""
    nh, nkv = 32, 8
    c, s = O.rope_tables(MAX_CTX, HD, 1e6)
    qkv = torch.from_numpy(O.normal(nh * HD + 2 * nkv * HD, 611, 1.0)).cuda()
    kc = O.normal(MAX_CTX * nkv * HD, 612, 1.0)
    vc = O.normal(MAX_CTX * nkv * HD, 613, 1.0)
    mk = lambda a: torch.from_numpy(a).to(torch.float16).cuda()  # noqa: E731
    tc, ts = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
    ref = torch.zeros(nh * HD, device=cuda)
    K.attn_decode(qkv, mk(kc), mk(vc), tc, ts, nh, nkv, 4095, MAX_CTX, 1, ref)
    got = torch.full((nh * HD,), float("nan"), device=cuda)
    assert _noalloc(qkv, mk(kc), mk(vc), tc, ts, 4095, 1, got, 0, nh, nkv) == L.EG_OK, \
        L.lib().eg_last_error()
    _compare(ref, got, 1)

    qkv, kc1, vc1, kc2, vc2, c, s = _inputs(4095, 1)
    ref = torch.zeros(NH * HD, device=cuda)
    K.attn_decode(qkv, kc1, vc1, c, s, NH, NKV, 4095, MAX_CTX, 1, ref, chunk=16)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    got = torch.full((NH * HD,), float("nan"), device=cuda)
    side.wait_stream(torch.cuda.current_stream())
    assert _noalloc(qkv, kc2, vc2, c, s, 4095, 1, got, 16, stream=side) == L.EG_OK
    side.synchronize()
    _compare(ref, got, 1)

    # 64 heads x 256 splits of 16 keys: past the 4096 slots
    big = torch.zeros(64 * HD + 2 * 8 * HD, device=cuda)
    out = torch.zeros(64 * HD, device=cuda)
    kc8 = torch.zeros(MAX_CTX * 8 * HD, dtype=torch.float16, device=cuda)
    assert _noalloc(big, kc8, kc8, c, s, 4095, 1, out, 16, nh=64, nkv=8) == L.EG_ERR_ARG
    assert b"static scratch" in L.lib().eg_last_error()
    torch.cuda.synchronize()
