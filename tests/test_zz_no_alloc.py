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


def _noalloc(qkv, kc, vc, c, s, pos, f16, out, chunk=0, nh=NH, nkv=NKV):
    return L.lib().eg_op_attn_decode_noalloc(
        qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(), c.data_ptr(), s.data_ptr(), nh, nkv, pos,
        MAX_CTX, int(f16), chunk, out.data_ptr(), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("f16", [1, 0])
def test_noalloc_matches_allocating_entry_two_calls(cuda, f16):
    # two calls in a row: the second reuses the static scratch the first left behind
    for pos, chunk in [(700, 0), (1500, 32)]:
        qkv, kc1, vc1, kc2, vc2, c, s = _inputs(pos, f16)
        ref = torch.zeros(NH * HD, device=cuda)
        K.attn_decode(qkv, kc1, vc1, c, s, NH, NKV, pos, MAX_CTX, f16, ref, chunk=chunk)
        got = torch.full((NH * HD,), float("nan"), device=cuda)
        assert _noalloc(qkv, kc2, vc2, c, s, pos, f16, got, chunk) == L.EG_OK, L.lib().eg_last_error()
        torch.cuda.synchronize()
        r, g = ref.cpu().numpy().astype(np.float64), got.cpu().numpy().astype(np.float64)
        d = np.abs(g - r)
        # the attention tolerance of tests/test_gpu_ops.py
        assert d.max() <= (2e-3 if f16 else 2e-5)
        assert d.mean() / np.abs(r).mean() <= (1e-3 if f16 else 1e-4)
        row = slice(pos * NKV * HD, (pos + 1) * NKV * HD)  # the appended KV row
        assert torch.equal(kc1[row], kc2[row]) and torch.equal(vc1[row], vc2[row])


def test_noalloc_rejects_oversize(cuda):
    qkv, kc, vc, _, _, c, s = _inputs(4095, 1)
    out = torch.zeros(NH * HD, device=cuda)
    # 16 heads x ceil(4096 / 16) splits = 4096 slots: the largest call that fits
    assert _noalloc(qkv, kc, vc, c, s, 4095, 1, out) == L.EG_OK
    assert _noalloc(qkv, kc, vc, c, s, 4095, 1, out, nh=32, nkv=8) == L.EG_ERR_ARG
    assert b"static scratch" in L.lib().eg_last_error()
    torch.cuda.synchronize()
