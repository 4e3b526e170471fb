"""The vocab-split LM head of one stream over several GPUs (parallel.py):
vocabulary slicing, the candidate merge (value desc, ties to the lower id,
NaN never wins -- ARGMAX kernels.js:771-784) and the all-gather merge with
world_size-2 gloo ranks on CPU; on a GPU, shards computed by
eg_lm_head_shard merge to the single-GPU argmax."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vibethinker_webgpu_lora_b200 import parallel as P


@pytest.mark.parametrize("vocab,world", [(151936, 2), (151936, 8), (5000, 3), (17, 4)])
def test_vocab_slices_cover_once_and_align(vocab, world):
    got = [P.vocab_slice(vocab, r, world) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == vocab
    for (a0, a1), (b0, _) in zip(got, got[1:]):
        assert a1 == b0
    assert all(r0 % 16 == 0 for r0, _ in got)


def test_merge_order_ties_and_nan():
    assert P.merge_argmax([1.0, 3.0, 3.0], [5, 9, 7]) == (3.0, 7)       # tie -> lower id
    assert P.merge_argmax([float("nan"), 0.5], [1, 2]) == (0.5, 2)       # NaN never wins
    assert P.merge_argmax([-2.0, -1.0], [0, 100]) == (-1.0, 100)


def test_merge_topk_is_the_global_topk_order():
    rng = np.random.default_rng(3)
    logits = rng.standard_normal(3000).astype(np.float32).round(1)  # many ties
    world, k = 3, 40
    vals, ids = [], []
    for r in range(world):
        r0, r1 = P.vocab_slice(len(logits), r, world)
        order = sorted(range(r0, r1), key=lambda i: (-logits[i], i))[:k]
        vals.append([logits[i] for i in order])
        ids.append(order)
    got_v, got_i = P.merge_topk(vals, ids, k)
    want = sorted(range(len(logits)), key=lambda i: (-logits[i], i))[:k]
    assert got_i == want and got_v == [logits[i] for i in want]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, ws, port, logits, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        r0, r1 = P.vocab_slice(len(logits), rank, ws)
        shard = torch.tensor(logits[r0:r1])
        i = int(torch.argmax(shard))  # first maximum = lowest id on ties
        v, gid = P.gather_merge(shard[i], torch.tensor(r0 + i), None)
        with open(os.path.join(outdir, f"rank{rank}"), "w") as f:
            f.write(f"{gid}")
    finally:
        dist.destroy_process_group()


def test_gather_merge_gloo_matches_global_argmax(tmp_path):
    rng = np.random.default_rng(7)
    logits = rng.standard_normal(1000).astype(np.float32)
    logits[[123, 777]] = 5.0  # a tie across the two ranks' slices: the lower id wins
    ws = 2
    mp.spawn(_rank, args=(ws, _free_port(), logits, str(tmp_path)), nprocs=ws, join=True)
    for r in range(ws):
        assert int((tmp_path / f"rank{r}").read_text()) == 123


def _rank_topk(rank, ws, port, logits, k, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        r0, r1 = P.vocab_slice(len(logits), rank, ws)
        order = sorted(range(r0, r1), key=lambda i: (-logits[i], i))[:k]
        v = torch.tensor([logits[i] for i in order], dtype=torch.float32)
        i = torch.tensor(order, dtype=torch.int32)
        gv = [torch.empty_like(v) for _ in range(ws)]
        gi = [torch.empty_like(i) for _ in range(ws)]
        dist.all_gather(gv, v)
        dist.all_gather(gi, i)
        _, mi = P.merge_topk([g.tolist() for g in gv], [g.tolist() for g in gi], k)
        with open(os.path.join(outdir, f"rank{rank}"), "w") as f:
            f.write(",".join(map(str, mi)))
    finally:
        dist.destroy_process_group()


def test_topk_all_gather_merge_gloo(tmp_path):
    """k = 40 candidates per rank, all-gathered over two gloo ranks, merge to
    the global TOPK_SELECT order on every rank (ties across the slice
    boundary go to the lower id)."""
    rng = np.random.default_rng(11)
    logits = rng.standard_normal(2000).astype(np.float32).round(1)
    ws, k = 2, 40
    mp.spawn(_rank_topk, args=(ws, _free_port(), logits, k, str(tmp_path)), nprocs=ws, join=True)
    want = sorted(range(len(logits)), key=lambda i: (-logits[i], i))[:k]
    for r in range(ws):
        assert [int(x) for x in (tmp_path / f"rank{r}").read_text().split(",")] == want


@pytest.mark.gpu
def test_lm_head_shards_topk_sample_equal_single_gpu(cuda):
    """Three shards of the LM head on one GPU (as three ranks would run them):
    local TOPK_SELECT with global ids, concatenation in rank order, the
    device merge and SAMPLE_TOPK give the single-GPU topKLogits(40) and
    sampleToken for several r."""
    import ctypes as C

    import vibethinker_webgpu_lora_b200 as E
    from vibethinker_webgpu_lora_b200 import _lib as L
    from vibethinker_webgpu_lora_b200 import kernels as K
    from vibethinker_webgpu_lora_b200.config import small_config
    from oracle import oracle as O

    cfg = small_config(layers=2, vocab=5000)
    rt = E.QwenB200(cfg, {"maxCtx": 64}).build("synthetic", seed=0xE6B00000)
    for t, tok in enumerate(O.token_ids(6, 5, cfg["vocabSize"])):
        rt.token(int(tok), t)
    want = rt.topKLogits(40)
    hidden = torch.from_numpy(rt.readHidden()).to(cuda)
    cv, ci = [], []
    for rank in range(3):
        r0, r1 = P.vocab_slice(cfg["vocabSize"], rank, 3)
        lg = torch.empty(r1 - r0, device=cuda)
        v = torch.empty(1, device=cuda)
        i = torch.empty(1, dtype=torch.int32, device=cuda)
        L.check(L.lib().eg_lm_head_shard(rt.handle, C.c_void_p(hidden.data_ptr()), r0, r1 - r0,
                                         C.c_void_p(lg.data_ptr()), C.c_void_p(v.data_ptr()),
                                         C.c_void_p(i.data_ptr()), None))
        ids = torch.empty(40, dtype=torch.int32, device=cuda)
        vals = torch.empty(40, device=cuda)
        K.topk(lg, r1 - r0, 40, ids, vals)
        cv.append(vals)
        ci.append(ids + r0)
    mids, mvals = P.topk_merge_device(torch.cat(cv), torch.cat(ci), 40)
    torch.cuda.synchronize()
    assert mids.cpu().tolist() == [w["id"] for w in want]
    assert mvals.cpu().tolist() == [w["logit"] for w in want]
    out = torch.empty(1, dtype=torch.int32, device=cuda)
    for r in (0.0, 0.3, 0.77, 1.0):
        K.sample_topk(mids, mvals, 40, 0.7, r, out)
        assert int(out.item()) == rt.sampleToken(0.7, r)


@pytest.mark.gpu
def test_lm_head_shards_merge_to_the_full_argmax(cuda):
    """Shards of the LM head computed on one GPU (as each rank would) merge to
    the single-GPU argmax and reproduce its logits."""
    import ctypes as C

    import vibethinker_webgpu_lora_b200 as E
    from vibethinker_webgpu_lora_b200 import _lib as L
    from vibethinker_webgpu_lora_b200.config import small_config
    from oracle import oracle as O

    cfg = small_config(layers=2, vocab=5000)
    rt = E.QwenB200(cfg, {"maxCtx": 64}).build("synthetic", seed=0xE6B00000)
    for t, tok in enumerate(O.token_ids(6, 3, cfg["vocabSize"])):
        rt.token(int(tok), t)
    full = rt.readLogits()
    want = rt.argmaxLogits()
    hidden = torch.from_numpy(rt.readHidden()).to(cuda)
    vals, ids = [], []
    got_logits = torch.empty(cfg["vocabSize"], device=cuda)
    for rank in range(3):
        r0, r1 = P.vocab_slice(cfg["vocabSize"], rank, 3)
        v = torch.empty(1, device=cuda)
        i = torch.empty(1, dtype=torch.int32, device=cuda)
        L.check(L.lib().eg_lm_head_shard(
            rt.handle, C.c_void_p(hidden.data_ptr()), r0, r1 - r0,
            C.c_void_p(got_logits[r0:].data_ptr()), C.c_void_p(v.data_ptr()),
            C.c_void_p(i.data_ptr()), None))
        torch.cuda.synchronize()
        vals.append(v.item())
        ids.append(i.item())
        assert r0 <= ids[-1] < r1
    assert P.merge_argmax(vals, ids)[1] == want
    np.testing.assert_allclose(got_logits.cpu().numpy(), full, rtol=0, atol=1e-5)
