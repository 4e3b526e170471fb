"""Multi-GPU pieces of the decode path.

Replicas (one process per GPU, each with the full 1.79 GB model, independent
sequences, no collective) are the unit of scale for many streams; bench.py
runs them.  For ONE stream the only step that splits is the LM head: every rank owns a slice of the vocabulary, the rank that ran the layers
broadcasts the 8 KB hidden state, each rank runs the final RMSNorm, its
slice of the int8 LM head and a local argmax with global ids
(``eg_lm_head_shard``), the ranks all-gather their (value, id) pairs and each
merges them with the reference's selection order -- larger value first, ties
to the lower id (ARGMAX, kernels.js:771-784) -- which reproduces the
single-GPU argmax exactly.  Sampling (top-k, temperature, r) splits the
same way: each rank selects its slice's top k with global ids, the ranks
all-gather the k (value, id) pairs, the concatenation (rank order) is
reduced to the global top k by the TOPK_SELECT kernel itself -- rank slices
are ordered by id, so "lower position" is "lower id" among equal values --
and every rank runs SAMPLE_TOPK with the shared r (runtime.js:1648-1732).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib as L


def vocab_slice(vocab: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [r0, r1) of the vocabulary owned by `rank`: contiguous, 16-row
    aligned (one LM-head tile), covering the vocabulary exactly once."""
    tiles = (vocab + 15) // 16
    t0, t1 = tiles * rank // world, tiles * (rank + 1) // world
    return 16 * t0, min(16 * t1, vocab)


def merge_argmax(vals, ids) -> tuple[float, int]:
    """Merge per-rank (value, id) candidates: larger value wins, ties go to
    the lower id; NaN never wins (the reference's `beats`)."""
    best_v, best_i = float("-inf"), None
    for v, i in zip(vals, ids):
        v, i = float(v), int(i)
        if v != v:  # NaN
            continue
        if best_i is None or v > best_v or (v == best_v and i < best_i):
            best_v, best_i = v, i
    return best_v, best_i


def gather_merge(best_val: torch.Tensor, best_id: torch.Tensor, group=None) -> tuple[float, int]:
    """All-gather every rank's (value, id) (one f64 pair per rank: an int32 id
    is exact in f64) and merge them; every rank gets the same answer."""
    world = dist.get_world_size(group)
    pair = torch.stack([best_val.to(torch.float64).reshape(()),
                        best_id.to(torch.float64).reshape(())])
    out = [torch.empty_like(pair) for _ in range(world)]
    dist.all_gather(out, pair, group=group)
    return merge_argmax([o[0].item() for o in out], [o[1].item() for o in out])


def merge_topk(vals_per_rank, ids_per_rank, k: int):
    """The global top-k of the ranks' candidate lists in the reference's
    TOPK_SELECT order (value descending, ties to the lower id, NaN and values
    at or below -1e30 never taken), as (values, ids).  Host restatement of the
    device merge, for tests."""
    cand = [(float(v), int(i)) for vs, iz in zip(vals_per_rank, ids_per_rank)
            for v, i in zip(vs, iz) if v == v and float(v) > -1e30]
    cand.sort(key=lambda p: (-p[0], p[1]))
    cand = cand[:k]
    return [c[0] for c in cand], [c[1] for c in cand]


def topk_merge_device(cat_vals: torch.Tensor, cat_ids: torch.Tensor, k: int, stream=None):
    """Global top-k of the concatenated per-rank candidate lists (each list in
    TOPK_SELECT order, lists in rank = vocabulary order) with the library's
    TOPK_SELECT kernel: returns (ids, vals) device tensors of length k."""
    from . import kernels as K
    pos = torch.empty(k, dtype=torch.int32, device=cat_vals.device)
    vals = torch.empty(k, dtype=torch.float32, device=cat_vals.device)
    K.topk(cat_vals, int(cat_vals.numel()), k, pos, vals, stream=stream)
    return cat_ids[pos.long()], vals


class VocabSplitLmHead:
    """The vocab-split LM head of one stream over the ranks of `group`; `rt`
    is this rank's QwenB200 (the full model, built the same way everywhere)."""

    def __init__(self, rt, group=None):
        self.rt = rt
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.r0, self.r1 = vocab_slice(rt.cfg["vocabSize"], self.rank, self.world)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.hidden = torch.empty(rt.cfg["hiddenSize"], dtype=torch.float32, device=dev)
        self.val = torch.empty(1, dtype=torch.float32, device=dev)
        self.idx = torch.empty(1, dtype=torch.int32, device=dev)
        self.rt_stream = torch.cuda.ExternalStream(rt.stream, device=dev)

    def argmax(self, hidden: torch.Tensor | None = None, src: int = 0) -> int:
        """Greedy next token of the stream whose last hidden state `src` holds
        (`hidden` on rank src; ignored elsewhere)."""
        cur = torch.cuda.current_stream()
        cur.wait_stream(self.rt_stream)  # the runtime's decode wrote hidden / owns the scratch
        if self.rank == src and hidden is not None:
            self.hidden.copy_(hidden)
        dist.broadcast(self.hidden, src=src, group=self.group)
        stream = cur.cuda_stream
        L.check(L.lib().eg_lm_head_shard(
            self.rt.handle, C.c_void_p(self.hidden.data_ptr()), self.r0, self.r1 - self.r0,
            None, C.c_void_p(self.val.data_ptr()), C.c_void_p(self.idx.data_ptr()),
            C.c_void_p(stream)))
        return gather_merge(self.val, self.idx, self.group)[1]

    def sample(self, k: int, temp: float, r: float, hidden: torch.Tensor | None = None,
               src: int = 0) -> int:
        """sampleToken(temp, r) of the stream (topKLogits(k) + SAMPLE_TOPK,
        runtime.js:1648-1732) over the vocab-split head: every rank returns
        the same id."""
        from . import kernels as K
        cur = torch.cuda.current_stream()
        cur.wait_stream(self.rt_stream)
        if self.rank == src and hidden is not None:
            self.hidden.copy_(hidden)
        dist.broadcast(self.hidden, src=src, group=self.group)
        rows = self.r1 - self.r0
        if not hasattr(self, "logits") or self.logits.numel() != rows:
            self.logits = torch.empty(rows, dtype=torch.float32, device=self.hidden.device)
        L.check(L.lib().eg_lm_head_shard(
            self.rt.handle, C.c_void_p(self.hidden.data_ptr()), self.r0, rows,
            C.c_void_p(self.logits.data_ptr()), C.c_void_p(self.val.data_ptr()),
            C.c_void_p(self.idx.data_ptr()), C.c_void_p(cur.cuda_stream)))
        ids = torch.empty(k, dtype=torch.int32, device=self.hidden.device)
        vals = torch.empty(k, dtype=torch.float32, device=self.hidden.device)
        K.topk(self.logits, rows, k, ids, vals)
        ids += self.r0  # global ids
        gv = [torch.empty_like(vals) for _ in range(self.world)]
        gi = [torch.empty_like(ids) for _ in range(self.world)]
        dist.all_gather(gv, vals, group=self.group)
        dist.all_gather(gi, ids, group=self.group)
        mids, mvals = topk_merge_device(torch.cat(gv), torch.cat(gi), k)
        out = torch.empty(1, dtype=torch.int32, device=self.hidden.device)
        K.sample_topk(mids, mvals, k, temp, r, out)
        return int(out.item())


def measure(steps: int = 200, warmup: int = 20) -> dict | None:
    """Per-token time of the vocab-split LM head of the 3B model on the
    ranks of the default group against the whole LM head on one GPU, both
    ending in the greedy id on the host.  Run under torchrun (NCCL); rank 0
    returns the result, timed with CUDA events, max over ranks."""
    from .config import QWEN25_3B
    from .runtime import QwenB200

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    rt = QwenB200(QWEN25_3B, {"maxCtx": 64, "device": dev.index}).build("synthetic", seed=0xE6B00000)
    g = torch.Generator().manual_seed(1)
    hidden = torch.randn(QWEN25_3B["hiddenSize"], generator=g).to(dev)
    head = VocabSplitLmHead(rt, None)
    stream = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(warmup):
            fn()
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / steps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    split_ms = timed(lambda: head.argmax(hidden, 0))
    ids = [head.argmax(hidden, 0)]

    def single():
        L.check(L.lib().eg_lm_head_shard(
            rt.handle, C.c_void_p(hidden.data_ptr()), 0, QWEN25_3B["vocabSize"], None,
            C.c_void_p(head.val.data_ptr()), C.c_void_p(head.idx.data_ptr()),
            C.c_void_p(stream.cuda_stream)))
        return int(head.idx.item())

    one_ms = timed(single)
    ids.append(single())
    rt.close()
    if rank:
        return None
    return {"what": "vocab-split LM head, one stream", "n_gpus": world,
            "split_ms_per_token": split_ms, "single_gpu_ms_per_token": one_ms,
            "speedup": one_ms / split_ms, "same_id": ids[0] == ids[1]}


if __name__ == "__main__":
    import json
    import os

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    r = measure()
    if r is not None:
        print(json.dumps(r), flush=True)
    dist.destroy_process_group()
