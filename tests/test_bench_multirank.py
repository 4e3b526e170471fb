"""The multi-GPU bench plumbing (one process per GPU, replicas, whole-job
throughput from the slowest rank's device time), exercised with world_size 2
gloo ranks on CPU."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, ws, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        local_ms = [120.0, 150.0][rank]  # rank 1 is the slow one
        ms = bench.max_over_ranks(local_ms, ws, torch.device("cpu"))
        with open(os.path.join(outdir, f"rank{rank}"), "w") as f:
            f.write(f"{ms} {bench.job_throughput(ws, 1000, ms)}")
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_job_throughput_gloo(tmp_path):
    ws = 2
    mp.spawn(_rank, args=(ws, _free_port(), str(tmp_path)), nprocs=ws, join=True)
    for r in range(ws):
        ms, tput = map(float, (tmp_path / f"rank{r}").read_text().split())
        assert ms == 150.0                   # every rank sees the max
        assert tput == pytest.approx(2 * 1000 / 0.150)


def test_single_rank_is_identity():
    assert bench.max_over_ranks(42.0, 1, torch.device("cpu")) == 42.0
    assert bench.job_throughput(1, 10, 1000.0) == 10.0


def test_positions_cycle_inside_the_window():
    got = bench.positions(32, 128, 300, 32)
    assert sum(k for _, k in got) == 300
    for p, k in got:
        assert 32 <= p and p + k <= 32 + 128


@pytest.mark.parametrize("ws", [1, 2, 4, 8, 3])
def test_batch16_sequences_shard_once(ws):
    got = [bench.shard_sequences(16, r, ws) for r in range(ws)]
    assert sum(got, []) == list(range(16))
    assert max(map(len, got)) - min(map(len, got)) <= 1
