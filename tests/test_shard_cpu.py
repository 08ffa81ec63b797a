"""Host-side logic of the multi-GPU run, on CPU with the gloo backend and
world_size 2: the (batch, head) / row split covers every unit exactly once,
and the timing reduction takes the slowest rank."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


@pytest.mark.parametrize("n", [1, 7, 32, 512, 65536])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_partition(n, world):
    spans = [bench.shard(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_flop_convention():
    # 4 * D * S(S+1)/2 per slice; config 3 totals 2.1996 TFLOP.
    total = 16 * 32 * bench.attn_flops_per_slice(4096, 128, True)
    assert abs(total / 1e12 - 2.1996) < 1e-3
    assert bench.attn_flops_per_slice(128, 64, False) == 4 * 64 * 128 * 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = bench.shard(512, world, rank)
        t = torch.tensor([float(10 + rank)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        cnt = torch.tensor([float(hi - lo)], dtype=torch.float64)
        dist.all_reduce(cnt, op=dist.ReduceOp.SUM)
        out[rank] = (t.item(), cnt.item())
    finally:
        dist.destroy_process_group()


def test_two_rank_reduction_gloo():
    world = 2
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        assert res[r] == (11.0, 512.0)
