"""Host logic of the multi-GPU composition (t4a_b200.dist) on CPU: the row partition,
and the sharded scatter_add's exchange over world_size-2 gloo ranks, with a CPU stand-in
for the per-rank CUDA step (injected; the product default is the CUDA kernel)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from t4a_b200 import dist as t4dist


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n", [0, 1, 7, 8, 64, 1000, 4194304])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_range_partitions(n, world):
    ranges = [t4dist.shard_range(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1 and sorted(sizes, reverse=True) == sizes


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        t4dist.shard_range(10, 2, 2)


def rank_batch(rank, rows, cols, n):
    g = torch.Generator().manual_seed(100 + rank)
    idx = torch.randint(0, rows, (n,), generator=g)
    upd = torch.randn(n, cols, generator=g, dtype=torch.float64)
    return idx, upd


def cpu_add(partial, idx, upd, workspace):
    partial.index_add_(0, idx, upd)


def scatter_worker(rank, world, port):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        rows, cols, n = 12, 3, 40
        operand = torch.arange(rows * cols, dtype=torch.float64).reshape(rows, cols)
        idx, upd = rank_batch(rank, rows, cols, n)
        partial = t4dist.scatter_partial(operand)
        assert torch.equal(partial, operand if rank == 0 else torch.zeros_like(operand))
        shard = t4dist.scatter_add_rows_sharded(partial, idx, upd, local_add=cpu_add)
        assert shard.shape == (rows // world, cols)
        shards = [torch.empty_like(shard) for _ in range(world)]
        dist.all_gather(shards, shard)
        want = operand.clone()
        for r in range(world):
            i, u = rank_batch(r, rows, cols, n)
            want.index_add_(0, i, u)
        assert torch.allclose(torch.cat(shards), want, rtol=0, atol=1e-12)
        with pytest.raises(ValueError):
            t4dist.scatter_add_rows_sharded(torch.zeros(13, cols, dtype=torch.float64), idx, upd,
                                            local_add=cpu_add)
    finally:
        dist.destroy_process_group()


def test_scatter_add_sharded_exchange_gloo():
    mp.spawn(scatter_worker, args=(2, free_port()), nprocs=2, join=True)
