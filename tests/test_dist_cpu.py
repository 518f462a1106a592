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


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_movement_slabs_tile_the_destination(world):
    """The destination slabs of every rank (movement_slab: the slowest destination axis
    split, each slab read through the strided source view) put together equal the whole
    materialization, for a permutation and for a reversed axis (negative stride), as
    computed by the CPU oracle."""
    import ctypes
    import numpy as np
    import oracle
    from t4a_b200 import abi
    rng = np.random.default_rng(5)
    x = rng.standard_normal((8, 6, 5, 7)).astype(np.float32)
    cases = []
    st = [s // 4 for s in x.strides]
    perm = (3, 1, 0, 2)
    cases.append(abi.numpy_layout([x.shape[p] for p in perm], [st[p] for p in perm]))
    cases.append(abi.numpy_layout(list(x.shape), [st[0], st[1], -st[2], st[3]], (x.shape[2] - 1) * st[2]))
    for full_l in cases:
        whole = np.zeros(x.size, np.float32)
        assert oracle.lib().t4a_oracle_strided_to_strided(abi.F32, oracle.ptr(whole), oracle.ptr(x),
                                                          ctypes.byref(full_l),
                                                          ctypes.byref(abi.layout(full_l.extents_list())), 1) == 0
        parts = []
        for rank in range(world):
            src_l, dst_l, start = t4dist.movement_slab(full_l, world, rank)
            assert start == t4dist.shard_range(full_l.extents[full_l.rank - 1], world, rank)[0]
            part = np.zeros(dst_l.count(), np.float32)
            assert oracle.lib().t4a_oracle_strided_to_strided(abi.F32, oracle.ptr(part), oracle.ptr(x),
                                                              ctypes.byref(src_l), ctypes.byref(dst_l), 1) == 0
            parts.append(part)
        assert np.array_equal(np.concatenate(parts), whole)


def test_shard_view_is_a_view():
    x = torch.arange(4 * 6 * 3, dtype=torch.float32).reshape(4, 6, 3)
    for world in (1, 2, 3):
        pieces = [t4dist.shard_view(x, 1, world, r) for r in range(world)]
        assert all(p.data_ptr() >= x.data_ptr() and p.untyped_storage().data_ptr() == x.untyped_storage().data_ptr()
                   for p in pieces)
        assert torch.equal(torch.cat(pieces, dim=1), x)
