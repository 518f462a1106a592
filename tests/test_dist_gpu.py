"""The multi-GPU composition on 2 GPUs (NCCL): sharded gather and reduction equal the
single-GPU results bit for bit; the sharded scatter_add (per-rank CUDA scatter into a
partial destination, then one reduce-scatter) equals the oracle sum of every rank's
updates within the F64 tolerance (1e-12 relative to max(|x|, 1))."""
import ctypes
import datetime
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_batch(rank, rows, cols, n):
    g = torch.Generator().manual_seed(1000 + rank)
    idx = torch.randint(0, rows, (n,), generator=g)
    upd = torch.randn(n, cols, generator=g, dtype=torch.float64)
    return idx, upd


def worker(rank, world, port):
    import t4a_b200 as t4
    from t4a_b200 import abi
    from t4a_b200 import dist as t4dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        dev = torch.device("cuda", rank)
        g = torch.Generator().manual_seed(7)
        # scatter_add: every rank's batch into one destination, rows owned by slices
        rows, cols, n = 4096, 128, 200000
        operand = torch.randn(rows, cols, generator=g, dtype=torch.float64)
        idx, upd = rank_batch(rank, rows, cols, n)
        partial = t4dist.scatter_partial(operand.to(dev))
        d_idx, d_upd = idx.to(dev), upd.to(dev)
        ws = t4.scatter_rows_workspace(partial, d_idx, d_upd)
        ws.zero_()
        shard = t4dist.scatter_add_rows_sharded(partial, d_idx, d_upd, workspace=ws)
        shards = [torch.empty_like(shard) for _ in range(world)]
        dist.all_gather(shards, shard)
        got = torch.cat(shards).cpu().numpy()
        want = operand.numpy().copy()
        for r in range(world):
            i, u = rank_batch(r, rows, cols, n)
            np.add.at(want, i.numpy(), u.numpy())
        err = np.abs(got - want) / np.maximum(np.abs(want), 1.0)
        assert err.max() <= 1e-12, err.max()
        # gather: index batches sharded, table replicated
        table = torch.randn(rows, cols, generator=g, dtype=torch.float32).to(dev)
        gidx = torch.randint(0, rows, (10000,), generator=g).to(dev)
        mine = t4dist.gather_rows_sharded(table, gidx)
        outs = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(outs, mine)
        assert torch.equal(torch.cat(outs), table[gidx])
        # reduction: slabs of a non-reduced axis
        x = torch.randn(64, 300, 32, generator=g, dtype=torch.float32).to(dev)
        slab = t4dist.reduce_sharded(t4dist.shard_view(x, 0, world, rank), 1, abi.SUM)
        full = t4.reduce(x, 1, abi.SUM)
        start, stop = t4dist.shard_range(64, world, rank)
        assert torch.equal(slab.view(torch.int32), full[start:stop].contiguous().view(torch.int32))
        # the same over a strided slab (axis 1 sharded, axis 0 reduced), no copy of the slab
        slab0 = t4dist.reduce_sharded(t4dist.shard_view(x, 1, world, rank), 0, abi.MAX)
        full0 = t4.reduce(x, 0, abi.MAX)
        s1, e1 = t4dist.shard_range(300, world, rank)
        assert torch.equal(slab0.view(torch.int32), full0[:, s1:e1].contiguous().view(torch.int32))
        # movement: destination slabs along the slowest axis from strided source views
        src = torch.randn(16, 12, 10, 8, generator=g, dtype=torch.float32).to(dev)
        view = src.permute(3, 1, 0, 2)
        full_l = t4.tensor_layout(view)
        want = view.contiguous()
        _, dst_l, axis, start = t4dist.movement_slab(full_l, world, rank)
        out = torch.empty(dst_l.count(), dtype=torch.float32, device=dev)
        t4dist.materialize_slab(t4.stream_handle(), abi.F32, ctypes.c_void_p(out.data_ptr()),
                                ctypes.c_void_p(src.data_ptr()), full_l, src.numel(), world, rank)
        np_axis = full_l.rank - 1 - axis
        part = want.narrow(np_axis, start, dst_l.extents[axis])
        assert torch.equal(out.view(part.shape), part.contiguous())
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


def test_sharded_ops_two_gpus(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(worker, args=(2, free_port()), nprocs=2, join=True)
