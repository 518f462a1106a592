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
def test_movement_parts_tile_the_destination(world):
    """The destination parts of every rank (movement_slab: the destination split along
    movement_shard_axis, each part read through the strided source view and stored
    compactly) put together along that axis equal the whole materialization, for a
    permutation and for a reversed axis (negative stride), as computed by the CPU
    oracle."""
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
        np_shape = list(reversed(full_l.extents_list()))
        parts, axis0 = [], None
        for rank in range(world):
            src_l, dst_l, axis, start = t4dist.movement_slab(full_l, world, rank)
            axis0 = axis if axis0 is None else axis0
            assert axis == axis0 == t4dist.movement_shard_axis(full_l)
            assert start == t4dist.shard_range(full_l.extents[axis], world, rank)[0]
            part = np.zeros(dst_l.count(), np.float32)
            assert oracle.lib().t4a_oracle_strided_to_strided(abi.F32, oracle.ptr(part), oracle.ptr(x),
                                                              ctypes.byref(src_l), ctypes.byref(dst_l), 1) == 0
            parts.append(part.reshape(list(reversed(dst_l.extents_list()))))
        np_axis = full_l.rank - 1 - axis0
        assert np.array_equal(np.concatenate(parts, axis=np_axis), whole.reshape(np_shape))


def test_movement_shard_axis_keeps_long_runs():
    """For the BASELINE config-2 permutations the shard axis is slow in both the source
    view and the destination (runs of 64^2 F32 / 16^4 C64 elements), and for the
    reversal it is the destination's slowest axis."""
    from t4a_b200 import abi

    def perm_layout(shape, perm):
        st, s = [], 1
        for e in reversed(shape):
            st.insert(0, s)
            s *= e
        return abi.numpy_layout([shape[p] for p in perm], [st[p] for p in perm])

    f32 = perm_layout([64] * 4, (3, 1, 0, 2))
    c64 = perm_layout([16] * 6, (5, 0, 4, 1, 3, 2))
    rev = abi.numpy_layout([64] * 4, [64 ** 3, 64 ** 2, -64, 1], 63 * 64)
    assert t4dist.movement_shard_axis(f32) == 2      # NumPy axis 1 of the destination
    assert t4dist.movement_shard_axis(c64) == 4      # NumPy axis 1 of the destination
    assert t4dist.movement_shard_axis(rev) == 3      # NumPy axis 0


def test_shard_view_is_a_view():
    x = torch.arange(4 * 6 * 3, dtype=torch.float32).reshape(4, 6, 3)
    for world in (1, 2, 3):
        pieces = [t4dist.shard_view(x, 1, world, r) for r in range(world)]
        assert all(p.data_ptr() >= x.data_ptr() and p.untyped_storage().data_ptr() == x.untyped_storage().data_ptr()
                   for p in pieces)
        assert torch.equal(torch.cat(pieces, dim=1), x)


# ---- row-sharded RRQR: the restatement and its exchanges ---------------------------------

def _low_rank(m, n, k, seed):
    import numpy as np
    g = np.random.default_rng(seed)
    a = g.standard_normal((m, k)) @ g.standard_normal((k, n)) + 1e-10 * g.standard_normal((m, n))
    return np.asfortranarray(a)


def _q_times_r_residual(work, coeff, perm, a):
    """|Q R - A P| / |A| for a factorization in the reference's storage (R in the upper
    triangle, reflector s below the diagonal of column s with an implicit 1, coefficient
    coeff[s]; H_s = I - coeff[s] v v^T)."""
    import numpy as np
    m, n = a.shape
    q = np.eye(m, n)
    for s in range(n - 1, -1, -1):
        v = np.zeros(m)
        v[s] = 1.0
        v[s + 1:] = work[s + 1:, s]
        q -= np.outer(v, coeff[s] * (v @ q))
    r = np.triu(work[:n, :])
    return np.linalg.norm(q @ r - a[:, perm]) / np.linalg.norm(a)


def test_sharded_rrqr_restatement_world_one_is_the_single_rrqr():
    """One rank: every combination of parts is exact, so the row-sharded restatement
    gives the single-matrix restatement's bits (matrix, permutation, coefficients)."""
    import numpy as np
    import oracle
    a = _low_rank(700, 20, 5, 1)
    w1, w2 = a.copy(order="F"), a.copy(order="F")
    p1, c1 = np.zeros(20, np.int64), np.zeros(20)
    p2, c2, piv = np.zeros(20, np.int64), np.zeros(20), np.zeros(20, np.int64)
    oracle.lib().t4a_oracle_rrqr_f64(oracle.ptr(w1.ravel(order="K")), 700, 20, 20, oracle.lptr(p1), oracle.ptr(c1),
                                     1e-8, 0.0, 1)
    st = oracle.lib().t4a_oracle_rrqr_rows_sharded_f64(oracle.ptr(w2.ravel(order="K")), 700, 20, 20, 1,
                                                       oracle.lptr(p2), oracle.ptr(c2), oracle.lptr(piv))
    assert st == 0
    assert np.array_equal(p1, p2)
    assert np.array_equal(c1.view(np.uint64), c2.view(np.uint64))
    assert np.array_equal(w1.view(np.uint64), w2.view(np.uint64))


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_sharded_rrqr_restatement_keeps_the_rank_revealing_prefix(world):
    """Several ranks round the norms and dots differently, but the pivots of the
    rank-revealing prefix (rank 6 here) are the single matrix's, and Q R = A P."""
    import numpy as np
    import oracle
    m, n, k = 1030, 24, 6
    a = _low_rank(m, n, k, 2)
    w1, w2 = a.copy(order="F"), a.copy(order="F")
    p1, c1 = np.zeros(n, np.int64), np.zeros(n)
    p2, c2, piv = np.zeros(n, np.int64), np.zeros(n), np.zeros(n, np.int64)
    oracle.lib().t4a_oracle_rrqr_f64(oracle.ptr(w1.ravel(order="K")), m, n, n, oracle.lptr(p1), oracle.ptr(c1),
                                     1e-8, 0.0, 1)
    oracle.lib().t4a_oracle_rrqr_rows_sharded_f64(oracle.ptr(w2.ravel(order="K")), m, n, n, world, oracle.lptr(p2),
                                                  oracle.ptr(c2), oracle.lptr(piv))
    assert np.array_equal(p1[:k], p2[:k])
    assert _q_times_r_residual(w2, c2, p2, a) <= 1e-8
    assert np.allclose(np.abs(np.diag(w2)[:k]), np.abs(np.diag(w1)[:k]), rtol=1e-10, atol=0)


def sharded_rrqr_worker(rank, world, port, m, n, k, result_path):
    """One rank of the row-sharded RRQR on CPU: the rank-local steps of the restatement
    (t4a_oracle_dist_*) with the two per-step exchanges done by gloo all-gathers, as the
    CUDA driver does them with NCCL."""
    import numpy as np
    import oracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        a = _low_rank(m, n, k, 3)
        r0, r1 = t4dist.shard_range(m, world, rank)
        mr = r1 - r0
        local = np.asfortranarray(a[r0:r1]).ravel(order="K").copy()
        perm = np.arange(n, dtype=np.int64)
        coeff, piv, status = np.zeros(n), np.zeros(n, np.int64), np.zeros(1, np.int64)
        lib = oracle.lib()

        def gather(x):
            parts = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(parts, x)
            return torch.cat(parts).numpy().copy()

        parts = np.zeros(n * 8)
        lib.t4a_oracle_dist_norm_parts(oracle.ptr(local), mr, n, mr, r0, 0, 0, oracle.ptr(parts))
        every = gather(torch.from_numpy(parts))
        for s in range(n):
            lib.t4a_oracle_dist_select_swap(oracle.ptr(local), mr, n, mr, r0, s, oracle.ptr(every), world,
                                            oracle.lptr(perm), oracle.ptr(coeff), oracle.lptr(piv),
                                            oracle.lptr(status))
            count = n - s - 1
            if count == 0:
                continue
            dots = np.zeros(count)
            lib.t4a_oracle_dist_dot_parts(oracle.ptr(local), mr, n, mr, r0, s, oracle.ptr(dots))
            all_dots = gather(torch.from_numpy(dots))
            lib.t4a_oracle_dist_update(oracle.ptr(local), mr, n, mr, r0, s, oracle.ptr(all_dots), world,
                                       oracle.ptr(coeff))
            if s + 1 < n:
                parts = np.zeros(count * 8)
                lib.t4a_oracle_dist_norm_parts(oracle.ptr(local), mr, n, mr, r0, s + 1, s + 1, oracle.ptr(parts))
                every = gather(torch.from_numpy(parts))
        blocks = [None] * world
        dist.all_gather_object(blocks, local)
        if rank == 0:
            full = np.zeros((m, n), order="F")
            for r in range(world):
                a0, a1 = t4dist.shard_range(m, world, r)
                full[a0:a1] = blocks[r].reshape(n, a1 - a0).T
            np.savez(result_path, work=full, perm=perm, coeff=coeff, piv=piv)
    finally:
        dist.destroy_process_group()


def test_sharded_rrqr_exchange_gloo(tmp_path):
    """Two gloo ranks exchanging norm and dot parts give the in-process restatement's
    bits (matrix, permutation, coefficients, pivots), and keep the rank-revealing
    prefix of the single matrix."""
    import numpy as np
    import oracle
    m, n, k, world = 777, 16, 5, 2
    path = str(tmp_path / "rrqr.npz")
    mp.spawn(sharded_rrqr_worker, args=(world, free_port(), m, n, k, path), nprocs=world, join=True)
    got = np.load(path)
    a = _low_rank(m, n, k, 3)
    w = a.copy(order="F")
    perm, coeff, piv = np.zeros(n, np.int64), np.zeros(n), np.zeros(n, np.int64)
    oracle.lib().t4a_oracle_rrqr_rows_sharded_f64(oracle.ptr(w.ravel(order="K")), m, n, n, world, oracle.lptr(perm),
                                                  oracle.ptr(coeff), oracle.lptr(piv))
    assert np.array_equal(got["perm"], perm) and np.array_equal(got["piv"], piv)
    assert np.array_equal(got["coeff"].view(np.uint64), coeff.view(np.uint64))
    assert np.array_equal(np.asarray(got["work"], order="F").view(np.uint64), w.view(np.uint64))
    w1, p1, c1 = a.copy(order="F"), np.zeros(n, np.int64), np.zeros(n)
    oracle.lib().t4a_oracle_rrqr_f64(oracle.ptr(w1.ravel(order="K")), m, n, n, oracle.lptr(p1), oracle.ptr(c1),
                                     1e-8, 0.0, 1)
    assert np.array_equal(p1[:k], perm[:k])
