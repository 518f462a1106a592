"""The row-sharded RRQR drivers on the GPU: t4a_dist_rrqr (exchanges as NCCL
all-gathers) and t4a_dist_rrqr_p2p (exchanges fused into the step kernels, stores into
every rank's memory over NVLink).

* One rank (no process group): each driver equals the single-GPU driver t4a_rrqr bit
  for bit -- matrix, permutation, coefficients, pivots -- because every combination of
  parts is exact with one part.
* Two ranks (two GPUs, one process each): each driver equals the CPU restatement of the
  row-sharded algorithm (oracle t4a_oracle_rrqr_rows_sharded_f64) bit for bit, keeps the
  single matrix's pivots over the rank-revealing prefix, and Q R = A P to 1e-8 |A|.  The
  NVLink driver runs twice on one exchange region (call ordering) with the same bits.
"""
import ctypes
import datetime
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
import t4a_b200 as t4
from t4a_b200 import abi
from t4a_b200 import dist as t4dist

pytestmark = pytest.mark.gpu


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def low_rank(m, n, k, seed):
    g = np.random.default_rng(seed)
    a = g.standard_normal((m, k)) @ g.standard_normal((k, n)) + 1e-10 * g.standard_normal((m, n))
    return np.asfortranarray(a)


def colmajor(a, device):
    """A CUDA flat column-major copy of a Fortran-ordered array."""
    return torch.from_numpy(np.asarray(a, order="F").ravel(order="K").copy()).to(device)


def run_sharded(local, m, n, row0, steps, dtype=torch.float64, exchange="p2p", comm=None):
    dev = local.device
    perm = torch.empty(n, dtype=torch.int64, device=dev)
    coeff = torch.zeros(max(steps, 1), dtype=dtype, device=dev)
    piv = torch.zeros(max(steps, 1), dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int64, device=dev)
    drv = t4dist.RrqrRowsSharded(local, m, n, row0, steps, comm=comm, exchange=exchange)
    try:
        drv.run(t4.stream_handle(), perm, coeff, piv, status)
        torch.cuda.synchronize()
    finally:
        drv.close()
    return perm, coeff, piv, status


@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
@pytest.mark.parametrize("m,n,k,dtype", [(4096, 48, 12, torch.float64), (3001, 40, 9, torch.float64),
                                         (70000, 64, 16, torch.float64), (4096, 32, 8, torch.float32)])
def test_world_of_one_equals_the_single_gpu_driver(cuda, m, n, k, dtype, exchange):
    a = low_rank(m, n, k, m + n)
    if dtype == torch.float32:
        a = np.asfortranarray(a.astype(np.float32))
    w_single = colmajor(a, cuda)
    w_shard = w_single.clone()
    perm1, coeff1, piv1, st1 = t4.rrqr(w_single.view(n, m).t(), n)
    perm2, coeff2, piv2, st2 = run_sharded(w_shard, m, n, 0, n, dtype, exchange)
    assert int(st1.item()) == 0 and int(st2.item()) == 0
    assert torch.equal(perm1, perm2) and torch.equal(piv1[:n], piv2[:n])
    ib = torch.int64 if dtype == torch.float64 else torch.int32
    assert torch.equal(coeff1[:n].view(ib), coeff2[:n].view(ib))
    assert torch.equal(w_single.view(ib), w_shard.view(ib))


def worker(rank, world, port, m, n, k):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        dev = torch.device("cuda", rank)
        a = low_rank(m, n, k, 7)
        r0, r1 = t4dist.shard_range(m, world, rank)
        # every driver run on a fresh copy of this rank's rows: NCCL, then the NVLink
        # driver twice on one exchange region; all must give the same bits
        results = []
        p2p = t4dist.P2pComm(n)
        try:
            for exchange, comm in (("nccl", None), ("p2p", p2p), ("p2p", p2p)):
                loc = colmajor(a[r0:r1], dev)
                perm, coeff, piv, status = run_sharded(loc, m, n, r0, n, exchange=exchange, comm=comm)
                assert int(status.item()) == 0, (exchange, int(status.item()))
                results.append((loc, perm, coeff, piv))
        finally:
            p2p.close()
        local, perm, coeff, piv = results[0]
        for loc, pp, cc, vv in results[1:]:
            assert torch.equal(loc.view(torch.int64), local.view(torch.int64))
            assert torch.equal(pp, perm) and torch.equal(vv, piv)
            assert torch.equal(cc.view(torch.int64), coeff.view(torch.int64))
        full = t4dist.gather_rows_colmajor(local, m, n, r0).cpu().numpy().reshape(n, m).T
        # the CPU restatement of the same sharding, bit for bit
        want = a.copy(order="F")
        wp, wc, wv = np.zeros(n, np.int64), np.zeros(n), np.zeros(n, np.int64)
        oracle.lib().t4a_oracle_rrqr_rows_sharded_f64(oracle.ptr(want.ravel(order="K")), m, n, n, world,
                                                      oracle.lptr(wp), oracle.ptr(wc), oracle.lptr(wv))
        assert np.array_equal(perm.cpu().numpy(), wp)
        assert np.array_equal(piv.cpu().numpy()[:n], wv)
        assert np.array_equal(coeff.cpu().numpy()[:n].view(np.uint64), wc.view(np.uint64))
        assert np.array_equal(np.ascontiguousarray(full).view(np.uint64), np.ascontiguousarray(want).view(np.uint64))
        # the single matrix's pivots over the rank-revealing prefix, and Q R = A P
        single = colmajor(a, dev)
        p1, _, _, _ = t4.rrqr(single.view(n, m).t(), n)
        assert torch.equal(p1[:k].cpu(), perm[:k].cpu())
        wfull = torch.from_numpy(np.asfortranarray(full).ravel(order="K").copy()).to(dev).view(n, m).t()
        q, qst = t4.rrqr_form_q(wfull, coeff[:n])
        r = torch.triu(wfull[:n, :])
        ad = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        resid = (torch.linalg.norm(q @ r - ad[:, perm]) / torch.linalg.norm(ad)).item()
        assert int(qst.item()) == 0 and resid <= 1e-8, resid
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


def test_two_gpus_match_the_sharded_restatement(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(worker, args=(2, free_port(), 8192, 64, 16), nprocs=2, join=True)
