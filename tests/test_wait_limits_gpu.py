"""Bounded waits on the GPU.

The kernels that stage data with bulk copies -- the RRQR column engine (fused driver,
Q formation, the engine forms of column_norms / reflector / apply_reflector) and the
scatter_add fold -- wait on mbarriers a bounded number of rounds.  A wait that runs out
stops the block's remaining staged work, reports it (RRQR: bit 1 of the status word;
primitives: bit 1 of t4a_rrqr_primitive_faults; scatter_add: the workspace's status word
set to 1), and the block still waits, with a separate limit, for every copy in flight
before it exits.

libt4a_waitzero.so is those kernels built with the staged-data wait limit set to zero
rounds, so that every such wait runs out at once (nothing is left waiting: the limit is
zero, not a flag that nobody sets).  Each test checks the report, then runs the same
operation through the regular library to show that the context is still healthy."""
import ctypes
import os

import numpy as np
import pytest
import torch

import t4a_b200 as t4
from t4a_b200 import abi

pytestmark = pytest.mark.gpu

P, I, LL, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_size_t
LP = ctypes.POINTER(abi.Layout)


def waitzero():
    lib = ctypes.CDLL(os.path.join(t4.MODULE_DIR, "libt4a_waitzero.so"))
    lib.t4a_rrqr.argtypes = [P, I, P, LP, LL, LL, P, P, P, P, P, SZ]
    lib.t4a_rrqr_form_q.argtypes = [P, I, P, LP, LL, P, LP, LL, P, LP, LL, P]
    lib.t4a_scatter_add.argtypes = [P, I, I, P, LP, LL, P, LP, LL, P, LP, LL, ctypes.POINTER(abi.ScatterPlan), P, SZ]
    lib.t4a_launch_column_norms.argtypes = [ctypes.POINTER(t4.Launch), P, P, P, I, abi.Layout, abi.Layout, LL]
    lib.t4a_rrqr_primitive_faults.argtypes = [ctypes.POINTER(ctypes.c_ulonglong)]
    return lib


def vp(t):
    return ctypes.c_void_p(t.data_ptr())


def low_rank(m, n, k, device):
    g = torch.Generator(device="cpu").manual_seed(3)
    a = torch.randn(m, k, generator=g, dtype=torch.float64) @ torch.randn(k, n, generator=g, dtype=torch.float64)
    return a.t().contiguous().to(device)  # [n, m]: the transpose of a column-major [m, n]


def test_rrqr_wait_that_runs_out_sets_status_bit_1(cuda):
    lib = waitzero()
    m, n = 8192, 16
    colmajor = low_rank(m, n, 4, cuda)
    work = colmajor.clone()
    layout = abi.layout([m, n], [1, m])
    nbytes = t4.rrqr_workspace_bytes(abi.F64, layout)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
    perm = torch.empty(n, dtype=torch.int64, device=cuda)
    coeff = torch.zeros(n, dtype=torch.float64, device=cuda)
    piv = torch.zeros(n, dtype=torch.int64, device=cuda)
    status = torch.zeros(1, dtype=torch.int64, device=cuda)
    assert lib.t4a_rrqr(t4.stream_handle(), abi.F64, vp(work), ctypes.byref(layout), m * n, n, vp(perm), vp(coeff),
                        vp(piv), vp(status), vp(ws), nbytes) == 0
    torch.cuda.synchronize()
    assert int(status.item()) & 2, "a wait that ran out must set bit 1"
    # Q formation on the engine reports the same way
    q = torch.empty((n, m), dtype=torch.float64, device=cuda).t()
    qst = torch.zeros(1, dtype=torch.int64, device=cuda)
    ql, cl = abi.layout([m, n], [1, m]), abi.layout([n])
    assert lib.t4a_rrqr_form_q(t4.stream_handle(), abi.F64, vp(work), ctypes.byref(layout), m * n, vp(coeff),
                               ctypes.byref(cl), n, vp(q), ctypes.byref(ql), m * n, vp(qst)) == 0
    torch.cuda.synchronize()
    assert int(qst.item()) & 2
    # the context is healthy: the regular library factorizes the same matrix cleanly
    again = colmajor.clone()
    _, _, _, st = t4.rrqr(again.view(n, m).t(), n)
    torch.cuda.synchronize()
    assert int(st.item()) == 0


def test_engine_primitive_wait_that_runs_out_is_reported(cuda):
    lib = waitzero()
    m, n = 8192, 8
    colmajor = low_rank(m, n, 8, cuda)
    wl, nl = abi.layout([m, n], [1, m]), abi.layout([n])
    plan = t4.plan_rrqr("column_norms", abi.F64, wl, m * n, nl, n, 0)
    assert plan.variant == 66  # the engine form
    norms = torch.full((n,), 7.0, dtype=torch.float64, device=cuda)
    faults = ctypes.c_ulonglong(0)
    assert lib.t4a_rrqr_primitive_faults(ctypes.byref(faults)) == 0  # cleared
    assert lib.t4a_launch_column_norms(ctypes.byref(plan), t4.stream_handle(), vp(colmajor), vp(norms), abi.F64, wl,
                                       nl, 0) == 0
    torch.cuda.synchronize()
    assert lib.t4a_rrqr_primitive_faults(ctypes.byref(faults)) == 0
    assert faults.value & 2
    assert lib.t4a_rrqr_primitive_faults(ctypes.byref(faults)) == 0 and faults.value == 0  # reading cleared it
    # the regular library: no fault, the norms of the columns
    t4.launch_rrqr("column_norms", plan, t4.stream_handle(), vp(colmajor), vp(norms), ctypes.c_int(abi.F64), wl, nl,
                   ctypes.c_longlong(0))
    torch.cuda.synchronize()
    assert t4.rrqr_primitive_faults() == 0
    want = torch.linalg.norm(colmajor.view(n, m), dim=1)
    assert torch.allclose(norms, want, rtol=1e-12)


def test_scatter_fold_wait_that_runs_out_sets_the_status_word(cuda):
    lib = waitzero()
    rows, cols, count = 4096, 32, 20000
    g = torch.Generator(device="cpu").manual_seed(5)
    idx = torch.randint(0, rows, (count,), generator=g).to(cuda)
    upd = torch.randn(count, cols, generator=g, dtype=torch.float64).to(cuda)
    dest = torch.zeros(rows, cols, dtype=torch.float64, device=cuda)
    ws = t4.scatter_rows_workspace(dest, idx, upd)
    ws.fill_(7)
    plan = abi.scatter_plan([0], [0], [1], 1, 2, 2)
    ol, il, ul = abi.numpy_layout([rows, cols]), abi.layout([count, 1]), abi.numpy_layout([count, cols])
    assert lib.t4a_scatter_add(t4.stream_handle(), abi.F64, abi.I64, vp(dest), ctypes.byref(ol), rows * cols, vp(idx),
                               ctypes.byref(il), count, vp(upd), ctypes.byref(ul), count * cols, ctypes.byref(plan),
                               vp(ws), ws.numel()) == 0
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 1, "a fold wait that ran out must set the status word"
    # the regular library adds every update
    dest.zero_()
    ws.zero_()
    t4.scatter_add_rows(dest, idx, upd, workspace=ws)
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 0
    want = torch.zeros_like(dest).index_add_(0, idx, upd)
    assert torch.allclose(dest, want, rtol=0, atol=1e-12)
