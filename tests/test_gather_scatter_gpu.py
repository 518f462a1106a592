"""GPU parity of gather (bit-exact) and scatter_add (within the stated tolerance)
against the CPU oracle.

Cases mirror the reference's tests/gpu_gather_scatter.rs (independent reference,
middle index vector, clamped starts on a strided operand, scalar output with float
indices, large output domain, two window dims with reversed offsets, strided
destinations with holes, bool data, scatter collisions, complex updates with index
vectors, windows that do not fit, zero updates), BASELINE config 4 at reduced size
(row gather from an F32 table with I64 indices; F64 scatter with Zipf(1.1) indices),
the reference bench's column-major table, and random plans over every data and index
dtype.  Every case runs through this library's launchers (scatter: the one-kernel path and the
two-kernel path with a workspace), its exported module symbols
(planner geometry and the reference's flat geometry, grid ceil(len/256) x 256) and the
reference's own kernels rebuilt from source (oracle/_ref).

Scatter tolerance (written here, from the reference's close_sum, bench_kernels.rs:398):
|got - want| <= tol * magnitude + atol per component, magnitude = |operand| + sum of
|update| landing there; tol = 1e-12 (F64, C64) or 1e-5 (F32, C32), atol = 1e-6 for
F32/C32 and 1e-300 for F64/C64.
"""
import ctypes
import os

import numpy as np
import pytest

import oracle
import t4a_b200 as t4
from cuda_module import Module
from t4a_b200 import abi

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OUR_CUBIN = os.path.join(ROOT, "t4a-cuda-kernels_b200", "t4a_b200", "lib", "gather_scatter.cubin")
REF_CUBIN = os.path.join(ROOT, "oracle", "_ref", "gather_scatter.cubin")
SENTINEL, GUARD = 0xCD, 256
THREADS = os.cpu_count() or 4
ESIZE = {abi.F32: 4, abi.F64: 8, abi.I32: 4, abi.I64: 8, abi.BOOL: 1, abi.C32: 8, abi.C64: 16}
INDEX_NP = {abi.F32: np.float32, abi.F64: np.float64, abi.I32: np.int32, abi.I64: np.int64}
COMPONENT_NP = {abi.F32: np.float32, abi.F64: np.float64, abi.C32: np.float32, abi.C64: np.float64}
TOL = {abi.F32: (1e-5, 1e-6), abi.C32: (1e-5, 1e-6), abi.F64: (1e-12, 1e-300), abi.C64: (1e-12, 1e-300)}
ROUTES = ["launcher", "module", "module-refgeom", "reference"]

_MODULES = {}


def module(path):
    if path not in _MODULES:
        if not os.path.exists(path):
            pytest.skip(f"{os.path.basename(path)} not built")
        _MODULES[path] = Module(path)
    return _MODULES[path]


def dev(buf):
    import torch
    return torch.from_numpy(np.frombuffer(bytearray(buf), dtype=np.uint8).copy()).cuda()


def sentinel(nbytes):
    import torch
    return torch.full((nbytes + GUARD,), SENTINEL, dtype=torch.uint8, device="cuda")


def take(t, nbytes):
    host = t.cpu().numpy()
    assert (host[nbytes:] == SENTINEL).all(), "a store landed past the destination"
    return host[:nbytes]


def span_of(l):
    hi = l.offset + sum((e - 1) * s for e, s in zip(l.extents_list(), l.strides_list()) if s > 0 and e > 0)
    return hi + 1


def vptr(t):
    return ctypes.c_void_p(t.data_ptr())


# ---- gather ---------------------------------------------------------------------

class Gather:
    def __init__(self, dtype, index_dtype, operand, operand_l, indices, indices_l, plan, out_l, out_elems=None):
        self.dtype, self.index_dtype = dtype, index_dtype
        self.operand = np.ascontiguousarray(operand).view(np.uint8).ravel()
        self.operand_l = operand_l
        self.indices = np.ascontiguousarray(indices, dtype=INDEX_NP[index_dtype])
        self.indices_l = indices_l
        self.plan = plan
        self.out_l = out_l
        self.out_elems = out_elems if out_elems is not None else span_of(out_l)

    @property
    def es(self):
        return ESIZE[self.dtype]

    def oracle(self):
        out = np.full(self.out_elems * self.es, SENTINEL, dtype=np.uint8)
        rc = oracle.lib().t4a_oracle_gather(self.dtype, self.index_dtype, oracle.ptr(out), oracle.ptr(self.operand),
                                            oracle.ptr(self.indices.view(np.uint8)), ctypes.byref(self.out_l),
                                            ctypes.byref(self.operand_l), ctypes.byref(self.indices_l),
                                            ctypes.byref(self.plan), THREADS)
        assert rc == 0
        return out

    def gpu(self, route):
        import torch
        op_len = len(self.operand) // self.es
        idx_len = self.indices.size
        d_op = dev(self.operand)
        d_idx = dev(self.indices.view(np.uint8)) if idx_len else torch.zeros(16, dtype=torch.uint8, device="cuda")
        d_out = sentinel(self.out_elems * self.es)
        if route == "launcher":
            t4.gather_raw(t4.stream_handle(), self.dtype, self.index_dtype, vptr(d_out), self.out_l, self.out_elems,
                          vptr(d_op), self.operand_l, op_len, vptr(d_idx), self.indices_l, idx_len, self.plan)
        else:
            launch, count = t4.plan_gather(self.dtype, self.index_dtype, self.out_l, self.out_elems,
                                           self.operand_l, op_len, self.indices_l, idx_len, self.plan)
            if route == "module":
                mod = module(OUR_CUBIN)
                geom = (tuple(launch.grid), tuple(launch.block), launch.shared_bytes)
            else:
                mod = module(OUR_CUBIN if route == "module-refgeom" else REF_CUBIN)
                geom = ((max(1, (count + 255) // 256),), (256,), 0)
            if count > 0 and launch.grid[0] > 0:
                mod.launch("t4a_cuda_gather", *geom, [
                    vptr(d_out), vptr(d_op), vptr(d_idx), ctypes.c_int(self.dtype), ctypes.c_int(self.index_dtype),
                    self.out_l, self.operand_l, self.indices_l, self.plan, ctypes.c_longlong(count)])
        torch.cuda.synchronize()
        return take(d_out, self.out_elems * self.es)

    def check(self, routes=ROUTES):
        want = self.oracle()
        for route in routes:
            got = self.gpu(route)
            assert np.array_equal(want, got), route


def gplan(window_dims, offset_dims, start_map, slices, ivd, out_rank):
    return abi.gather_plan(window_dims, offset_dims, start_map, slices, ivd, out_rank)


def test_gather_independent_reference(cuda):
    # Operand [4, 3] (axis 0 fastest), axis 0 collapsed; indices [2, 1].
    op = np.arange(12, dtype=np.float64) * 0.5 - 2.0
    Gather(abi.F64, abi.I64, op, abi.layout([4, 3]), np.array([2, 0]), abi.layout([2, 1]),
           gplan([1], [1], [0], [1, 3], 1, 2), abi.layout([2, 3])).check()


def test_gather_middle_index_vector(cuda):
    op = (np.arange(24) % 11).astype(np.float64) - 5.0
    idx = np.array([2, 0, 0, 1, 1, 3, 1, 2, 2, 2, 0, 0])
    Gather(abi.F64, abi.I64, op, abi.layout([3, 4, 2]), idx, abi.layout([2, 2, 3]),
           gplan([1], [0], [0, 2], [1, 2, 1], 1, 3), abi.layout([2, 2, 3])).check()


def test_gather_clamps_starts_on_a_strided_operand(cuda):
    buf = (np.arange(40) % 17).astype(np.float64) * 0.25
    Gather(abi.F64, abi.I64, buf, abi.layout([2, 6], [16, 1], 3), np.array([-9, 100, 2]), abi.layout([3, 1]),
           gplan([1], [1], [0], [1, 3], 1, 2), abi.layout([3, 3])).check()


@pytest.mark.parametrize("index_dtype", [abi.F32, abi.F64])
def test_gather_scalar_output_float_indices(cuda, index_dtype):
    op = np.arange(5, dtype=np.float64) + 0.5
    for start in [3.0, 3.9, -0.5, 7.2, np.inf, -np.inf, np.nan, 1e30]:
        Gather(abi.F64, index_dtype, op, abi.layout([5]), np.array([start]), abi.layout([1]),
               gplan([], [], [0], [1], 0, 0), abi.layout([])).check()


def test_gather_large_output_domain(cuda):
    outputs, rows, cols = 1 << 16, 512, 8
    op = np.arange(rows * cols, dtype=np.float32)
    idx = (np.arange(outputs) * 7) % rows
    Gather(abi.F32, abi.I64, op, abi.layout([rows, cols]), idx, abi.layout([outputs]),
           gplan([1], [1], [0], [1, cols], 1, 2), abi.layout([outputs, cols])).check()


def test_gather_two_window_dims_reversed_offsets(cuda):
    op = (np.arange(60) % 23).astype(np.float64) * 0.5
    idx = np.array([0, 0, 2, 1, 1, 3, 0, 2])
    Gather(abi.F64, abi.I64, op, abi.layout([3, 4, 5]), idx, abi.layout([4, 2]),
           gplan([0, 2], [2, 0], [0, 1], [2, 1, 3], 1, 3), abi.layout([3, 4, 2])).check()


def test_gather_strided_destination_keeps_holes(cuda):
    op = np.arange(6, dtype=np.float32) + 1.5
    Gather(abi.F32, abi.I64, op, abi.layout([2, 3]), np.array([1, 0]), abi.layout([2, 1]),
           gplan([1], [1], [0], [1, 3], 1, 2), abi.layout([2, 3], [1, 4], 2), out_elems=14).check()


def test_gather_bool_data(cuda):
    rng = np.random.default_rng(5)
    op = rng.integers(0, 2, size=64, dtype=np.uint8)
    idx = rng.integers(-2, 10, size=24)
    Gather(abi.BOOL, abi.I32, op, abi.layout([8, 8]), idx, abi.layout([24]),
           gplan([1], [1], [0], [1, 8], 1, 2), abi.layout([24, 8])).check()


@pytest.mark.parametrize("index_dtype", [abi.I64, abi.I32, abi.F32, abi.F64])
def test_gather_config4_rows(cuda, index_dtype):
    """BASELINE config 4a shape at reduced size: row-major F32 table [rows, 128],
    one start per gathered row (uniform, plus out-of-range starts)."""
    rng = np.random.default_rng(40 + index_dtype)
    rows, cols, n = 4096, 128, 50_000
    table = rng.standard_normal(rows * cols).astype(np.float32)
    idx = rng.integers(0, rows, size=n)
    idx[:64] = rng.integers(-1000, rows + 1000, size=64)
    Gather(abi.F32, index_dtype, table, abi.numpy_layout([rows, cols]), idx, abi.layout([n, 1]),
           gplan([0], [0], [1], [cols, 1], 1, 2), abi.numpy_layout([n, cols])).check()


def test_gather_reference_bench_layout(cuda):
    """The reference bench's own plan (examples/bench_kernels.rs:1649-1690): a table
    [rows, cols] with rows fastest, so every gathered window is strided."""
    rng = np.random.default_rng(41)
    rows, cols, n = 1000, 256, 1024
    table = rng.standard_normal(rows * cols).astype(np.float32)
    idx = rng.integers(0, rows, size=n).astype(np.int32)
    Gather(abi.F32, abi.I32, table, abi.layout([rows, cols]), idx, abi.layout([n, 1]),
           gplan([1], [1], [0], [1, cols], 1, 2), abi.layout([n, cols])).check()


def random_strided(rng, ext):
    """A strided view over `ext` (axis 0 fastest): padded rows, an offset and maybe
    one reversed axis.  Returns (layout, span in elements)."""
    st, s = [], 1
    for i, e in enumerate(ext):
        st.append(s)
        s *= e + (int(rng.integers(0, 3)) if i == 0 else 0)
    off = int(rng.integers(0, 4))
    if ext and rng.random() < 0.3:
        a = int(rng.integers(0, len(ext)))
        if ext[a] > 1:
            off += (ext[a] - 1) * st[a]
            st[a] = -st[a]
    l = abi.layout(ext, st, off)
    return l, span_of(l)


def random_indices(rng, ext_idx, high, index_dtype):
    n = int(np.prod(ext_idx)) if ext_idx else 1
    vals = rng.integers(-3, high + 4, size=n)
    if index_dtype in (abi.F32, abi.F64):
        vals = vals + rng.random(n) * (rng.random(n) < 0.3)
    return vals


def random_gather(rng, dtype, index_dtype):
    r = int(rng.integers(1, 5))
    ext = [int(rng.integers(1, 7)) for _ in range(r)]
    win = [a for a in range(r) if rng.random() < 0.6]
    rng.shuffle(win)
    slices = [1] * r
    for a in win:
        slices[a] = int(rng.integers(1, ext[a] + 1))
    k = int(rng.integers(0, r + 1))
    start_map = [int(a) for a in rng.permutation(r)[:k]]
    nb = int(rng.integers(0, 3))
    bext = [int(rng.integers(1, 6)) for _ in range(nb)]
    if k == 1 and rng.random() < 0.3:
        ivd, iext = nb, list(bext)
    else:
        ivd = int(rng.integers(0, nb + 1))
        iext = bext[:ivd] + [k] + bext[ivd:]
    out_rank = nb + len(win)
    offset_dims = [int(a) for a in rng.permutation(out_rank)[:len(win)]]
    out_ext, b = [0] * out_rank, 0
    for q, a in enumerate(win):
        out_ext[offset_dims[q]] = slices[a]
    for ax in range(out_rank):
        if ax not in offset_dims:
            out_ext[ax] = bext[b]
            b += 1
    op_l, op_span = random_strided(rng, ext)
    operand = rng.integers(0, 256, size=op_span * ESIZE[dtype], dtype=np.uint8)
    if rng.random() < 0.5:
        out_l, out_elems = abi.layout(out_ext), None
    else:
        out_l, out_elems = random_strided(rng, out_ext)
        if any(s < 0 for s in out_l.strides_list()):
            out_l, out_elems = abi.layout(out_ext), None
    idx = random_indices(rng, iext, max(ext), index_dtype)
    plan = gplan(win, offset_dims, start_map, slices, ivd, out_rank)
    return Gather(dtype, index_dtype, operand, op_l, idx, abi.layout(iext), plan, out_l, out_elems)


@pytest.mark.parametrize("dtype", [abi.BOOL, abi.F32, abi.F64, abi.I32, abi.I64, abi.C32, abi.C64])
@pytest.mark.parametrize("index_dtype", [abi.I64, abi.F32])
def test_gather_random_plans(cuda, dtype, index_dtype):
    rng = np.random.default_rng(1000 + 10 * dtype + index_dtype)
    for _ in range(25):
        random_gather(rng, dtype, index_dtype).check()


# ---- scatter_add ------------------------------------------------------------------

class Scatter:
    def __init__(self, dtype, index_dtype, dest, dest_l, indices, indices_l, updates, updates_l, plan):
        self.dtype, self.index_dtype = dtype, index_dtype
        self.comp = COMPONENT_NP[dtype]
        self.dest = np.ascontiguousarray(dest).view(self.comp).ravel().copy()
        self.dest_l = dest_l
        self.indices = np.ascontiguousarray(indices, dtype=INDEX_NP[index_dtype])
        self.indices_l = indices_l
        self.updates = np.ascontiguousarray(updates).view(self.comp).ravel().copy()
        self.updates_l = updates_l
        self.plan = plan

    @property
    def es(self):
        return ESIZE[self.dtype]

    def _oracle(self, dest, updates):
        out = dest.copy()
        rc = oracle.lib().t4a_oracle_scatter_add(self.dtype, self.index_dtype, oracle.ptr(out),
                                                 oracle.ptr(self.indices.view(np.uint8)), oracle.ptr(updates),
                                                 ctypes.byref(self.dest_l), ctypes.byref(self.indices_l),
                                                 ctypes.byref(self.updates_l), ctypes.byref(self.plan), THREADS)
        assert rc == 0
        return out

    def gpu(self, route):
        import torch
        comps = self.es // np.dtype(self.comp).itemsize
        dest_len = self.dest.size // comps
        upd_len = self.updates.size // comps
        idx_len = self.indices.size
        d_out = sentinel(self.dest.nbytes)
        d_out[:self.dest.nbytes] = dev(self.dest.view(np.uint8))
        d_upd = dev(self.updates.view(np.uint8)) if upd_len else torch.zeros(16, dtype=torch.uint8, device="cuda")
        d_idx = dev(self.indices.view(np.uint8)) if idx_len else torch.zeros(16, dtype=torch.uint8, device="cuda")
        if route in ("launcher", "launcher-ws"):
            ws, nbytes = None, 0
            if route == "launcher-ws":
                nbytes = t4.scatter_add_workspace_bytes(self.dtype, self.index_dtype, self.dest_l, self.indices_l,
                                                        self.updates_l, self.plan)
                d_ws = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device="cuda")
                ws = vptr(d_ws)
            t4.scatter_add_raw(t4.stream_handle(), self.dtype, self.index_dtype, vptr(d_out), self.dest_l, dest_len,
                               vptr(d_idx), self.indices_l, idx_len, vptr(d_upd), self.updates_l, upd_len, self.plan,
                               ws, nbytes)
        else:
            launch = t4.plan_scatter_add(self.dtype, self.index_dtype, self.dest_l, dest_len, self.indices_l,
                                         idx_len, self.updates_l, upd_len, self.plan)
            count = self.updates_l.count()
            if route == "module":
                mod = module(OUR_CUBIN)
                geom = (tuple(launch.grid), tuple(launch.block), launch.shared_bytes)
            else:
                mod = module(OUR_CUBIN if route == "module-refgeom" else REF_CUBIN)
                geom = ((max(1, (count + 255) // 256),), (256,), 0)
            if count > 0 and self.dest_l.count() > 0 and (route != "module" or launch.grid[0] > 0):
                mod.launch("t4a_cuda_scatter_add", *geom, [
                    vptr(d_out), vptr(d_idx), vptr(d_upd), ctypes.c_int(self.dtype), ctypes.c_int(self.index_dtype),
                    self.dest_l, self.indices_l, self.updates_l, self.plan, ctypes.c_longlong(count)])
        torch.cuda.synchronize()
        if route == "launcher-ws":
            assert int(d_ws[:4].view(torch.int32).item()) == 0, "a bulk copy wait ran out"
        return take(d_out, self.dest.nbytes).view(self.comp)

    def check(self, routes=ROUTES + ["launcher-ws"]):
        want = self._oracle(self.dest, self.updates)
        mag = self._oracle(np.abs(self.dest), np.abs(self.updates))
        tol, atol = TOL[self.dtype]
        for route in routes:
            got = self.gpu(route)
            same = (got == want) | (np.abs(got - want) <= tol * mag + atol)
            bad = np.flatnonzero(~same)
            assert bad.size == 0, (route, bad[:8], got[bad[:8]], want[bad[:8]])


def splan(window_dims, update_window_dims, scatter_dims, ivd, operand_rank, updates_rank):
    return abi.scatter_plan(window_dims, update_window_dims, scatter_dims, ivd, operand_rank, updates_rank)


def test_scatter_independent_reference(cuda):
    Scatter(abi.F64, abi.I64, np.ones(6), abi.layout([6]), np.array([0, 1, 5, 4]), abi.layout([4]),
            np.arange(8) + 0.25, abi.layout([4, 2]), splan([0], [1], [0], 1, 1, 2)).check()


def test_scatter_complex_index_vectors(cuda):
    dest = np.arange(12) - 1j * np.arange(12)
    upd = 0.5 * (np.arange(2) + 1.0) - 1j * np.arange(2)
    Scatter(abi.C64, abi.I64, dest.astype(np.complex128), abi.layout([3, 4]), np.array([0, 2, 1, 3]),
            abi.layout([2, 2]), upd.astype(np.complex128), abi.layout([2]), splan([], [], [0, 1], 1, 2, 1)).check()


def test_scatter_skips_windows_that_do_not_fit(cuda):
    Scatter(abi.F64, abi.I64, np.full(6, 2.0), abi.layout([6]), np.array([0, 5]), abi.layout([2, 1]),
            np.ones(14), abi.layout([2, 7]), splan([0], [1], [0], 1, 1, 2)).check()


def test_scatter_zero_updates(cuda):
    Scatter(abi.F64, abi.I64, np.arange(3.0), abi.layout([3]), np.zeros(0), abi.layout([0]),
            np.zeros(0), abi.layout([0]), splan([], [], [0], 1, 1, 1)).check()


def test_scatter_collisions_large_domain(cuda):
    count, dests = 1 << 16, 64
    idx = np.arange(count) % dests
    upd = (np.arange(count) % 5).astype(np.float64)
    Scatter(abi.F64, abi.I64, np.zeros(dests), abi.layout([dests]), idx, abi.layout([count]), upd,
            abi.layout([count]), splan([], [], [0], 1, 1, 1)).check()


def test_scatter_two_window_dims_reversed(cuda):
    rng = np.random.default_rng(7)
    dest = rng.standard_normal(4 * 5 * 3)
    idx = np.array([0, 1, 2, 0, 1, 1])
    upd = rng.standard_normal(3 * 2 * 2)  # updates [3 (window on dest axis 2), 2 (batch), 2 (window on axis 0)]
    Scatter(abi.F64, abi.I64, dest, abi.layout([4, 5, 3]), idx, abi.layout([2, 3]), upd,
            abi.layout([3, 2, 2]), splan([2, 0], [0, 2], [0, 1, 2], 1, 3, 3)).check()


def test_scatter_strided_destination_keeps_holes(cuda):
    rng = np.random.default_rng(8)
    dest = rng.standard_normal(20).astype(np.float32)
    Scatter(abi.F32, abi.I32, dest, abi.layout([2, 3], [1, 5], 3), np.array([1, 0, 1]), abi.layout([3, 1]),
            rng.standard_normal(9).astype(np.float32), abi.layout([3, 3]), splan([1], [1], [0], 1, 2, 2)).check()


def zipf_rows(rng, n, rows, s=1.1):
    """Zipf(s) over ranks 1..rows by inverse CDF, row = rank - 1."""
    w = np.arange(1, rows + 1, dtype=np.float64) ** -s
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    return np.minimum(np.searchsorted(cdf, rng.random(n), side="right"), rows - 1)


@pytest.mark.parametrize("dtype", [abi.F64, abi.F32, abi.C32, abi.C64])
def test_scatter_config4_zipf_rows(cuda, dtype):
    """BASELINE config 4b shape at reduced size: row-major destination [rows, 128],
    update rows with Zipf(1.1) destinations (heavy collisions on the first rows)."""
    rng = np.random.default_rng(50 + dtype)
    rows, cols, n = 2048, 128, 20_000
    comp = COMPONENT_NP[dtype]
    k = 2 if dtype in (abi.C32, abi.C64) else 1
    dest = rng.standard_normal(rows * cols * k).astype(comp)
    upd = rng.standard_normal(n * cols * k).astype(comp)
    idx = zipf_rows(rng, n, rows)
    Scatter(dtype, abi.I64, dest, abi.numpy_layout([rows, cols]), idx, abi.layout([n, 1]), upd,
            abi.numpy_layout([n, cols]), splan([0], [0], [1], 1, 2, 2)).check()


def test_scatter_one_hot_row(cuda):
    """Every update lands on one row (the worst collision case)."""
    rng = np.random.default_rng(9)
    rows, cols, n = 16, 96, 30_000
    Scatter(abi.F64, abi.I32, np.zeros(rows * cols), abi.numpy_layout([rows, cols]), np.full(n, 3),
            abi.layout([n, 1]), rng.standard_normal(n * cols), abi.numpy_layout([n, cols]),
            splan([0], [0], [1], 1, 2, 2)).check()


def test_scatter_reference_bench_slots(cuda):
    """The reference bench's scatter (examples/bench_kernels.rs:1747-1800), scaled:
    scalar updates into 16 slots, indices (i*7 + i/3) % 16."""
    n = 200_000
    i = np.arange(n)
    idx = ((i * 7 + i // 3) % 16).astype(np.int32)
    rng = np.random.default_rng(10)
    Scatter(abi.F32, abi.I32, np.arange(16, dtype=np.float32), abi.layout([16]), idx, abi.layout([n, 1]),
            rng.random(n).astype(np.float32), abi.layout([n]), splan([], [], [0], 1, 1, 1)).check()


def random_scatter(rng, dtype, index_dtype):
    r = int(rng.integers(1, 4))
    ext = [int(rng.integers(1, 7)) for _ in range(r)]
    win = [a for a in range(r) if rng.random() < 0.6]
    rng.shuffle(win)
    k = int(rng.integers(1, r + 1))
    sdims = [int(a) for a in rng.permutation(r)[:k]]
    nb = int(rng.integers(0, 3))
    bext = [int(rng.integers(1, 9)) for _ in range(nb)]
    if k == 1 and rng.random() < 0.3:
        ivd, iext = nb, list(bext)
    else:
        ivd = int(rng.integers(0, nb + 1))
        iext = bext[:ivd] + [k] + bext[ivd:]
    urank = nb + len(win)
    uwd = [int(a) for a in rng.permutation(urank)[:len(win)]]
    uext, b = [0] * urank, 0
    for q, a in enumerate(win):
        uext[uwd[q]] = int(rng.integers(1, ext[a] + 1)) if rng.random() < 0.95 else ext[a] + 1
    for ax in range(urank):
        if ax not in uwd:
            uext[ax] = bext[b]
            b += 1
    comp = COMPONENT_NP[dtype]
    k2 = 2 if dtype in (abi.C32, abi.C64) else 1
    dest_l, dest_span = (abi.layout(ext), int(np.prod(ext))) if rng.random() < 0.5 else random_strided(rng, ext)
    if any(s < 0 for s in dest_l.strides_list()):
        dest_l, dest_span = abi.layout(ext), int(np.prod(ext))
    upd_l, upd_span = (abi.layout(uext), int(np.prod(uext))) if rng.random() < 0.5 else random_strided(rng, uext)
    dest = rng.standard_normal(dest_span * k2).astype(comp)
    upd = rng.standard_normal(upd_span * k2).astype(comp)
    idx = random_indices(rng, iext, max(ext), index_dtype)
    return Scatter(dtype, index_dtype, dest, dest_l, idx, abi.layout(iext), upd, upd_l,
                   splan(win, uwd, sdims, ivd, r, urank))


@pytest.mark.parametrize("dtype", [abi.F32, abi.F64, abi.C32, abi.C64])
@pytest.mark.parametrize("index_dtype", [abi.I32, abi.F64])
def test_scatter_random_plans(cuda, dtype, index_dtype):
    rng = np.random.default_rng(2000 + 10 * dtype + index_dtype)
    for _ in range(25):
        random_scatter(rng, dtype, index_dtype).check()


def test_config4_full_size_properties(cuda):
    """BASELINE config 4 at full size through the row helpers, checked by properties
    that do not need a CPU pass over 6 GB: gather = the oracle on 65,536 sampled output
    rows (bit-exact); scatter_add from a zero destination = per-column sums of the
    updates (linearity; tolerance 1e-12 x the column's sum of |update|), and the hottest
    row = the sum of its updates (same tolerance)."""
    import torch
    rows, cols, n = 1 << 20, 128, 1 << 22
    g = torch.Generator(device="cuda").manual_seed(4)
    table = torch.randn((rows, cols), dtype=torch.float32, device="cuda", generator=g)
    gidx = torch.randint(0, rows, (n,), dtype=torch.int64, device="cuda", generator=g)
    out = t4.gather_rows(table, gidx)
    torch.cuda.synchronize()
    sample = torch.randint(0, n, (1 << 16,), device="cuda", generator=g)
    got = out[sample].cpu().numpy()
    idx = gidx[sample].cpu().numpy()
    host_table = table.cpu().numpy()
    want = np.empty_like(got)
    plan = abi.gather_plan([0], [0], [1], [cols, 1], 1, 2)
    rc = oracle.lib().t4a_oracle_gather(abi.F32, abi.I64, oracle.ptr(want), oracle.ptr(host_table), oracle.ptr(idx),
                                        ctypes.byref(abi.numpy_layout([idx.size, cols])),
                                        ctypes.byref(abi.numpy_layout([rows, cols])),
                                        ctypes.byref(abi.layout([idx.size, 1])), ctypes.byref(plan), THREADS)
    assert rc == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    del out, table, host_table

    upd = torch.randn((n, cols), dtype=torch.float64, device="cuda", generator=g)
    w = torch.arange(1, rows + 1, dtype=torch.float64, device="cuda") ** -1.1
    cdf = torch.cumsum(w, 0)
    cdf /= cdf[-1].clone()
    sidx = torch.clamp(torch.searchsorted(cdf, torch.rand(n, dtype=torch.float64, device="cuda", generator=g),
                                          right=True), max=rows - 1)
    dest = torch.zeros((rows, cols), dtype=torch.float64, device="cuda")
    t4.scatter_add_rows(dest, sidx, upd, workspace=t4.scatter_rows_workspace(dest, sidx, upd))
    torch.cuda.synchronize()
    col_got = dest.sum(dim=0)
    col_want = upd.sum(dim=0)
    col_mag = upd.abs().sum(dim=0)
    assert bool(((col_got - col_want).abs() <= 1e-12 * col_mag).all())
    hot = int(torch.mode(sidx[: 1 << 16]).values)
    sel = upd[sidx == hot]
    assert sel.shape[0] > 100_000
    row_err = (dest[hot] - sel.sum(dim=0)).abs()
    assert bool((row_err <= 1e-12 * sel.abs().sum(dim=0)).all())


# ---- general-rank twins (`_any`) ------------------------------------------------

ANY_ROUTES = ["launcher", "module", "refgeom"]


def any_layout(l, pad=0):
    """A by-value layout as t4a_cuda_layout_any, with `pad` trailing extent-1 axes."""
    return t4.layout_any(l.extents_list() + [1] * pad, l.strides_list() + [0] * pad, l.offset)


def any_launch(route, name, n, args):
    import torch
    if route == "launcher":
        t4.launch_movement_any(name, t4.gather_scatter_any_geometry(n), t4.stream_handle(), *args)
    elif n > 0:
        if route == "module":
            g = t4.gather_scatter_any_geometry(n)
            geom = (tuple(g.grid), tuple(g.block), 0)
        else:
            geom = ((max(1, (n + 255) // 256),), (256,), 0)
        module(OUR_CUBIN).launch("t4a_cuda_" + name + "_any", *geom, args)
    torch.cuda.synchronize()


def gather_any(case, route, pad):
    """Case `case` through t4a_cuda_gather_any; `pad` extent-1 operand axes become
    window axes of slice 1 on as many new trailing output axes (rank up to 4 + pad)."""
    import torch
    p = case.plan
    w, k = p.window_rank, p.start_map_len
    r, out_rank = p.operand_rank, p.out_rank
    win = list(p.window_dims[:w]) + list(range(r, r + pad))
    offs = list(p.offset_dims[:w]) + list(range(out_rank, out_rank + pad))
    slices = list(p.slice_sizes[:r]) + [1] * pad
    plan, keep_p = t4.gather_plan_any(win, offs, list(p.start_index_map[:k]), slices, p.index_vector_dim,
                                      out_rank + pad)
    ol, k1 = any_layout(case.out_l, pad)
    al, k2 = any_layout(case.operand_l, pad)
    il, k3 = any_layout(case.indices_l)
    n = case.out_l.count()
    d_op = dev(case.operand)
    d_idx = dev(case.indices.view(np.uint8)) if case.indices.size else torch.zeros(16, dtype=torch.uint8,
                                                                                     device="cuda")
    d_out = sentinel(case.out_elems * case.es)
    any_launch(route, "gather", n, [vptr(d_out), vptr(d_op), vptr(d_idx), ctypes.c_int(case.dtype),
                                    ctypes.c_int(case.index_dtype), ol, al, il, plan, ctypes.c_longlong(n)])
    del keep_p, k1, k2, k3
    return take(d_out, case.out_elems * case.es)


def scatter_any(case, route, pad):
    """Case `case` through t4a_cuda_scatter_add_any; `pad` extent-1 destination axes
    become window axes fed by as many new trailing extent-1 update axes."""
    import torch
    p = case.plan
    w, k = p.window_rank, p.scatter_map_len
    r, ur = p.operand_rank, p.updates_rank
    plan, keep_p = t4.scatter_plan_any(list(p.window_dims[:w]) + list(range(r, r + pad)),
                                       list(p.update_window_dims[:w]) + list(range(ur, ur + pad)),
                                       list(p.scatter_dims[:k]), p.index_vector_dim, r + pad, ur + pad)
    ol, k1 = any_layout(case.dest_l, pad)
    il, k2 = any_layout(case.indices_l)
    ul, k3 = any_layout(case.updates_l, pad)
    n = case.updates_l.count()
    d_out = sentinel(case.dest.nbytes)
    d_out[:case.dest.nbytes] = dev(case.dest.view(np.uint8))
    d_upd = dev(case.updates.view(np.uint8)) if case.updates.size else torch.zeros(16, dtype=torch.uint8,
                                                                                     device="cuda")
    d_idx = dev(case.indices.view(np.uint8)) if case.indices.size else torch.zeros(16, dtype=torch.uint8,
                                                                                     device="cuda")
    any_launch(route, "scatter_add", n, [vptr(d_out), vptr(d_idx), vptr(d_upd), ctypes.c_int(case.dtype),
                                         ctypes.c_int(case.index_dtype), ol, il, ul, plan, ctypes.c_longlong(n)])
    del keep_p, k1, k2, k3
    return take(d_out, case.dest.nbytes).view(case.comp)


@pytest.mark.parametrize("route", ANY_ROUTES)
@pytest.mark.parametrize("dtype", [abi.BOOL, abi.F64, abi.C32, abi.C64])
@pytest.mark.parametrize("index_dtype", [abi.I64, abi.F32])
def test_gather_any_random_plans(cuda, route, dtype, index_dtype):
    """The general-rank gather equals the oracle bit for bit on random plans, as given
    (rank <= 4) and padded with extent-1 window axes to rank 9-12."""
    rng = np.random.default_rng(3000 + 10 * dtype + index_dtype + 100 * ANY_ROUTES.index(route))
    for i in range(12):
        case = random_gather(rng, dtype, index_dtype)
        want = case.oracle()
        for pad in (0, 8):
            got = gather_any(case, route, pad)
            assert np.array_equal(want, got), (i, pad)


@pytest.mark.parametrize("route", ANY_ROUTES)
@pytest.mark.parametrize("dtype", [abi.F32, abi.F64, abi.C32, abi.C64])
@pytest.mark.parametrize("index_dtype", [abi.I32, abi.F64])
def test_scatter_add_any_random_plans(cuda, route, dtype, index_dtype):
    """The general-rank scatter_add equals the oracle (within the atomics' rounding) on
    random plans, including windows that do not fit, as given and padded to rank 9-11."""
    rng = np.random.default_rng(4000 + 10 * dtype + index_dtype + 100 * ANY_ROUTES.index(route))
    tol, atol = TOL[dtype]
    for i in range(12):
        case = random_scatter(rng, dtype, index_dtype)
        want = case._oracle(case.dest, case.updates)
        mag = case._oracle(np.abs(case.dest), np.abs(case.updates))
        for pad in (0, 8):
            got = scatter_any(case, route, pad)
            ok = (got == want) | (np.abs(got - want) <= tol * mag + atol)
            assert ok.all(), (i, pad, np.flatnonzero(~ok)[:8])


def test_any_twins_on_config4_rows(cuda):
    """BASELINE config 4's row gather and Zipf scatter_add (reduced row counts) through
    the general-rank twins, against the fast entries."""
    import torch
    rng = np.random.default_rng(5)
    rows, cols, n = 4096, 128, 20000
    table = torch.from_numpy(rng.standard_normal((rows, cols)).astype(np.float32)).cuda()
    gidx = torch.from_numpy(rng.integers(0, rows, n)).cuda()
    want = t4.gather_rows(table, gidx)
    plan, kp = t4.gather_plan_any([0], [0], [1], [cols, 1], 1, 2)
    ol, k1 = t4.layout_any([cols, n], [1, cols])
    al, k2 = t4.layout_any([cols, rows], [1, cols])
    il, k3 = t4.layout_any([n, 1])
    out = torch.empty((n, cols), dtype=torch.float32, device="cuda")
    any_launch("launcher", "gather", n * cols, [vptr(out), vptr(table), vptr(gidx), ctypes.c_int(abi.F32),
                                                ctypes.c_int(abi.I64), ol, al, il, plan, ctypes.c_longlong(n * cols)])
    assert torch.equal(out, want)
    dest = torch.from_numpy(rng.standard_normal((rows, cols))).cuda()
    sidx = torch.from_numpy(zipf_rows(rng, n, rows)).cuda()
    upd = torch.from_numpy(rng.standard_normal((n, cols))).cuda()
    want = t4.scatter_add_rows(dest.clone(), sidx, upd)
    splan_any, kq = t4.scatter_plan_any([0], [0], [1], 1, 2, 2)
    dl, k4 = t4.layout_any([cols, rows], [1, cols])
    sl, k5 = t4.layout_any([n, 1])
    ul, k6 = t4.layout_any([cols, n], [1, cols])
    got = dest.clone()
    any_launch("launcher", "scatter_add", n * cols, [vptr(got), vptr(sidx), vptr(upd), ctypes.c_int(abi.F64),
                                                     ctypes.c_int(abi.I64), dl, sl, ul, splan_any,
                                                     ctypes.c_longlong(n * cols)])
    assert torch.allclose(got, want, rtol=0, atol=1e-12 * float(want.abs().max()))
    del kp, kq, k1, k2, k3, k4, k5, k6


@pytest.mark.parametrize("route", ["launcher", "module"])
def test_any_twins_leave_malformed_maps_untouched(cuda, route):
    """The kernels check the device-resident maps before walking: a repeated offset
    dimension, a window axis past the operand's rank, or a count beyond the walked
    layout's extents makes every block return, so the destination keeps its sentinel."""
    import torch
    rows, cols, n = 64, 8, 16
    table = dev(np.arange(rows * cols, dtype=np.float32).view(np.uint8))
    idx = dev(np.arange(n, dtype=np.int64).view(np.uint8))
    ol, k1 = t4.layout_any([cols, n], [1, cols])
    al, k2 = t4.layout_any([cols, rows], [1, cols])
    il, k3 = t4.layout_any([n, 1])
    bad_plans = [
        t4.gather_plan_any([0, 1], [0, 0], [1], [cols, 1], 1, 2),  # offset dimension repeated
        t4.gather_plan_any([5], [0], [1], [cols, 1], 1, 2),        # window axis past the operand
    ]
    good, kg = t4.gather_plan_any([0], [0], [1], [cols, 1], 1, 2)
    cases = [(p, n * cols) for p, _ in bad_plans] + [(good, n * cols + 1)]  # last: count beyond the extents
    for plan, count in cases:
        out = sentinel(n * cols * 4)
        args = [vptr(out), vptr(table), vptr(idx), ctypes.c_int(abi.F32), ctypes.c_int(abi.I64), ol, al, il, plan,
                ctypes.c_longlong(count)]
        if route == "launcher":
            try:
                t4.launch_movement_any("gather", t4.gather_scatter_any_geometry(count), t4.stream_handle(), *args)
            except t4.T4AError:
                pass  # refused on the host: nothing launched
        else:
            g = t4.gather_scatter_any_geometry(count)
            module(OUR_CUBIN).launch("t4a_cuda_gather_any", tuple(g.grid), tuple(g.block), 0, args)
        torch.cuda.synchronize()
        assert (take(out, n * cols * 4) == SENTINEL).all()
    # scatter: update window wider than the updates' rank is refused on the host; a
    # repeated update window dimension is refused by the kernel.
    dest = dev(np.zeros(rows * cols, np.float64).view(np.uint8))
    upd = dev(np.ones(n * cols, np.float64).view(np.uint8))
    dl, k4 = t4.layout_any([cols, rows], [1, cols])
    ul, k5 = t4.layout_any([cols, n], [1, cols])
    splan, ks = t4.scatter_plan_any([0, 1], [0, 0], [1], 1, 2, 2)
    args = [vptr(dest), vptr(idx), vptr(upd), ctypes.c_int(abi.F64), ctypes.c_int(abi.I64), dl, il, ul, splan,
            ctypes.c_longlong(n * cols)]
    g = t4.gather_scatter_any_geometry(n * cols)
    if route == "launcher":
        try:
            t4.launch_movement_any("scatter_add", g, t4.stream_handle(), *args)
        except t4.T4AError:
            pass
    else:
        module(OUR_CUBIN).launch("t4a_cuda_scatter_add_any", tuple(g.grid), tuple(g.block), 0, args)
    torch.cuda.synchronize()
    assert (take(dest, rows * cols * 8).view(np.float64) == 0).all()
    del k1, k2, k3, k4, k5, kg, ks, bad_plans


@pytest.mark.parametrize("dtype,cols", [(abi.F64, 128), (abi.F32, 32), (abi.C64, 16), (abi.F64, 3)])
def test_scatter_range_shards_tile_the_destination(cuda, dtype, cols):
    """t4a_scatter_add_range (owner-computes sharding): three uneven row slices of a
    row-major destination, each scattered into its own buffer from the whole index list,
    together equal t4a_scatter_add over the whole destination within the bound on
    reordering a sum of k terms, 2 (k - 1) u sum|x| per element (u the unit roundoff).
    The indices include values below 0 and past the last row, which clamp."""
    import torch
    tdt = {abi.F64: torch.float64, abi.F32: torch.float32, abi.C64: torch.complex128}[dtype]
    u = 2.0 ** -24 if dtype == abi.F32 else 2.0 ** -53
    rng = np.random.default_rng(77 + dtype + cols)
    rows, n = 5000, 60000
    idx_np = zipf_rows(rng, n, rows + 20) - 10
    idx = torch.from_numpy(idx_np.astype(np.int64)).cuda()
    g = torch.Generator(device="cpu").manual_seed(5)
    upd = torch.randn(n, cols, generator=g, dtype=tdt).cuda()
    dest0 = torch.randn(rows, cols, generator=g, dtype=tdt).cuda()
    whole = dest0.clone()
    ws = t4.scatter_rows_workspace(whole, idx, upd)
    t4.scatter_add_rows(whole, idx, upd, workspace=ws)
    clamped = idx.clamp(0, rows - 1)
    comp = (lambda t: torch.view_as_real(t)) if dtype == abi.C64 else (lambda t: t)
    absum = comp(dest0).abs().clone().index_add_(0, clamped, comp(upd).abs())
    count = torch.zeros(rows, dtype=torch.float64, device="cuda").index_add_(
        0, clamped, torch.ones(n, dtype=torch.float64, device="cuda"))
    shape = (rows,) + (1,) * (absum.dim() - 1)
    bound = (2.0 * count * u).view(shape) * absum.double()
    for r0, r1 in [(0, 1700), (1700, 1701), (1701, rows)]:
        shard = dest0[r0:r1].clone()
        ws2 = t4.scatter_rows_workspace(whole, idx, upd)
        t4.scatter_add_rows_range(shard, rows, r0, idx, upd, ws2)
        torch.cuda.synchronize()
        assert int(ws2[:4].view(torch.int32).item()) == 0
        err = (comp(shard) - comp(whole[r0:r1])).abs().double()
        assert bool((err <= bound[r0:r1]).all()), (r0, r1, float((err - bound[r0:r1]).max()))


@pytest.mark.parametrize("dtype,cols", [(abi.F64, 128), (abi.F32, 32), (abi.C64, 16), (abi.F64, 3)])
def test_scatter_cyclic_owners_tile_the_destination(cuda, dtype, cols):
    """t4a_scatter_add_cyclic (block-cyclic owner-computes sharding, one row per block):
    three owners, each scattering the whole index list into its rows r % 3 == owner,
    together equal t4a_scatter_add over the whole destination within the reordering
    bound.  The indices include values below 0 and past the last row, which clamp."""
    import torch
    tdt = {abi.F64: torch.float64, abi.F32: torch.float32, abi.C64: torch.complex128}[dtype]
    u = 2.0 ** -24 if dtype == abi.F32 else 2.0 ** -53
    rng = np.random.default_rng(88 + dtype + cols)
    rows, n, owners = 5000, 60000, 3
    idx = torch.from_numpy((zipf_rows(rng, n, rows + 20) - 10).astype(np.int64)).cuda()
    g = torch.Generator(device="cpu").manual_seed(6)
    upd = torch.randn(n, cols, generator=g, dtype=tdt).cuda()
    dest0 = torch.randn(rows, cols, generator=g, dtype=tdt).cuda()
    whole = dest0.clone()
    t4.scatter_add_rows(whole, idx, upd, workspace=t4.scatter_rows_workspace(whole, idx, upd))
    clamped = idx.clamp(0, rows - 1)
    comp = (lambda t: torch.view_as_real(t)) if dtype == abi.C64 else (lambda t: t)
    absum = comp(dest0).abs().clone().index_add_(0, clamped, comp(upd).abs())
    count = torch.zeros(rows, dtype=torch.float64, device="cuda").index_add_(
        0, clamped, torch.ones(n, dtype=torch.float64, device="cuda"))
    bound = (2.0 * count * u).view((rows,) + (1,) * (absum.dim() - 1)) * absum.double()
    for owner in range(owners):
        shard = dest0[owner::owners].clone()
        ws = t4.scatter_rows_workspace(whole, idx, upd)
        t4.scatter_add_rows_cyclic(shard, rows, owners, owner, idx, upd, ws)
        torch.cuda.synchronize()
        assert int(ws[:4].view(torch.int32).item()) == 0
        err = (comp(shard) - comp(whole[owner::owners])).abs().double()
        assert bool((err <= bound[owner::owners]).all()), (owner, float((err - bound[owner::owners]).max()))

