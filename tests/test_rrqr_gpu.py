"""GPU parity of the RRQR primitives and of the fused factorization (t4a_rrqr).

Each entry runs through this library's launcher, its exported module symbol (the
planner's geometry and the reference's: one 32-lane block per task, flat entries
ceil(len/256) x 256) and the reference's own kernel rebuilt from source (oracle/_ref),
and is compared with the CPU oracle: bit for bit for F32/F64 (norms, pivots, status,
reflectors, updates), and for C32/C64 within 1e-5 / 1e-12 relative to the column
scale (the oracle's complex sums are not contracted like the device's; against the
reference's own kernels complex norms and reflectors are bit-identical, complex
updates agree within rounding).  Destinations carry
sentinel bytes and guard bytes, as in the reference tests (tests/gpu_rrqr.rs:193-360).
Cases follow tests/gpu_rrqr.rs: norms with the -1 sentinel, pivot tie breaks, swap,
reflector, apply, extract_r, prefix_rank, initialize_permutation; and the whole loop
of BASELINE config 5 (A = U V^T + 1e-10 N) at reduced and full size.
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
OUR_CUBIN = os.path.join(ROOT, "t4a-cuda-kernels_b200", "t4a_b200", "lib", "rrqr.cubin")
REF_CUBIN = os.path.join(ROOT, "oracle", "_ref", "rrqr.cubin")
OUR_LINALG = os.path.join(ROOT, "t4a-cuda-kernels_b200", "t4a_b200", "lib", "linalg_aux.cubin")
REF_LINALG = os.path.join(ROOT, "oracle", "_ref", "linalg_aux.cubin")
SENTINEL, GUARD = 0xCD, 256
THREADS = os.cpu_count() or 4
NP = {abi.F32: np.float32, abi.F64: np.float64, abi.C32: np.complex64, abi.C64: np.complex128,
      abi.I32: np.int32, abi.I64: np.int64}
REAL = {abi.F32: abi.F32, abi.F64: abi.F64, abi.C32: abi.F32, abi.C64: abi.F64}
ROUTES = ["launcher", "module", "module-refgeom", "reference"]
_MODULES = {}


def module(path):
    if path not in _MODULES:
        if not os.path.exists(path):
            pytest.skip(f"{os.path.basename(path)} not built")
        _MODULES[path] = Module(path)
    return _MODULES[path]


def dev(arr):
    import torch
    b = np.ascontiguousarray(arr).view(np.uint8).ravel()
    return torch.from_numpy(np.concatenate([b, np.full(GUARD, SENTINEL, np.uint8)])).cuda()


def sentinel_dev(nbytes):
    import torch
    return torch.full((nbytes + GUARD,), SENTINEL, dtype=torch.uint8, device="cuda")


def host(t, nbytes, dtype):
    h = t.cpu().numpy()
    assert (h[nbytes:] == SENTINEL).all(), "a store landed past the buffer"
    return h[:nbytes].view(dtype).copy()


def vp(t):
    return ctypes.c_void_p(t.data_ptr())


def launch(route, name, plan_launch, ref_geom, args):
    """Run entry `name` by `route`; args: ctypes objects in kernel order."""
    import torch
    if route == "launcher":
        t4.launch_rrqr(name, plan_launch, t4.stream_handle(), *args)
    else:
        if route == "module":
            mod = module(OUR_CUBIN)
            geom = (tuple(plan_launch.grid), tuple(plan_launch.block), plan_launch.shared_bytes)
        else:
            mod = module(OUR_CUBIN if route == "module-refgeom" else REF_CUBIN)
            geom = ref_geom
        if plan_launch.grid[0] > 0:
            mod.launch("t4a_cuda_" + name, *geom, list(args))
    torch.cuda.synchronize()


def plane(tasks):
    return ((max(1, tasks),), (32,), 0)


def flat(n):
    return ((max(1, (n + 255) // 256),), (256,), 0)


def rand_matrix(rng, dtype, m, n, shift=0.0):
    if dtype in (abi.C32, abi.C64):
        a = rng.standard_normal((n, m)) + 1j * rng.standard_normal((n, m)) + shift
    else:
        a = rng.standard_normal((n, m)) + shift
    return a.astype(NP[dtype])  # row j = column j (column-major [m, n])


def same(dtype, got, want, scale=None):
    got, want = np.asarray(got).ravel(), np.asarray(want).ravel()
    if dtype in (abi.F32, abi.F64, abi.I32, abi.I64):
        return np.array_equal(np.asarray(got).view(np.uint8), np.asarray(want).view(np.uint8))
    tol = 1e-5 if dtype == abi.C32 else 1e-12
    s = np.abs(want).max() if scale is None else scale
    return np.allclose(got, want, rtol=0, atol=tol * max(s, 1e-30))


# ---- column_norms ---------------------------------------------------------------

@pytest.mark.parametrize("dtype", [abi.F32, abi.F64, abi.C32, abi.C64])
@pytest.mark.parametrize("m,n,step", [(1000, 12, 0), (4099, 40, 7), (64, 70, 63), (33, 36, 32)])
def test_column_norms(cuda, dtype, m, n, step):
    rng = np.random.default_rng(m + n + step + dtype)
    a = rand_matrix(rng, dtype, m, n)
    a[1, 3 % m] = np.nan            # column 1: non-finite -> -1
    if n > 2:
        a[2, m - 1] = np.inf         # column 2: non-finite -> -1
    a[n - 1] *= 1e30 if dtype in (abi.F64, abi.C64) else 1e18  # a large column (scaling)
    wl, nl = abi.layout([m, n]), abi.layout([n])
    rd = REAL[dtype]
    want = np.full(n, -7.0, dtype=NP[rd])
    assert oracle.lib().t4a_oracle_column_norms(dtype, oracle.ptr(a), oracle.ptr(want), ctypes.byref(wl),
                                                ctypes.byref(nl), step, THREADS) == 0
    pl = t4.plan_rrqr("column_norms", dtype, wl, m * n, nl, n, step)
    got = {}
    for route in ROUTES:
        d_a = dev(a)
        d_n = dev(np.full(n, -7.0, dtype=NP[rd]))
        launch(route, "column_norms", pl, plane(n - step),
               [vp(d_a), vp(d_n), ctypes.c_int(dtype), wl, nl, ctypes.c_longlong(step)])
        got[route] = host(d_n, n * np.dtype(NP[rd]).itemsize, NP[rd])
        assert np.array_equal(got[route][:step], want[:step]), route  # untouched
        if dtype in (abi.F32, abi.F64):
            assert same(rd, got[route], want), (route, got[route][:6], want[:6])
        else:
            assert np.allclose(got[route], want, rtol=1e-5 if dtype == abi.C32 else 1e-12), route
    # The reference's own kernel and this library's agree bit for bit (complex too).
    assert np.array_equal(got["launcher"].view(np.uint8), got["reference"].view(np.uint8))


# ---- select_pivot -----------------------------------------------------------------

def pivot_case(route, dtype, norms, perm, step, tasks_layout=None):
    norms = np.asarray(norms, dtype=NP[dtype])
    perm = np.asarray(perm, dtype=np.int64)
    n = norms.size
    nl = abi.layout([n])
    pl = t4.plan_rrqr("select_pivot", dtype, nl, n, nl, n, 1, 1, step)
    d_norms, d_perm = dev(norms), dev(perm)
    d_piv, d_st = dev(np.zeros(1, np.int64)), dev(np.zeros(1, np.int64))
    launch(route, "select_pivot", pl, plane(1),
           [vp(d_norms), vp(d_perm), vp(d_piv), vp(d_st), ctypes.c_int(dtype), nl, nl, ctypes.c_longlong(step)])
    return int(host(d_piv, 8, np.int64)[0]), int(host(d_st, 8, np.int64)[0])


@pytest.mark.parametrize("route", ROUTES)
def test_select_pivot_tie_breaks(cuda, route):
    f = abi.F32
    assert pivot_case(route, f, [1, 5, 3, 2, 4, 0], range(6), 0) == (1, 0)     # clear maximum
    assert pivot_case(route, f, [1, 5, 5, 2], [0, 3, 1, 2], 0) == (2, 0)       # smaller original wins
    assert pivot_case(route, f, [5, 5], [7, 7], 0) == (0, 0)                   # then the smaller column
    assert pivot_case(route, f, [9, 1, 4, 5], range(4), 2) == (3, 0)           # step skips leading columns
    assert pivot_case(route, f, [1, -1, 3], range(3), 0) == (2, 1)             # negative norm -> status
    assert pivot_case(route, f, [-1, -1], range(2), 0) == (0, 1)               # nothing valid -> step


@pytest.mark.parametrize("dtype", [abi.F32, abi.F64])
def test_select_pivot_random(cuda, dtype):
    rng = np.random.default_rng(11 + dtype)
    for _ in range(20):
        n = int(rng.integers(1, 300))
        step = int(rng.integers(0, n + 1))
        norms = rng.integers(0, 6, n).astype(NP[dtype])   # many ties
        perm = rng.permutation(n).astype(np.int64)
        want_p = np.zeros(1, np.int64)
        want_s = np.zeros(1, np.int64)
        nl = abi.layout([n])
        assert oracle.lib().t4a_oracle_select_pivot(dtype, oracle.ptr(norms), oracle.lptr(perm), oracle.lptr(want_p),
                                                    oracle.lptr(want_s), ctypes.byref(nl), ctypes.byref(nl),
                                                    step) == 0
        for route in ROUTES:
            assert pivot_case(route, dtype, norms, perm, step) == (int(want_p[0]), int(want_s[0])), route


# ---- swap_columns -------------------------------------------------------------------

@pytest.mark.parametrize("dtype", [abi.F32, abi.F64, abi.I32, abi.I64, abi.C32, abi.C64])
def test_swap_columns(cuda, dtype):
    rng = np.random.default_rng(20 + dtype)
    m, n = 3001, 9
    a = (rng.integers(-1000, 1000, (n, m)) if dtype in (abi.I32, abi.I64) else rand_matrix(rng, dtype, m, n))
    a = a.astype(NP[dtype])
    wl, pl_ = abi.layout([m, n]), abi.layout([n])
    for step, pivot in [(2, 7), (4, 4), (0, 8)]:
        perm = rng.permutation(n).astype(np.int64)
        want_a, want_p = a.copy(), perm.copy()
        piv = np.array([pivot], np.int64)
        assert oracle.lib().t4a_oracle_swap_columns(dtype, oracle.ptr(want_a), oracle.lptr(want_p), oracle.lptr(piv),
                                                    ctypes.byref(wl), ctypes.byref(pl_), step) == 0
        plan = t4.plan_rrqr("swap_columns", dtype, wl, m * n, pl_, n, 1, step)
        for route in ROUTES:
            d_a, d_p, d_piv = dev(a), dev(perm), dev(piv)
            launch(route, "swap_columns", plan, flat(m),
                   [vp(d_a), vp(d_p), vp(d_piv), ctypes.c_int(dtype), wl, pl_, ctypes.c_longlong(step)])
            assert np.array_equal(host(d_a, a.nbytes, NP[dtype]).view(np.uint8), want_a.ravel().view(np.uint8)), route
            assert np.array_equal(host(d_p, perm.nbytes, np.int64), want_p), route


# ---- reflector and apply_reflector -----------------------------------------------------

@pytest.mark.parametrize("dtype", [abi.F32, abi.F64, abi.C32, abi.C64])
@pytest.mark.parametrize("m,n,step", [(2000, 8, 0), (4097, 20, 5), (40, 40, 39)])
def test_reflector_and_apply(cuda, dtype, m, n, step):
    rng = np.random.default_rng(m * 3 + n + step + dtype)
    a = rand_matrix(rng, dtype, m, n, shift=0.5)
    wl, cl = abi.layout([m, n]), abi.layout([n])
    coeff0 = np.zeros(n, NP[dtype])
    want_a, want_c = a.copy(), coeff0.copy()
    assert oracle.lib().t4a_oracle_reflector(dtype, oracle.ptr(want_a), oracle.ptr(want_c), ctypes.byref(wl),
                                             ctypes.byref(cl), step) == 0
    plan = t4.plan_rrqr("reflector", dtype, wl, m * n, cl, n, step)
    results = {}
    for route in ROUTES:
        d_a, d_c = dev(a), dev(coeff0)
        launch(route, "reflector", plan, plane(1),
               [vp(d_a), vp(d_c), ctypes.c_int(dtype), wl, cl, ctypes.c_longlong(step)])
        got_a, got_c = host(d_a, a.nbytes, NP[dtype]), host(d_c, coeff0.nbytes, NP[dtype])
        results[route] = (got_a, got_c)
        assert same(dtype, got_a, want_a), route
        assert same(dtype, got_c, want_c), route
    if dtype in (abi.C32, abi.C64):
        assert np.array_equal(results["launcher"][0].view(np.uint8), results["reference"][0].view(np.uint8))
    # apply_reflector: the reflector of `step` (packed = a copy of the reflected matrix)
    # onto the trailing columns step+1..n of the reflected matrix.
    packed = want_a.copy()
    first, count = step + 1, n - step - 1
    if count == 0:
        return
    want_t = want_a.copy()
    assert oracle.lib().t4a_oracle_apply_reflector(dtype, oracle.ptr(packed), oracle.ptr(want_t), oracle.ptr(want_c),
                                                   ctypes.byref(wl), ctypes.byref(wl), ctypes.byref(cl), step, first,
                                                   count, THREADS) == 0
    plan = t4.plan_rrqr("apply_reflector", dtype, wl, m * n, wl, m * n, cl, n, step, first, count)
    got = {}
    for route in ROUTES:
        d_p, d_t, d_c = dev(packed), dev(want_a), dev(want_c)
        launch(route, "apply_reflector", plan, plane(count),
               [vp(d_p), vp(d_t), vp(d_c), ctypes.c_int(dtype), wl, wl, cl, ctypes.c_longlong(step),
                ctypes.c_longlong(first), ctypes.c_longlong(count)])
        got[route] = host(d_t, a.nbytes, NP[dtype])
        assert same(dtype, got[route], want_t, scale=np.abs(want_a).max() * 4), route
    # Complex updates: the compiler's contraction of the complex products may differ
    # from the reference kernel's, so they agree within rounding, not bit for bit.
    if dtype in (abi.C32, abi.C64):
        assert same(dtype, got["launcher"], got["reference"], scale=np.abs(want_a).max() * 4)


# ---- extract_r, prefix_rank, initialize_permutation ------------------------------------

@pytest.mark.parametrize("dtype", [abi.F32, abi.F64, abi.C32, abi.C64])
def test_extract_r_and_prefix_rank(cuda, dtype):
    rng = np.random.default_rng(30 + dtype)
    m, n, k = 50, 12, 12
    a = rand_matrix(rng, dtype, m, n)
    wl, rl = abi.layout([m, n]), abi.layout([k, n])
    want_r = np.zeros(k * n, NP[dtype])
    assert oracle.lib().t4a_oracle_extract_r(dtype, oracle.ptr(a), oracle.ptr(want_r), ctypes.byref(wl),
                                             ctypes.byref(rl)) == 0
    plan = t4.plan_rrqr("extract_r", dtype, wl, m * n, rl, k * n)
    for route in ROUTES:
        d_a, d_r = dev(a), sentinel_dev(want_r.nbytes)
        launch(route, "extract_r", plan, flat(k * n), [vp(d_a), vp(d_r), ctypes.c_int(dtype), wl, rl])
        assert np.array_equal(host(d_r, want_r.nbytes, NP[dtype]).view(np.uint8), want_r.view(np.uint8)), route
    # prefix_rank: a diagonal that decays, one non-finite entry variant.
    diag = np.geomspace(1.0, 1e-14, k)
    for bad in (False, True):
        r = np.zeros((n, k), NP[dtype])  # column-major [k, n]
        for d in range(k):
            r[d, d] = diag[d]
        if bad:
            r[5, 5] = np.nan
        rl2 = abi.layout([k, n])
        for rtol, atol in [(1e-8, 0.0), (0.0, 1e-3), (1e-16, 1e-20)]:
            want_rank, want_st = np.zeros(1, np.int64), np.zeros(1, np.int64)
            assert oracle.lib().t4a_oracle_prefix_rank(dtype, oracle.ptr(r), oracle.lptr(want_rank),
                                                       oracle.lptr(want_st), ctypes.byref(rl2), rtol, atol) == 0
            plan = t4.plan_rrqr("prefix_rank", dtype, rl2, k * n, 1, 1, rtol, atol)
            for route in ROUTES:
                d_r, d_rank, d_st = dev(r), dev(np.zeros(1, np.int64)), dev(np.zeros(1, np.int64))
                launch(route, "prefix_rank", plan, plane(1),
                       [vp(d_r), vp(d_rank), vp(d_st), ctypes.c_int(dtype), rl2, ctypes.c_double(rtol),
                        ctypes.c_double(atol)])
                assert int(host(d_rank, 8, np.int64)[0]) == int(want_rank[0]), (route, rtol, atol, bad)
                assert int(host(d_st, 8, np.int64)[0]) == int(want_st[0]), (route, bad)


@pytest.mark.parametrize("route", ROUTES)
def test_initialize_permutation(cuda, route):
    n, length = 37, 37 * 5
    plan = t4.plan_rrqr("initialize_permutation", n, length)
    d = sentinel_dev(length * 8)
    launch(route, "initialize_permutation", plan, flat(length),
           [vp(d), ctypes.c_longlong(n), ctypes.c_longlong(length)])
    assert np.array_equal(host(d, length * 8, np.int64), np.arange(length) % n)


# ---- the whole loop ---------------------------------------------------------------------

def config5_matrix(m, n, rank, seed=10):
    rng = np.random.default_rng(seed)
    u = rng.standard_normal((m, rank))
    v = rng.standard_normal((n, rank))
    noise = rng.standard_normal((m, n))
    a = u @ v.T + 1e-10 * noise
    return np.asfortranarray(a)  # column-major [m, n]


def oracle_rrqr(a, steps):
    m, n = a.shape
    work = np.asfortranarray(a).copy(order="F")
    perm = np.zeros(n, np.int64)
    coeff = np.zeros(max(steps, 1))
    rank = oracle.lib().t4a_oracle_rrqr_f64(oracle.ptr(work.ravel(order="K")), m, n, steps, oracle.lptr(perm),
                                            oracle.ptr(coeff), 1e-8, 0.0, THREADS)
    return work, perm, coeff, rank


def primitives_rrqr(a, steps, dtype=abi.F64, ld=None):
    """The reference bench's loop through this library's launchers (column stride
    `ld`, default m)."""
    import torch
    m, n = a.shape
    ld = m if ld is None else ld
    tdt = torch.float64 if dtype == abi.F64 else torch.float32
    span = ld * (n - 1) + m
    wl, vl, cl = abi.layout([m, n], [1, ld]), abi.layout([n]), abi.layout([steps])
    packed_l = abi.layout([m, n], [1, 0])
    d_w = to_strided(a, ld, tdt)
    d_perm = torch.zeros(n, dtype=torch.int64, device="cuda")
    d_norms = torch.zeros(n, dtype=tdt, device="cuda")
    d_piv = torch.zeros(1, dtype=torch.int64, device="cuda")
    d_st = torch.zeros(1, dtype=torch.int64, device="cuda")
    d_coeff = torch.zeros(steps, dtype=tdt, device="cuda")
    d_packed = torch.zeros(m, dtype=tdt, device="cuda")
    s = t4.stream_handle()
    pivots = []
    t4.launch_rrqr("initialize_permutation", t4.plan_rrqr("initialize_permutation", n, n), s, vp(d_perm),
                   ctypes.c_longlong(n), ctypes.c_longlong(n))
    for step in range(steps):
        st = ctypes.c_longlong(step)
        t4.launch_rrqr("column_norms", t4.plan_rrqr("column_norms", dtype, wl, span, vl, n, step), s, vp(d_w),
                       vp(d_norms), ctypes.c_int(dtype), wl, vl, st)
        t4.launch_rrqr("select_pivot", t4.plan_rrqr("select_pivot", dtype, vl, n, vl, n, 1, 1, step), s,
                       vp(d_norms), vp(d_perm), vp(d_piv), vp(d_st), ctypes.c_int(dtype), vl, vl, st)
        pivots.append(d_piv.clone())
        t4.launch_rrqr("swap_columns", t4.plan_rrqr("swap_columns", dtype, wl, span, vl, n, 1, step), s, vp(d_w),
                       vp(d_perm), vp(d_piv), ctypes.c_int(dtype), wl, vl, st)
        t4.launch_rrqr("reflector", t4.plan_rrqr("reflector", dtype, wl, span, cl, steps, step), s, vp(d_w),
                       vp(d_coeff), ctypes.c_int(dtype), wl, cl, st)
        if n - step - 1 > 0:
            d_packed.copy_(d_w[step * ld:step * ld + m])
            t4.launch_rrqr("apply_reflector",
                           t4.plan_rrqr("apply_reflector", dtype, packed_l, m, wl, span, cl, steps, step, step + 1,
                                        n - step - 1), s,
                           vp(d_packed), vp(d_w), vp(d_coeff), ctypes.c_int(dtype), packed_l, wl, cl, st,
                           ctypes.c_longlong(step + 1), ctypes.c_longlong(n - step - 1))
    torch.cuda.synchronize()
    return (from_strided(d_w, m, n, ld), d_perm.cpu().numpy(), d_coeff.cpu().numpy(),
            np.array([int(p.item()) for p in pivots]))


def to_strided(a, ld, tdt):
    """Column-major device copy of `a` with column stride `ld` (padding rows NaN)."""
    import torch
    m, n = a.shape
    buf = np.full((n, ld), np.nan, dtype=a.dtype)
    buf[:, :m] = a.T
    return torch.from_numpy(buf.ravel()[:ld * (n - 1) + m].copy()).to(tdt).cuda()


def from_strided(d_w, m, n, ld):
    flat = d_w.cpu().numpy()
    return np.stack([flat[c * ld:c * ld + m] for c in range(n)], axis=1)


def fused_rrqr(a, steps, dtype=abi.F64, ld=None):
    import torch
    m, n = a.shape
    ld = m if ld is None else ld
    tdt = torch.float64 if dtype == abi.F64 else torch.float32
    d_w = to_strided(a, ld, tdt)
    t = torch.as_strided(d_w, (m, n), (1, ld))
    perm, coeff, pivots, status = t4.rrqr(t, steps)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return from_strided(d_w, m, n, ld), perm.cpu().numpy(), coeff.cpu().numpy()[:steps], pivots.cpu().numpy()[:steps]


@pytest.mark.parametrize("m,n,rank", [(600, 40, 10), (4096, 96, 24)])
def test_rrqr_loop_matches_oracle_bit_for_bit(cuda, m, n, rank):
    a = config5_matrix(m, n, rank, seed=m + n)
    steps = min(m, n)
    w_o, perm_o, coeff_o, _ = oracle_rrqr(a, steps)
    w_p, perm_p, coeff_p, piv_p = primitives_rrqr(a, steps)
    w_f, perm_f, coeff_f, piv_f = fused_rrqr(a, steps)
    assert np.array_equal(perm_p, perm_o) and np.array_equal(perm_f, perm_o)
    assert np.array_equal(piv_f, piv_p)
    assert np.array_equal(coeff_p.view(np.uint64), coeff_o.view(np.uint64))
    assert np.array_equal(coeff_f.view(np.uint64), coeff_o.view(np.uint64))
    assert np.array_equal(np.asarray(w_p, order="F").view(np.uint64), np.asarray(w_o, order="F").view(np.uint64))
    assert np.array_equal(np.asarray(w_f, order="F").view(np.uint64), np.asarray(w_o, order="F").view(np.uint64))


def test_rrqr_config5_full_size(cuda):
    """BASELINE config 5 at full size: A = U V^T + 1e-10 N, U [65536,64], V [256,64],
    256 steps.  The fused loop's pivots, permutation, coefficients and matrix equal the
    oracle's bit for bit, and the prefix rank at rtol 1e-8 is 64."""
    m, n, rank = 65536, 256, 64
    a = config5_matrix(m, n, rank, seed=10)
    w_o, perm_o, coeff_o, rank_o = oracle_rrqr(a, n)
    w_f, perm_f, coeff_f, piv_f = fused_rrqr(a, n)
    assert rank_o == 64
    assert np.array_equal(perm_f, perm_o)
    assert np.array_equal(coeff_f.view(np.uint64), coeff_o.view(np.uint64))
    assert np.array_equal(np.asarray(w_f, order="F").view(np.uint64), np.asarray(w_o, order="F").view(np.uint64))


@pytest.mark.parametrize("m,n,dtype,ld", [(1001, 40, abi.F64, 1001), (1001, 40, abi.F64, 1003),
                                          (777, 33, abi.F32, 777), (9001, 24, abi.F32, 9003),
                                          (20001, 12, abi.F64, 20001)])
def test_rrqr_loop_odd_rows_and_strides(cuda, m, n, dtype, ld):
    """Odd row counts and padded column strides put the pivot column and the trailing
    columns at different addresses modulo 16, so the chain passes' aligned bulk spans
    and their plain-load edges differ per operand: the fused loop still equals the
    loop of primitives bit for bit (and the oracle, for F64)."""
    a = config5_matrix(m, n, 8, seed=m + ld)
    if dtype == abi.F32:
        a = a.astype(np.float32)
    steps = min(m, n)
    w_p, perm_p, coeff_p, piv_p = primitives_rrqr(a, steps, dtype, ld)
    w_f, perm_f, coeff_f, piv_f = fused_rrqr(a, steps, dtype, ld)
    assert np.array_equal(perm_f, perm_p) and np.array_equal(piv_f, piv_p)
    assert np.array_equal(coeff_f, coeff_p) and np.array_equal(coeff_f.view(np.uint8), coeff_p.view(np.uint8))
    assert np.array_equal(w_f.view(np.uint8), w_p.view(np.uint8))
    if dtype == abi.F64:
        w_o, perm_o, coeff_o, _ = oracle_rrqr(a, steps)
        assert np.array_equal(perm_f, perm_o)
        assert np.array_equal(coeff_f.view(np.uint64), coeff_o.view(np.uint64))
        assert np.array_equal(np.ascontiguousarray(w_f).view(np.uint64), np.ascontiguousarray(w_o).view(np.uint64))


@pytest.mark.parametrize("m,n,steps,dtype", [(600, 40, 13, abi.F64), (777, 33, 1, abi.F32), (2048, 64, 63, abi.F64)])
def test_rrqr_partial_factorization(cuda, m, n, steps, dtype):
    """Fewer steps than min(m, n): the last column pass updates the trailing columns
    without the next step's norms and pivot; matrix, permutation, pivots and
    coefficients equal the loop of primitives run for the same steps, bit for bit."""
    a = config5_matrix(m, n, 6, seed=m + steps)
    if dtype == abi.F32:
        a = a.astype(np.float32)
    w_p, perm_p, coeff_p, piv_p = primitives_rrqr(a, steps, dtype)
    w_f, perm_f, coeff_f, piv_f = fused_rrqr(a, steps, dtype)
    assert np.array_equal(perm_f, perm_p) and np.array_equal(piv_f, piv_p)
    assert np.array_equal(coeff_f.view(np.uint8), coeff_p.view(np.uint8))
    assert np.array_equal(w_f.view(np.uint8), w_p.view(np.uint8))


@pytest.mark.parametrize("dtype,offset", [(abi.F64, 1), (abi.F32, 1), (abi.F32, 3)])
def test_rrqr_loop_unaligned_base(cuda, dtype, offset):
    """A matrix that starts `offset` elements past a 16-byte boundary: the chain
    passes' aligned copies must not reach before the matrix, so the first column's
    leading elements are loaded one by one; the results still equal the loop of
    primitives (on an aligned copy) bit for bit."""
    import torch
    m, n = 1003, 24
    a = config5_matrix(m, n, 6, seed=5 + offset)
    if dtype == abi.F32:
        a = a.astype(np.float32)
    tdt = torch.float64 if dtype == abi.F64 else torch.float32
    w_p, perm_p, coeff_p, piv_p = primitives_rrqr(a, n, dtype)
    flat = torch.from_numpy(np.asfortranarray(a).ravel(order="K").copy()).to(tdt)
    buf = torch.cat([torch.full((offset,), float("nan"), dtype=tdt), flat]).cuda()
    t = torch.as_strided(buf, (m, n), (1, m), storage_offset=offset)
    assert t.data_ptr() % 16 != 0
    perm, coeff, pivots, status = t4.rrqr(t, n)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    w_f = from_strided(buf[offset:], m, n, m)
    assert np.array_equal(perm.cpu().numpy(), perm_p) and np.array_equal(pivots.cpu().numpy()[:n], piv_p)
    assert np.array_equal(coeff.cpu().numpy()[:n].view(np.uint8), coeff_p.view(np.uint8))
    assert np.array_equal(w_f.view(np.uint8), w_p.view(np.uint8))
    assert torch.isnan(buf[:offset]).all()


def test_rrqr_loop_special_values(cuda):
    """Integer entries (exact quotients, powers of two, ties in the pivot norms) and a
    tiny and a huge column (operands outside the fast quotient's range): the fused loop
    still equals the oracle and the loop of primitives bit for bit."""
    rng = np.random.default_rng(77)
    m, n = 2048, 48
    a = np.asfortranarray(rng.integers(-3, 4, (m, n)).astype(np.float64))
    a[:, 5] *= 1e-290
    a[:, 7] *= 1e280
    steps = n
    w_o, perm_o, coeff_o, _ = oracle_rrqr(a, steps)
    w_p, perm_p, coeff_p, piv_p = primitives_rrqr(a, steps)
    w_f, perm_f, coeff_f, piv_f = fused_rrqr(a, steps)
    assert np.array_equal(perm_p, perm_o) and np.array_equal(perm_f, perm_o)
    assert np.array_equal(piv_f, piv_p)
    assert np.array_equal(coeff_f.view(np.uint64), coeff_o.view(np.uint64))
    assert np.array_equal(np.asarray(w_p, order="F").view(np.uint64), np.asarray(w_o, order="F").view(np.uint64))
    assert np.array_equal(np.asarray(w_f, order="F").view(np.uint64), np.asarray(w_o, order="F").view(np.uint64))


# ---- general-rank twins (`_any`) ----------------------------------------------

def rrqr_loop(dtype, mats, steps, mode):
    """The reference bench's loop of primitives over a batch of matrices ([m, n, B]
    layouts, batch axis last), then extract_r and prefix_rank.  mode "fast": this
    library's launchers with the planners' geometry; "any-launcher" / "any-module":
    the general-rank twins (launchers / module symbols) on the same layouts padded to
    rank 9-10 with trailing extent-1 axes, on t4a_rrqr_any_geometry."""
    import torch
    B = len(mats)
    m, n = mats[0].shape[1], mats[0].shape[0]
    es = np.dtype(NP[dtype]).itemsize
    rdt = np.float32 if dtype in (abi.F32, abi.C32) else np.float64
    work = np.concatenate([mt.ravel() for mt in mats])
    d_w = dev(work)
    d_norms = dev(np.zeros(n * B, rdt))
    d_perm = dev(np.zeros(n * B, np.int64))
    d_piv = dev(np.zeros(B, np.int64))
    d_st = dev(np.zeros(B, np.int64))
    d_coeff = dev(np.zeros(steps * B, NP[dtype]))
    d_packed = dev(np.zeros(m * B, NP[dtype]))
    k = min(m, n)
    d_r = dev(np.zeros(k * n * B, NP[dtype]))
    d_rank, d_rst = dev(np.zeros(B, np.int64)), dev(np.zeros(B, np.int64))
    shapes = {"w": ([m, n, B], [1, m, m * n]), "v": ([n, B], [1, n]), "c": ([steps, B], [1, steps]),
              "p": ([m, n, B], [1, 0, m]), "r": ([k, n, B], [1, k, k * n])}
    keep = []

    def lay(key):
        ext, st = shapes[key]
        if mode == "fast":
            return abi.layout(ext, st)
        pad = 10 - len(ext) if key in ("w", "p", "r") else 9 - len(ext)
        la, arr = t4.layout_any(ext + [1] * pad, st + [0] * pad)
        keep.append(arr)
        return la
    wl, vl, cl, pk, rl = lay("w"), lay("v"), lay("c"), lay("p"), lay("r")
    fl = {"w": abi.layout(*shapes["w"]), "v": abi.layout(*shapes["v"]), "c": abi.layout(*shapes["c"]),
          "p": abi.layout(*shapes["p"]), "r": abi.layout(*shapes["r"])}
    s = t4.stream_handle()

    def run(name, plan_args, tasks, is_flat, args):
        if mode == "fast":
            t4.launch_rrqr(name, t4.plan_rrqr(name, *plan_args), s, *args)
        else:
            g = t4.rrqr_any_geometry(tasks, is_flat)
            if mode == "any-launcher":
                t4.launch_rrqr(name + "_any", g, s, *args)
            elif g.grid[0] > 0:
                module(OUR_CUBIN).launch("t4a_cuda_" + name + "_any", tuple(g.grid), tuple(g.block), 0, list(args))
    t4.launch_rrqr("initialize_permutation", t4.plan_rrqr("initialize_permutation", n, n * B), s, vp(d_perm),
                   ctypes.c_longlong(n), ctypes.c_longlong(n * B))
    span = m * n * B
    for step in range(steps):
        st = ctypes.c_longlong(step)
        run("column_norms", (dtype, fl["w"], span, fl["v"], n * B, step), B * (n - step), False,
            [vp(d_w), vp(d_norms), ctypes.c_int(dtype), wl, vl, st])
        pdt = abi.F32 if rdt == np.float32 else abi.F64
        run("select_pivot", (pdt, fl["v"], n * B, fl["v"], n * B, B, B, step), B, False,
            [vp(d_norms), vp(d_perm), vp(d_piv), vp(d_st), ctypes.c_int(pdt), vl, vl, st])
        run("swap_columns", (dtype, fl["w"], span, fl["v"], n * B, B, step), m * B, True,
            [vp(d_w), vp(d_perm), vp(d_piv), ctypes.c_int(dtype), wl, vl, st])
        run("reflector", (dtype, fl["w"], span, fl["c"], steps * B, step), B, False,
            [vp(d_w), vp(d_coeff), ctypes.c_int(dtype), wl, cl, st])
        if n - step - 1 > 0:
            wv = d_w[:span * es].view(torch.uint8)
            for b in range(B):
                src = wv[(b * m * n + step * m) * es:(b * m * n + step * m + m) * es]
                d_packed[b * m * es:(b + 1) * m * es].copy_(src)
            run("apply_reflector", (dtype, fl["p"], m * B, fl["w"], span, fl["c"], steps * B, step, step + 1,
                                    n - step - 1), B * (n - step - 1), False,
                [vp(d_packed), vp(d_w), vp(d_coeff), ctypes.c_int(dtype), pk, wl, cl, st,
                 ctypes.c_longlong(step + 1), ctypes.c_longlong(n - step - 1)])
    run("extract_r", (dtype, fl["w"], span, fl["r"], k * n * B), k * n * B, True,
        [vp(d_w), vp(d_r), ctypes.c_int(dtype), wl, rl])
    run("prefix_rank", (dtype, fl["r"], k * n * B, B, B, 1e-8, 0.0), B, False,
        [vp(d_r), vp(d_rank), vp(d_rst), ctypes.c_int(dtype), rl, ctypes.c_double(1e-8), ctypes.c_double(0.0)])
    torch.cuda.synchronize()
    out = (host(d_w, span * es, NP[dtype]), host(d_perm, n * B * 8, np.int64), host(d_coeff, steps * B * es, NP[dtype]),
           host(d_piv, B * 8, np.int64), host(d_r, k * n * B * es, NP[dtype]), host(d_rank, B * 8, np.int64))
    del keep
    return out


@pytest.mark.parametrize("mode", ["any-launcher", "any-module"])
@pytest.mark.parametrize("dtype", [abi.F64, abi.F32, abi.C64])
def test_any_twins_match_the_fast_primitives(cuda, mode, dtype):
    """Two batched matrices, rank-10 layouts: the general-rank twins give the fast
    primitives' results (bit for bit for F32/F64; complex within 1e-12 relative to the
    column scale, as the complex product's contraction may differ between kernels)."""
    rng = np.random.default_rng(60 + int(dtype))
    m, n, steps = 300, 24, 20
    mats = [rand_matrix(rng, dtype, m, n), rand_matrix(rng, dtype, m, n, shift=0.5)]
    fast = rrqr_loop(dtype, mats, steps, "fast")
    got = rrqr_loop(dtype, mats, steps, mode)
    for name, a, b in zip(["work", "perm", "coeff", "pivots", "R", "rank"], got, fast):
        if name in ("perm", "pivots", "rank") or dtype in (abi.F32, abi.F64):
            assert np.array_equal(np.asarray(a).view(np.uint8), np.asarray(b).view(np.uint8)), name
        else:
            assert same(dtype, a, b), name


# ---- RRQR epilogue: identity_shifted and Q formation ---------------------------------

IDENTITY_CASES = [  # the reference's own cases (tests/gpu_linalg_aux.rs:1153-1185), then batched ones
    (abi.F64, [4, 3], [1, 5], 1, 0), (abi.F64, [3, 2], [1, 3], 0, 2), (abi.F32, [3, 2], [1, 3], 0, 2),
    (abi.I32, [3, 2], [1, 3], 0, 0), (abi.I64, [3, 2], [1, 3], 0, 1), (abi.C32, [5, 3, 2], [1, 5, 15], 0, 1),
    (abi.C64, [4, 4, 3], [2, 8, 40], 1, 0), (abi.F64, [1000, 300], [1, 1003], 5, 0),
]


@pytest.mark.parametrize("route", ["launcher", "module", "module-refgeom", "reference", "any-launcher", "any-module"])
def test_identity_shifted(cuda, route):
    """Every route writes the oracle's shifted identity bit for bit and leaves the
    strided layout's holes untouched; `_any` routes run the layouts padded to rank 10."""
    import torch
    for dtype, ext, st, off, start in IDENTITY_CASES:
        es = np.dtype(NP[dtype]).itemsize
        span = off + sum((e - 1) * x for e, x in zip(ext, st)) + 1
        lay = abi.layout(ext, st, off)
        want = np.full(span, 7, NP[dtype])
        assert oracle.lib().t4a_oracle_identity_shifted(dtype, oracle.ptr(want), ctypes.byref(lay), start) == 0
        d = dev(np.full(span, 7, NP[dtype]))
        count = int(np.prod(ext))
        args = [vp(d), ctypes.c_int(dtype), lay, ctypes.c_longlong(start)]
        if route == "launcher":
            t4.launch_rrqr("identity_shifted", t4.plan_rrqr("identity_shifted", dtype, lay, span, start),
                           t4.stream_handle(), *args)
        elif route in ("module", "module-refgeom", "reference"):
            plan = t4.plan_rrqr("identity_shifted", dtype, lay, span, start)
            geom = (tuple(plan.grid), tuple(plan.block), 0) if route == "module" else flat(count)
            module(REF_LINALG if route == "reference" else OUR_LINALG).launch("t4a_cuda_identity_shifted", *geom,
                                                                               args)
        else:
            pad = 10 - len(ext)
            la, keep = t4.layout_any(ext + [1] * pad, st + [0] * pad, off)
            g = t4.rrqr_any_geometry(count, True)
            any_args = [vp(d), ctypes.c_int(dtype), la, ctypes.c_longlong(start)]
            if route == "any-launcher":
                t4.launch_rrqr("identity_shifted_any", g, t4.stream_handle(), *any_args)
            else:
                module(OUR_LINALG).launch("t4a_cuda_identity_shifted_any", tuple(g.grid), tuple(g.block), 0,
                                          any_args)
        torch.cuda.synchronize()
        got = host(d, span * es, NP[dtype])
        assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (route, dtype, ext, start)


def oracle_form_q(work, coeff, dtype, k):
    """The reference bench's Q formation on the oracle: identity, then apply_reflector
    for step = k-1 .. 0 over all k columns (work: column-major [m, n] host array)."""
    m, n = work.shape
    w = np.asfortranarray(work)
    q = np.zeros((m, k), NP[dtype], order="F")
    wl, ql, cl = abi.layout([m, n]), abi.layout([m, k]), abi.layout([k])
    assert oracle.lib().t4a_oracle_identity_shifted(dtype, oracle.ptr(q.ravel(order="K")), ctypes.byref(ql), 0) == 0
    c = np.ascontiguousarray(coeff[:k])
    for step in range(k - 1, -1, -1):
        assert oracle.lib().t4a_oracle_apply_reflector(dtype, oracle.ptr(w.ravel(order="K")),
                                                       oracle.ptr(q.ravel(order="K")), oracle.ptr(c),
                                                       ctypes.byref(wl), ctypes.byref(ql), ctypes.byref(cl), step, 0,
                                                       k, THREADS) == 0
    return q


@pytest.mark.parametrize("dtype", [abi.F64, abi.F32])
@pytest.mark.parametrize("m,n,k", [(300, 24, 24), (517, 40, 13)])
def test_form_q_matches_the_oracle(cuda, dtype, m, n, k):
    """t4a_rrqr_form_q after the fused factorization equals the oracle's loop bit for
    bit, and Q is orthonormal with Q R = A P on the factorized columns."""
    import torch
    rng = np.random.default_rng(m + n + k + dtype)
    a = np.asfortranarray(rng.standard_normal((m, n)).astype(NP[dtype]))
    tdt = torch.float64 if dtype == abi.F64 else torch.float32
    d_w = to_strided(a, m, tdt)
    t = torch.as_strided(d_w, (m, n), (1, m))
    perm, coeff, _, status = t4.rrqr(t, k)
    q, qst = t4.rrqr_form_q(t, coeff[:k])
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and int(qst.item()) == 0
    work = from_strided(d_w, m, n, m)
    want = oracle_form_q(work, coeff.cpu().numpy(), dtype, k)
    got = q.cpu().numpy()
    assert np.array_equal(np.ascontiguousarray(got).view(np.uint8), np.ascontiguousarray(want).view(np.uint8))
    eps = 1e-12 if dtype == abi.F64 else 2e-5
    q64 = got.astype(np.float64)
    assert np.abs(q64.T @ q64 - np.eye(k)).max() < eps * m
    r = np.triu(work[:k, :].astype(np.float64))
    ap = a.astype(np.float64)[:, perm.cpu().numpy()]
    assert np.abs(q64 @ r - ap)[:, :k].max() < eps * m * np.abs(a).max()


def unitary_reflectors(m, k, dtype, seed):
    """Column-major work [m, k] whose column s holds a reflector's tail below row s, and
    coefficients with I - c v v^H unitary: c = (1 + e^{i theta}) / (v^H v) (real dtypes:
    theta = 0, c = 2 / (v^H v))."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((m, k))
    if dtype in (abi.C32, abi.C64):
        w = w + 1j * rng.standard_normal((m, k))
    c = np.zeros(k, np.complex128 if dtype in (abi.C32, abi.C64) else np.float64)
    for s in range(k):
        vv = 1.0 + float(np.sum(np.abs(w[s + 1:, s]) ** 2))
        c[s] = (1 + np.exp(1j * rng.uniform(0, 2 * np.pi))) / vv if np.iscomplexobj(c) else 2.0 / vv
    return np.asfortranarray(w.astype(NP[dtype])), c.astype(NP[dtype])


@pytest.mark.parametrize("dtype,m,k", [(abi.C64, 300, 24), (abi.C64, 3000, 16), (abi.C32, 517, 13),
                                       (abi.F64, 4096, 16), (abi.F64, 300, 24)])
def test_form_q_primitive_route_matches_the_oracle(cuda, dtype, m, k):
    """t4a_rrqr_form_q without a status word (and for complex types, which the column
    pass does not take) runs identity_shifted and apply_reflector for step = k-1 .. 0 as
    planned launches.  Against the oracle's loop: F32/F64 bit for bit; C32/C64 within
    rounding (the oracle's complex sums are not contracted like the device's).  Q is
    unitary for these coefficients."""
    import torch
    w, c = unitary_reflectors(m, k, dtype, seed=m + k + dtype)
    es = np.dtype(NP[dtype]).itemsize
    d_w, d_c = dev(w.ravel(order="K")), dev(c)
    d_q = sentinel_dev(m * k * es)
    wl, ql, cl = abi.layout([m, k]), abi.layout([m, k]), abi.layout([k])
    t4.check(t4.lib().t4a_rrqr_form_q(t4.stream_handle(), dtype, vp(d_w), ctypes.byref(wl), m * k, vp(d_c),
                                      ctypes.byref(cl), k, vp(d_q), ctypes.byref(ql), m * k, None), "form_q")
    torch.cuda.synchronize()
    got = host(d_q, m * k * es, NP[dtype]).reshape(k, m).T
    want = oracle_form_q(w, c, dtype, k)
    if dtype in (abi.F32, abi.F64):
        assert np.array_equal(np.ascontiguousarray(got).view(np.uint8), np.ascontiguousarray(want).view(np.uint8))
    else:
        tol = 1e-12 if dtype == abi.C64 else 2e-5
        assert np.abs(got - want).max() <= tol * np.sqrt(m) * k
    q = got.astype(np.complex128)
    assert np.abs(q.conj().T @ q - np.eye(k)).max() < (1e-12 if dtype in (abi.F64, abi.C64) else 1e-4) * m


def test_form_q_config5_properties(cuda):
    """BASELINE config 5 at full size (m 65536, 256 reflectors): the Q formation's Q is
    orthonormal and Q R equals A P, checked on the GPU in F64."""
    import torch
    m, n, rank = 65536, 256, 64
    a = config5_matrix(m, n, rank, seed=10)
    d_w = to_strided(a, m, torch.float64)
    t = torch.as_strided(d_w, (m, n), (1, m))
    perm, coeff, _, status = t4.rrqr(t, n)
    q, qst = t4.rrqr_form_q(t, coeff)
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and int(qst.item()) == 0
    eye = torch.eye(n, dtype=torch.float64, device="cuda")
    assert float((q.T @ q - eye).abs().max()) < 1e-12
    r = torch.triu(t[:n, :])
    ap = torch.from_numpy(np.ascontiguousarray(a)).cuda()[:, perm]
    assert float((q @ r - ap).abs().max()) < 1e-12 * float(ap.abs().max()) * 100
