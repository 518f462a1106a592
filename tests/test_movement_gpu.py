"""GPU parity of the strided movement entries (bit-exact against the CPU oracle).

Covers BASELINE config 2 at full size (F32 [64]^4 permuted (3,1,0,2), C64 [16]^6
permuted (5,0,4,1,3,2), F32 [64]^4 with axis 2 reversed), random permutations,
offsets and negative strides over every dtype, tiled_transpose, broadcast_in_dim,
copy_exact, contiguous_to_view and the zero fills, through this library's launchers
and through its exported module symbols (with the planner's geometry and with the
reference's flat geometry, grid ceil(len/256) x 256).  Destinations are
sentinel-filled with guard bytes, as in the reference tests.
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
OUR_CUBIN = os.path.join(ROOT, "t4a-cuda-kernels_b200", "t4a_b200", "lib", "movement.cubin")
SENTINEL, GUARD = 0xCD, 256
THREADS = os.cpu_count() or 4
ESIZE = {abi.F32: 4, abi.F64: 8, abi.I32: 4, abi.I64: 8, abi.BOOL: 1, abi.C32: 8, abi.C64: 16}


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


def oracle_copy(dtype, src_bytes, src_l, dst_l, dst_nbytes):
    dst = np.full(dst_nbytes, SENTINEL, dtype=np.uint8)
    rc = oracle.lib().t4a_oracle_strided_to_strided(dtype, oracle.ptr(dst), oracle.ptr(src_bytes),
                                                    ctypes.byref(src_l), ctypes.byref(dst_l), THREADS)
    assert rc == 0
    return dst


def span_of(l):
    hi = l.offset + sum((e - 1) * s for e, s in zip(l.extents_list(), l.strides_list()) if s > 0)
    return hi + 1


def gpu_copy(route, dtype, src_bytes, src_l, dst_l, dst_nbytes, module=None, base=0):
    """strided_to_strided by `route`; `base` shifts both device buffers by that many
    bytes from the allocation's (256-byte aligned) start."""
    import torch
    es = ESIZE[dtype]
    src = dev(np.concatenate([np.zeros(base, np.uint8), src_bytes]))[base:]
    dst = sentinel(dst_nbytes + base)[base:]
    src_len, dst_len = len(src_bytes) // es, dst_nbytes // es
    n = src_l.count()
    if route == "launcher":
        t4.copy_strided_raw(t4.stream_handle(), dtype, ctypes.c_void_p(dst.data_ptr()), dst_l, dst_len,
                            ctypes.c_void_p(src.data_ptr()), src_l, src_len)
    else:
        if route == "module":
            launch = t4.plan_strided_to_strided(dtype, src_l, src_len, dst_l, dst_len)
            geom = (tuple(launch.grid), tuple(launch.block), launch.shared_bytes)
        else:
            geom = ((max(1, (n + 255) // 256),), (256,), 0)
        if n > 0:
            module.launch("t4a_cuda_strided_to_strided", *geom, [
                ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(src.data_ptr()), ctypes.c_int(dtype), src_l, dst_l,
                ctypes.c_longlong(n)])
    torch.cuda.synchronize()
    return take(dst, dst_nbytes)


def permuted_view(shape, perm, esize_strides=None):
    """Source layout of `x.transpose(perm)` for a compact NumPy array x of `shape`."""
    st, s = [], 1
    for e in reversed(shape):
        st.insert(0, s)
        s *= e
    out_shape = [shape[p] for p in perm]
    return abi.numpy_layout(out_shape, [st[p] for p in perm]), out_shape


def check_config_case(dtype, nbytes_elem, src_l, rng):
    n = src_l.count()
    src = rng.integers(0, 256, size=n * nbytes_elem, dtype=np.uint8)
    dst_l = abi.layout(src_l.extents_list())
    want = oracle_copy(dtype, src, src_l, dst_l, n * nbytes_elem)
    got = gpu_copy("launcher", dtype, src, src_l, dst_l, n * nbytes_elem)
    assert np.array_equal(want, got)


def test_config2a_f32_permutation(cuda):
    l, _ = permuted_view([64] * 4, (3, 1, 0, 2))
    check_config_case(abi.F32, 4, l, np.random.default_rng(2))


def test_config2b_c64_permutation(cuda):
    l, _ = permuted_view([16] * 6, (5, 0, 4, 1, 3, 2))
    check_config_case(abi.C64, 16, l, np.random.default_rng(3))


def test_config2c_f32_reversal(cuda):
    # NumPy axis 2 reversed: stride -64 and the offset rebased to the last row.
    l = abi.numpy_layout([64] * 4, [64 ** 3, 64 ** 2, -64, 1], 63 * 64)
    check_config_case(abi.F32, 4, l, np.random.default_rng(4))


def random_case(rng, dtype):
    rank = int(rng.integers(1, 7))
    shape = [int(rng.integers(1, 9 if rank > 3 else 70)) for _ in range(rank)]
    perm = list(rng.permutation(rank))
    es = ESIZE[dtype]
    base = int(rng.integers(0, 5))
    src_l, out_shape = permuted_view(shape, perm)
    st = src_l.strides_list()
    ext = src_l.extents_list()
    off = base
    # Reverse a random axis (negative stride, offset rebased).
    if rank > 1 and rng.random() < 0.5:
        a = int(rng.integers(0, rank))
        off += (ext[a] - 1) * st[a]
        st[a] = -st[a]
    src_l = abi.layout(ext, st, off)
    total = int(np.prod(shape)) + base
    src = rng.integers(0, 256, size=total * es, dtype=np.uint8)
    # Destination: compact, or a padded view with a gap per row.
    if rng.random() < 0.5:
        dst_l = abi.layout(ext)
    else:
        pad = int(rng.integers(1, 4))
        dst_st, s = [], 1
        for e in ext:
            dst_st.append(s)
            s *= e + (pad if len(dst_st) == 1 else 0)
        dst_l = abi.layout(ext, dst_st, pad)
    return src, src_l, dst_l, span_of(dst_l) * es


@pytest.mark.parametrize("route", ["launcher", "module", "module-refgeom"])
@pytest.mark.parametrize("dtype", [abi.BOOL, abi.F32, abi.I64, abi.C32, abi.C64])
def test_random_strided_copies(cuda, route, dtype):
    rng = np.random.default_rng(100 + dtype)
    module = Module(OUR_CUBIN) if route != "launcher" else None
    for _ in range(40):
        src, src_l, dst_l, dst_nbytes = random_case(rng, dtype)
        want = oracle_copy(dtype, src, src_l, dst_l, dst_nbytes)
        got = gpu_copy(route, dtype, src, src_l, dst_l, dst_nbytes, module)
        assert np.array_equal(want, got), (src_l, dst_l)


@pytest.mark.parametrize("m,n,batches,offset", [(4096, 4096, 1, 0), (4093, 4099, 1, 5), (256, 256, 64, 0),
                                                (1, 777, 3, 2), (33, 1, 2, 0), (100, 300, 7, 11)])
@pytest.mark.parametrize("dtype", [abi.F32, abi.F64, abi.C64])
def test_tiled_transpose(cuda, m, n, batches, offset, dtype):
    import torch
    es = ESIZE[dtype]
    rng = np.random.default_rng(m * 7 + n + batches)
    total = offset + m * n * batches
    src = rng.integers(0, 256, size=total * es, dtype=np.uint8)
    want = np.full(m * n * batches * es, SENTINEL, dtype=np.uint8)
    assert oracle.lib().t4a_oracle_tiled_transpose(dtype, oracle.ptr(want), oracle.ptr(src), offset, m * n, m, n,
                                                   batches, THREADS) == 0
    cfg = abi.transpose_config()
    launch = t4.plan_tiled_transpose(dtype, cfg, offset, m * n, m, n, batches, total, m * n * batches)
    for route in ["launcher", "module"]:
        d_src, d_dst = dev(src), sentinel(m * n * batches * es)
        if route == "launcher":
            t4.check(t4.lib().t4a_launch_tiled_transpose(ctypes.byref(launch), t4.stream_handle(),
                                                         ctypes.c_void_p(d_dst.data_ptr()),
                                                         ctypes.c_void_p(d_src.data_ptr()), dtype, offset, m * n, m, n,
                                                         cfg))
        else:
            Module(OUR_CUBIN).launch("t4a_cuda_tiled_transpose", tuple(launch.grid), tuple(launch.block),
                                     launch.shared_bytes, [
                                         ctypes.c_void_p(d_dst.data_ptr()), ctypes.c_void_p(d_src.data_ptr()),
                                         ctypes.c_int(dtype), ctypes.c_longlong(offset), ctypes.c_longlong(m * n),
                                         ctypes.c_longlong(m), ctypes.c_longlong(n), cfg])
        torch.cuda.synchronize()
        assert np.array_equal(want, take(d_dst, m * n * batches * es)), route


@pytest.mark.parametrize("out_shape,in_shape,dims", [
    ([8192, 8192], [8192], [0]),            # NumPy [8192] -> [8192, 8192] along rows (ref dims)
    ([7, 5, 3], [7, 1], [0, 2]),
    ([4, 6], [], []),
    ([16, 3, 9], [9, 16], [2, 0]),
])
@pytest.mark.parametrize("dtype", [abi.F32, abi.C64])
def test_broadcast_in_dim(cuda, out_shape, in_shape, dims, dtype):
    """Shapes here are reference order (axis 0 fastest)."""
    import torch
    es = ESIZE[dtype]
    out_l = abi.layout(out_shape)
    in_l = abi.layout(in_shape)
    n_in, n_out = max(1, in_l.count()), out_l.count()
    rng = np.random.default_rng(n_out)
    src = rng.integers(0, 256, size=n_in * es, dtype=np.uint8)
    want = np.full(n_out * es, SENTINEL, dtype=np.uint8)
    av = abi.axis_values(dims)
    assert oracle.lib().t4a_oracle_broadcast_in_dim(dtype, oracle.ptr(want), oracle.ptr(src), ctypes.byref(out_l),
                                                    ctypes.byref(in_l), ctypes.byref(av), THREADS) == 0
    launch = t4.plan_broadcast_in_dim(dtype, out_l, n_out, in_l, n_in, dims)
    d_src, d_dst = dev(src), sentinel(n_out * es)
    t4.check(t4.lib().t4a_launch_broadcast_in_dim(ctypes.byref(launch), t4.stream_handle(),
                                                  ctypes.c_void_p(d_dst.data_ptr()), ctypes.c_void_p(d_src.data_ptr()),
                                                  dtype, out_l, in_l, av, n_out))
    torch.cuda.synchronize()
    assert np.array_equal(want, take(d_dst, n_out * es))


def test_copy_exact_view_copies_and_fills(cuda):
    import torch
    rng = np.random.default_rng(9)
    n = 1_000_003
    src = rng.integers(0, 256, size=n * 8, dtype=np.uint8)
    d_src, d_dst = dev(src), sentinel(n * 8)
    launch = t4.Launch()
    t4.check(t4.lib().t4a_plan_copy_exact(abi.F64, n, ctypes.byref(launch)))
    t4.check(t4.lib().t4a_launch_copy_exact(ctypes.byref(launch), t4.stream_handle(), ctypes.c_void_p(d_dst.data_ptr()),
                                            ctypes.c_void_p(d_src.data_ptr()), abi.F64, n))
    torch.cuda.synchronize()
    assert np.array_equal(src, take(d_dst, n * 8))
    # contiguous_to_view: a compact source scattered into a strided (reversed) view.
    view = abi.layout([1000, 1000], [2, -2000], 999 * 2000)
    dst_bytes = (999 * 2000 + 2 * 999 + 1) * 4
    src = rng.integers(0, 256, size=1000 * 1000 * 4, dtype=np.uint8)
    want = np.full(dst_bytes, SENTINEL, dtype=np.uint8)
    assert oracle.lib().t4a_oracle_contiguous_to_view(abi.F32, oracle.ptr(want), oracle.ptr(src), ctypes.byref(view),
                                                      THREADS) == 0
    launch = t4.plan_contiguous_to_view(abi.F32, view, dst_bytes // 4)
    d_src, d_dst = dev(src), sentinel(dst_bytes)
    t4.check(t4.lib().t4a_launch_contiguous_to_view(ctypes.byref(launch), t4.stream_handle(),
                                                    ctypes.c_void_p(d_dst.data_ptr()),
                                                    ctypes.c_void_p(d_src.data_ptr()), abi.F32, view, 10 ** 6))
    torch.cuda.synchronize()
    assert np.array_equal(want, take(d_dst, dst_bytes))
    # fill_zero_view zeroes exactly the view.
    d = sentinel(dst_bytes)
    launch = t4.Launch()
    t4.check(t4.lib().t4a_plan_fill_zero_view(abi.F32, ctypes.byref(view), dst_bytes // 4, ctypes.byref(launch)))
    t4.check(t4.lib().t4a_launch_fill_zero_view(ctypes.byref(launch), t4.stream_handle(), ctypes.c_void_p(d.data_ptr()),
                                                abi.F32, view, 10 ** 6))
    torch.cuda.synchronize()
    got = take(d, dst_bytes).view(np.uint32)
    mask = np.zeros(dst_bytes // 4, dtype=bool)
    idx = (999 * 2000 + 2 * np.arange(1000)[:, None] - 2000 * np.arange(1000)[None, :]).reshape(-1)
    mask[idx] = True
    assert (got[mask] == 0).all() and (got[~mask] == 0xCDCDCDCD).all()


# ---- general-rank twins (`_any`) ----------------------------------------------

ANY_EXTENTS = [2, 3, 2, 2, 1, 2, 3, 2, 2, 2]  # rank 10, 576 elements


def random_view(rng, extents):
    """Strides and offset of a bijective view of a compact buffer: a random storage
    order of the axes, one axis reversed (its stride negated, the offset rebased)."""
    strides, acc = [0] * len(extents), 1
    for d in rng.permutation(len(extents)):
        strides[d] = acc
        acc *= extents[d]
    offset = 0
    flip = int(rng.integers(len(extents)))
    if extents[flip] > 1:
        offset = (extents[flip] - 1) * strides[flip]
        strides[flip] = -strides[flip]
    return strides, offset, acc


def view_index(extents, strides, offset):
    """Element index of flat position f (axis 0 fastest) for every f."""
    n = int(np.prod(extents))
    f = np.arange(n, dtype=np.int64)
    idx = np.full(n, offset, dtype=np.int64)
    for e, s in zip(extents, strides):
        idx += (f % e) * s
        f //= e
    return idx


def any_launch(route, name, n, args):
    """One `_any` entry through the library launcher, or the module symbol under this
    library's geometry ("module") or the reference's ceil(n/256) x 256 ("refgeom")."""
    import torch
    if route == "launcher":
        t4.launch_movement_any(name, t4.movement_any_geometry(n), t4.stream_handle(), *args)
    else:
        if route == "module":
            g = t4.movement_any_geometry(n)
            geom = (tuple(g.grid), tuple(g.block), 0)
        else:
            geom = ((max(1, (n + 255) // 256),), (256,), 0)
        Module(OUR_CUBIN).launch("t4a_cuda_" + name + "_any", *geom, args)
    torch.cuda.synchronize()


ANY_ROUTES = ["launcher", "module", "refgeom"]


@pytest.mark.parametrize("route", ANY_ROUTES)
@pytest.mark.parametrize("dtype,base", [(abi.F32, 0), (abi.C64, 0), (abi.BOOL, 0), (abi.C32, 4), (abi.C64, 8)])
def test_any_twins_of_the_view_copies(cuda, route, dtype, base):
    """materialize_strided, contiguous_to_view, strided_to_strided and fill_zero_view
    over rank-10 layouts (random storage orders, a reversed axis, offsets), against the
    index arithmetic, with sentinel-guarded destinations.  `base` shifts every buffer
    off the allocation's alignment: complex64 is 4-byte and complex128 8-byte aligned in
    the ABI."""
    import torch
    es = ESIZE[dtype]

    def dev(buf):
        return globals()["dev"](np.concatenate([np.zeros(base, np.uint8), buf]))[base:]

    def sentinel(nbytes):
        return globals()["sentinel"](nbytes + base)[base:]
    rng = np.random.default_rng(int(dtype) * 7 + ANY_ROUTES.index(route))
    ext = ANY_EXTENTS
    n = int(np.prod(ext))
    s_str, s_off, total = random_view(rng, ext)
    d_str, d_off, _ = random_view(rng, ext)
    s_any, k1 = t4.layout_any(ext, s_str, s_off)
    d_any, k2 = t4.layout_any(ext, d_str, d_off)
    src = rng.integers(0, 256, size=total * es, dtype=np.uint8)
    src_e = src.reshape(total, es)
    s_idx, d_idx = view_index(ext, s_str, s_off), view_index(ext, d_str, d_off)
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    # materialize_strided: dst[f] = src[view(f)]
    d_src, d_dst = dev(src), sentinel(n * es)
    any_launch(route, "materialize_strided", n, [vp(d_dst), vp(d_src), ctypes.c_int(dtype), s_any, ctypes.c_longlong(n)])
    assert np.array_equal(take(d_dst, n * es).reshape(n, es), src_e[s_idx])
    # contiguous_to_view: dst[view(f)] = src[f]
    d_dst = sentinel(total * es)
    any_launch(route, "contiguous_to_view", n, [vp(d_dst), vp(d_src), ctypes.c_int(dtype), d_any, ctypes.c_longlong(n)])
    want = np.full((total, es), SENTINEL, dtype=np.uint8)
    want[d_idx] = src_e[:n]
    assert np.array_equal(take(d_dst, total * es).reshape(total, es), want)
    # strided_to_strided: dst[dst_view(f)] = src[src_view(f)]
    d_dst = sentinel(total * es)
    any_launch(route, "strided_to_strided", n, [vp(d_dst), vp(d_src), ctypes.c_int(dtype), s_any, d_any,
                                                ctypes.c_longlong(n)])
    want = np.full((total, es), SENTINEL, dtype=np.uint8)
    want[d_idx] = src_e[s_idx]
    assert np.array_equal(take(d_dst, total * es).reshape(total, es), want)
    # fill_zero_view: zeros exactly at the view
    d_dst = sentinel(total * es)
    any_launch(route, "fill_zero_view", n, [vp(d_dst), ctypes.c_int(dtype), d_any, ctypes.c_longlong(n)])
    want = np.full((total, es), SENTINEL, dtype=np.uint8)
    want[d_idx] = 0
    assert np.array_equal(take(d_dst, total * es).reshape(total, es), want)
    del k1, k2


@pytest.mark.parametrize("route", ANY_ROUTES)
@pytest.mark.parametrize("dtype", [abi.F64, abi.C64])
def test_any_twin_of_broadcast_in_dim(cuda, route, dtype):
    """broadcast_in_dim into a rank-10 compact destination from a rank-3 strided input
    mapped to destination axes (1, 5, 8), one of them broadcast (input extent 1)."""
    es = ESIZE[dtype]
    rng = np.random.default_rng(int(dtype) + 31 * ANY_ROUTES.index(route))
    out_ext = ANY_EXTENTS
    n = int(np.prod(out_ext))
    dims = [1, 5, 8]
    in_ext = [out_ext[1], 1, out_ext[8]]
    in_str, in_off, total = random_view(rng, in_ext)
    out_any, k1 = t4.layout_any(out_ext)
    in_any, k2 = t4.layout_any(in_ext, in_str, in_off)
    av, k3 = t4.axis_values_any(dims)
    src = rng.integers(0, 256, size=total * es, dtype=np.uint8)
    f = np.arange(n, dtype=np.int64)
    coords, rest = [], f.copy()
    for e in out_ext:
        coords.append(rest % e)
        rest //= e
    idx = np.full(n, in_off, dtype=np.int64)
    for a, d in enumerate(dims):
        if in_ext[a] != 1:
            idx += coords[d] * in_str[a]
    d_src, d_dst = dev(src), sentinel(n * es)
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    any_launch(route, "broadcast_in_dim", n, [vp(d_dst), vp(d_src), ctypes.c_int(dtype), out_any, in_any, av,
                                              ctypes.c_longlong(n)])
    assert np.array_equal(take(d_dst, n * es).reshape(n, es), src.reshape(total, es)[idx])
    del k1, k2, k3


@pytest.mark.parametrize("route", ["launcher", "module", "module-refgeom"])
def test_complex64_bases_off_8_bytes(cuda, route):
    """complex64 buffers 4 bytes off an 8-byte boundary (legal: the ABI's complex64 is
    4-byte aligned) through the by-value entries: permutations, a reversal and fills."""
    import torch
    rng = np.random.default_rng(77)
    es = ESIZE[abi.C32]
    mod = Module(OUR_CUBIN) if route != "launcher" else None
    for shape, perm in [((64, 48), (1, 0)), ((6, 5, 7), (2, 0, 1)), ((300,), (0,))]:
        src_l, out_shape = permuted_view(shape, perm)
        n = src_l.count()
        src = rng.integers(0, 256, size=n * es, dtype=np.uint8)
        dst_l = abi.layout(src_l.extents_list())
        want = oracle_copy(abi.C32, src, src_l, dst_l, n * es)
        got = gpu_copy(route, abi.C32, src, src_l, dst_l, n * es, module=mod, base=4)
        assert np.array_equal(want, got), (shape, perm)
    # fill_zero_view of every other element of a 4-off buffer
    n = 257
    view = abi.layout([n], [2], 1)
    d = sentinel(2 * n * es + 4)[4:]
    if route == "launcher":
        launch = t4.Launch()
        t4.check(t4.lib().t4a_plan_fill_zero_view(abi.C32, ctypes.byref(view), 2 * n, ctypes.byref(launch)))
        t4.check(t4.lib().t4a_launch_fill_zero_view(ctypes.byref(launch), t4.stream_handle(),
                                                    ctypes.c_void_p(d.data_ptr()), abi.C32, view, n))
    else:
        mod.launch("t4a_cuda_fill_zero_view", (2,), (256,), 0,
                   [ctypes.c_void_p(d.data_ptr()), ctypes.c_int(abi.C32), view, ctypes.c_longlong(n)])
    torch.cuda.synchronize()
    got = take(d, 2 * n * es).reshape(2 * n, es)
    assert (got[1::2] == 0).all() and (got[0::2] == SENTINEL).all()
