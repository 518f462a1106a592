"""GPU parity of the reductions (t4a_cuda_reduce / t4a_cuda_reduce_partials).

Three sources of truth, all compared bit for bit (NaN payloads aside, which the ABI
does not make contractual):
  * the reference golden (tests/golden/reduce_golden.tsv: the reference kernels'
    partials hash and final bytes for 666 cases);
  * the CPU oracle, at the BASELINE shapes and on strided, reversed and broadcast
    layouts;
  * the reference's own kernels compiled from source for sm_100a (oracle/_ref),
    when that build is present.
Destinations are sentinel-filled with guard bytes past the end, as in the
reference tests (tests/gpu_reduce_golden.rs:39-41), to catch stray stores.
"""
import ctypes
import os

import numpy as np
import pytest

import oracle
import reduce_inputs as ri
import t4a_b200 as t4
from cuda_module import Module
from reduce_cases import DT, OP, golden_case, partials_hash_matches, same_bits_or_nan
from t4a_b200 import abi

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FIXTURE = ri.load_fixture(os.path.join(ROOT, "tests", "golden", "reduce_golden.tsv"))
SENTINEL = 0xCD
GUARD = 256
REF_CUBIN = os.path.join(ROOT, "oracle", "_ref", "reduce.cubin")
OUR_CUBIN = os.path.join(ROOT, "t4a-cuda-kernels_b200", "t4a_b200", "lib", "reduce.cubin")


def device_bytes(nbytes):
    import torch
    return torch.full((nbytes + GUARD,), SENTINEL, dtype=torch.uint8, device="cuda")


def take(buf, nbytes):
    host = buf.cpu().numpy()
    assert (host[nbytes:] == SENTINEL).all(), "a store landed past the destination"
    return host[:nbytes].tobytes()


def to_device(arr):
    import torch
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.uint8)).cuda()


def reference_geometry(w, outputs, splits, chunk, topo_strategy=None, width=None, pass1=False):
    """The reference planner's launch geometry (src/lib.rs:3243-3289, :3342-3431)."""
    if pass1:
        cubes = outputs * splits
        planes = 4 if (w == 32 and cubes <= 8192 and chunk <= 1024) else 1
        return ((cubes + planes - 1) // planes,), (w * planes,), 0
    if topo_strategy == abi.UNIT:
        return ((outputs + width - 1) // width,), (width,), 0
    return (outputs,), (width,), 0


def launch_args(*items):
    out = []
    for kind, value in items:
        out.append({"p": ctypes.c_void_p, "i": ctypes.c_int, "l": ctypes.c_longlong}[kind](value)
                   if kind in "pil" else value)
    return out


def run_case(route, case, module=None):
    """Run one golden case; returns (finals bytes, partials bytes or None, ftype, comps)."""
    import torch
    s, w, d, o, k = case
    arr, in_l, out_l, axis, ftype, comps, splits = golden_case(*case)
    esize = arr.itemsize * comps
    dtype, op = DT[d], OP[o]
    src = to_device(arr)
    outputs = out_l.count()
    out = device_bytes(outputs * esize)
    plan = t4.plan_reduction(dtype, op, out_l, outputs, in_l, in_l.count(), axis, w)
    assert plan.is_split, "golden shapes split"
    part_l = t4.reduction_partials_layout(in_l, axis, plan.split.splits)
    part = device_bytes(part_l.count() * esize)
    stream = torch.cuda.current_stream().cuda_stream
    if route.startswith("any"):
        # The general-rank twins, with every layout padded to rank 12 by trailing
        # extent-1 axes (the flat output order is unchanged).
        pad = 12 - in_l.rank

        def padded(lay):
            return t4.layout_any(lay.extents_list() + [1] * pad, lay.strides_list() + [0] * pad, lay.offset)
        (in_any, k1), (part_any, k2), (out_any, k3) = padded(in_l), padded(part_l), padded(out_l)
        g1 = t4.reduce_any_geometry(abi.PLANE, w, outputs, plan.split.splits)
        width = plan.pass2.block[0] if plan.pass2.block[0] > 32 else w
        g2 = t4.reduce_any_geometry(plan.combine_strategy, width, outputs)
        if route == "any-launcher":
            t4.launch_reduce_partials_any(g1, ctypes.c_void_p(stream), ctypes.c_void_p(part.data_ptr()),
                                          ctypes.c_void_p(src.data_ptr()), dtype, op, part_any, in_any, axis, outputs,
                                          plan.split.splits, plan.split.chunk_len)
            t4.launch_reduce_any(g2, ctypes.c_void_p(stream), ctypes.c_void_p(out.data_ptr()),
                                 ctypes.c_void_p(part.data_ptr()), dtype, plan.combine_op, plan.combine_strategy,
                                 out_any, part_any, axis, outputs)
        else:
            module.launch("t4a_cuda_reduce_partials_any", tuple(g1.grid), tuple(g1.block), 0, launch_args(
                ("p", part.data_ptr()), ("p", src.data_ptr()), ("i", dtype), ("i", op), ("s", part_any),
                ("s", in_any), ("i", axis), ("l", outputs), ("l", plan.split.splits), ("l", plan.split.chunk_len)))
            module.launch("t4a_cuda_reduce_any", tuple(g2.grid), tuple(g2.block), 0, launch_args(
                ("p", out.data_ptr()), ("p", part.data_ptr()), ("i", dtype), ("i", plan.combine_op),
                ("i", plan.combine_strategy), ("s", out_any), ("s", part_any), ("i", axis), ("l", outputs)))
        torch.cuda.synchronize()
        del k1, k2, k3
    elif route == "launcher":
        t4.check(t4.lib().t4a_launch_reduce_partials(
            ctypes.byref(plan.pass1), ctypes.c_void_p(stream), ctypes.c_void_p(part.data_ptr()),
            ctypes.c_void_p(src.data_ptr()), dtype, op, part_l, in_l, axis, outputs, plan.split.splits,
            plan.split.chunk_len))
        t4.check(t4.lib().t4a_launch_reduce(
            ctypes.byref(plan.pass2), ctypes.c_void_p(stream), ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(part.data_ptr()), dtype, plan.combine_op, plan.combine_strategy, out_l, part_l,
            axis, outputs))
    else:
        if route == "module":
            g1 = tuple(plan.pass1.grid), tuple(plan.pass1.block), plan.pass1.shared_bytes
            g2 = tuple(plan.pass2.grid), tuple(plan.pass2.block), plan.pass2.shared_bytes
        else:  # the reference planner's geometry, on either module
            g1 = reference_geometry(w, outputs, plan.split.splits, plan.split.chunk_len, pass1=True)
            width = plan.pass2.block[0] if plan.pass2.block[0] > 32 else w
            g2 = reference_geometry(w, outputs, plan.split.splits, plan.split.chunk_len,
                                    plan.combine_strategy, width)
        module.launch("t4a_cuda_reduce_partials", *g1, launch_args(
            ("p", part.data_ptr()), ("p", src.data_ptr()), ("i", dtype), ("i", op), ("s", part_l), ("s", in_l),
            ("i", axis), ("l", outputs), ("l", plan.split.splits), ("l", plan.split.chunk_len)))
        module.launch("t4a_cuda_reduce", *g2, launch_args(
            ("p", out.data_ptr()), ("p", part.data_ptr()), ("i", dtype), ("i", plan.combine_op),
            ("i", plan.combine_strategy), ("s", out_l), ("s", part_l), ("i", axis), ("l", outputs)))
    torch.cuda.synchronize()
    return take(out, outputs * esize), take(part, part_l.count() * esize), ftype


ROUTES = ["launcher", "module", "module-refgeom", "reference", "any-launcher", "any-module"]


@pytest.mark.parametrize("route", ROUTES)
@pytest.mark.parametrize("shape", list(ri.SHAPES))
def test_golden_split_reductions(cuda, route, shape):
    module = None
    if route in ("module", "module-refgeom", "any-module"):
        module = Module(OUR_CUBIN)
    elif route == "reference":
        if not os.path.exists(REF_CUBIN):
            pytest.skip("reference kernels not built (make -C oracle ref)")
        module = Module(REF_CUBIN)
    bad, partial_bad, exact = [], [], 0
    for case in [c for c in ri.cases() if c[0] == shape]:
        key = "|".join([case[0], f"w{case[1]}", case[2], case[3], case[4]])
        plan_s, nbytes, fnv, finals, variant = FIXTURE[key]
        got, partials, ftype = run_case(route, case, module)
        if partials_hash_matches(partials, nbytes, fnv, ftype) is False:
            partial_bad.append(key)
        if got.hex() == finals:
            exact += 1
        elif not same_bits_or_nan(finals, got, ftype, variant):
            bad.append((key, finals, got.hex()))
    assert not partial_bad, partial_bad[:5]
    assert not bad, bad[:5]
    assert exact > 0


# ---- against the CPU oracle ---------------------------------------------------

def check_against_oracle(arr, numpy_axis, op, dtype, ftype=None, comps=1, slice_rows=None):
    """Reduce `arr` on the GPU (full tensor) and with the oracle; compare bit for bit.
    `slice_rows`: compare only outputs of the first rows of a non-reduced leading axis
    (the oracle then folds that slice; each output depends only on its own line)."""
    import torch
    x = torch.from_numpy(arr).cuda()
    got = t4.reduce(x, numpy_axis, op).cpu().numpy()
    ref_in = arr
    if slice_rows is not None:
        lead = 1 if numpy_axis == 0 else 0
        ref_in = np.ascontiguousarray(np.take(arr, np.arange(slice_rows), axis=lead))
        got = np.take(got, np.arange(slice_rows), axis=lead)
    nd = arr.ndim
    in_l = abi.numpy_layout(ref_in.shape)
    oshape = list(ref_in.shape)
    oshape[numpy_axis] = 1
    out_l = abi.numpy_layout(oshape)
    want = np.zeros(oshape, dtype=arr.dtype)
    oracle.reduce(dtype, op, want, out_l, np.ascontiguousarray(ref_in), in_l, nd - 1 - numpy_axis)
    a = want.reshape(-1).view(ftype or arr.dtype)
    b = np.ascontiguousarray(got).reshape(-1).view(ftype or arr.dtype)
    if np.issubdtype(a.dtype, np.floating):
        ok = ((a == b) & (np.signbit(a) == np.signbit(b))) | (np.isnan(a) & np.isnan(b))
    else:
        ok = a == b
    assert ok.all(), f"{(~ok).sum()} of {ok.size} outputs differ"


OPS3 = [abi.SUM, abi.SUM_SQUARES, abi.MAX]


@pytest.mark.parametrize("op", [abi.SUM, abi.MAX])
def test_config1_f64_axis1(cuda, op):
    arr = np.random.default_rng(0).uniform(-1, 1, size=(256, 1024, 64))
    check_against_oracle(arr, 1, op, abi.F64)


@pytest.mark.parametrize("op", OPS3)
@pytest.mark.parametrize("numpy_axis", [0, 1, 2])
def test_config3_structure_f32(cuda, op, numpy_axis):
    arr = np.random.default_rng(4).standard_normal((512, 1024, 32), dtype=np.float32)
    check_against_oracle(arr, numpy_axis, op, abi.F32)


@pytest.fixture(scope="module")
def config3_full():
    return np.random.default_rng(4).standard_normal((4096, 4096, 32), dtype=np.float32)


@pytest.mark.parametrize("op", OPS3)
@pytest.mark.parametrize("numpy_axis", [0, 1, 2])
def test_config3_full_size_f32(cuda, config3_full, op, numpy_axis):
    check_against_oracle(config3_full, numpy_axis, op, abi.F32, slice_rows=48)


def test_config3_c64_axis1(cuda):
    rng = np.random.default_rng(5)
    arr = (rng.standard_normal((1024, 8192)) + 1j * rng.standard_normal((1024, 8192))).astype(np.complex128)
    check_against_oracle(arr, 1, abi.SUM, abi.C64, ftype=np.float64)


def test_config3_c64_axis1_full_size(cuda):
    """The configuration's own C64 case at full size: sum along axis 1 of [8192, 8192]
    (1 GiB), every output compared bit for bit with the oracle."""
    rng = np.random.default_rng(6)
    arr = np.empty((8192, 8192), np.complex128)
    arr.real = rng.standard_normal((8192, 8192))
    arr.imag = rng.standard_normal((8192, 8192))
    check_against_oracle(arr, 1, abi.SUM, abi.C64, ftype=np.float64)


@pytest.mark.parametrize("dtype,np_dtype", [(abi.I32, np.int32), (abi.I64, np.int64)])
@pytest.mark.parametrize("op", [abi.SUM, abi.PROD, abi.MAX, abi.MIN])
@pytest.mark.parametrize("numpy_axis", [0, 1, 2])
def test_integer_reductions_wrap(cuda, dtype, np_dtype, op, numpy_axis):
    info = np.iinfo(np_dtype)
    rng = np.random.default_rng(11)
    arr = rng.integers(info.max // 4, info.max, size=(64, 700, 12), dtype=np_dtype)
    arr[::3] = -arr[::3]
    check_against_oracle(arr, numpy_axis, op, dtype)


@pytest.mark.parametrize("op", [abi.SUM, abi.PROD, abi.SUM_SQUARES, abi.MAX, abi.MIN])
@pytest.mark.parametrize("shape,numpy_axis", [((3, 5000, 7), 1), ((9000, 3), 0), ((2, 33, 40), 2),
                                              ((1, 1), 0), ((17,), 0), ((100, 1), 1), ((6, 300, 8), 0)])
def test_ragged_shapes_f64(cuda, op, shape, numpy_axis):
    rng = np.random.default_rng(hash((shape, numpy_axis)) % 2**32)
    arr = rng.uniform(0.5, 1.5, size=shape) if op == abi.PROD else rng.standard_normal(shape)
    check_against_oracle(arr, numpy_axis, op, abi.F64)


def raw_reduce(buf, base_elems, in_l, in_len, out_l, out_len, axis, op, dtype, esize):
    """Reduce a raw layout (any signed strides) over the device buffer `buf`."""
    import torch
    out = device_bytes(out_len * esize)
    ws_n = t4.reduce_workspace_bytes(dtype, op, out_l, out_len, in_l, in_len, axis)
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device="cuda")
    t4.reduce_raw(t4.stream_handle(), dtype, op, ctypes.c_void_p(out.data_ptr()), out_l, out_len,
                  ctypes.c_void_p(buf.data_ptr() + base_elems * esize), in_l, in_len, axis, 32,
                  ctypes.c_void_p(ws.data_ptr()), ws_n)
    torch.cuda.synchronize()
    return take(out, out_len * esize)


@pytest.mark.parametrize("dtype,np_dtype", [(abi.F32, np.float32), (abi.F64, np.float64), (abi.I32, np.int32),
                                            (abi.I64, np.int64)])
@pytest.mark.parametrize("op", [abi.SUM, abi.PROD, abi.SUM_SQUARES, abi.MAX, abi.MIN])
def test_rows_of_32(cuda, dtype, np_dtype, op):
    """A contiguous reduced axis of exactly 32 (the warp-private rows kernel): 315
    outputs (not a multiple of 32), NaN and infinities in float rows."""
    if op == abi.SUM_SQUARES and dtype in (abi.I32, abi.I64):
        pytest.skip("sum_squares is a float reduction here")
    rng = np.random.default_rng(int(dtype) * 10 + int(op))
    shape = (7, 45, 32)
    if np.issubdtype(np_dtype, np.integer):
        arr = rng.integers(-1000, 1000, size=shape).astype(np_dtype)
    else:
        arr = (rng.uniform(0.9, 1.1, size=shape) if op == abi.PROD else rng.standard_normal(shape)).astype(np_dtype)
        arr[1, 2, 5] = np.nan
        arr[3, 4, 0] = np.inf
        arr[5, 6, 31] = -np.inf
    check_against_oracle(arr, 2, op, dtype)


@pytest.mark.parametrize("base_elems", [0, 1])
def test_rows_of_32_strided_destination_and_unaligned_base(cuda, base_elems):
    """Rows of 32 into a transposed destination (outputs placed through their
    coordinates), from a base aligned to 16 bytes and from one 8 bytes past it (the
    rows path without 16-byte staging)."""
    rng = np.random.default_rng(21 + base_elems)
    data = rng.standard_normal(1 + 45 * 7 * 32)
    buf = to_device(data)
    in_l = abi.layout([32, 45, 7])
    out_l = abi.layout([1, 45, 7], [0, 7, 1])  # transposed: output (i, j) at 7 i + j
    sub = data[base_elems:base_elems + 45 * 7 * 32]
    got = raw_reduce(buf, base_elems, in_l, len(sub), out_l, 45 * 7, 0, abi.SUM, abi.F64, 8)
    want = np.zeros(45 * 7)
    oracle.reduce(abi.F64, abi.SUM, want, out_l, np.ascontiguousarray(sub), in_l, 0)
    assert same_bits_or_nan(want.tobytes().hex(), got, np.float64)


@pytest.mark.parametrize("op", [abi.SUM, abi.MAX, abi.SUM_SQUARES])
@pytest.mark.parametrize("axis", [0, 1, 2])
def test_reversed_and_broadcast_layouts(cuda, op, axis):
    """Negative strides with a rebased offset, and a stride-0 broadcast axis."""
    rng = np.random.default_rng(7)
    data = rng.standard_normal(40 * 3000).astype(np.float64)
    buf = to_device(data)
    ext = [40, 75, 40]
    strides = [1, -40, 0]  # axis 1 reversed, axis 2 broadcast
    offset = 40 * 74
    in_l = abi.layout(ext, strides, offset)
    out_ext = list(ext)
    out_ext[axis] = 1
    out_l = abi.layout(out_ext)
    got = raw_reduce(buf, 0, in_l, len(data), out_l, out_l.count(), axis, op, abi.F64, 8)
    want = np.zeros(out_l.count())
    oracle.reduce(abi.F64, op, want, out_l, data, in_l, axis)
    assert same_bits_or_nan(want.tobytes().hex(), got, np.float64)
