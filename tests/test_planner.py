"""Device-free tests of the C++ planner behind the C ABI (libt4a_b200.so).

The validation rules and the numerical-topology choices are the reference
planner's; these cases restate the reference's own planning tests
(tests/planning.rs:698-1100).  Launch geometry is this library's and is checked
for consistency (non-empty, within limits), not against the reference's numbers.
"""
import ctypes
import glob
import os
import re

import pytest

import t4a_b200 as t4
from t4a_b200 import abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for path in glob.glob(os.path.join(ROOT, "include", "**", "*.h"), recursive=True):
        text = open(path).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(t4a_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    lib = t4.lib()
    names = declared_symbols()
    assert len(names) >= 12
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_revision_and_status_strings():
    assert t4.lib().t4a_abi_revision() == 14
    assert t4.status_string(0) == "ok"
    assert "plane width" in t4.status_string(22)


def reduced(extents, axis):
    out = list(extents)
    out[axis] = 1
    return abi.layout(extents), abi.layout(out)


def status_of(fn, *args):
    try:
        fn(*args)
    except t4.T4AError as e:
        return e.status
    return 0


def test_split_policy_matches_the_reference_table():
    sp = t4.split_policy
    assert sp(255) is None and sp(256) is None
    assert (sp(512).splits, sp(512).chunk_len) == (2, 256)
    assert (sp(513).splits, sp(513).chunk_len) == (2, 256)
    assert (sp(1000).splits, sp(1000).chunk_len) == (3, 333)
    assert (sp(8448).splits, sp(8448).chunk_len) == (33, 256)
    capped = sp(10_000_000)
    assert (capped.splits, capped.chunk_len) == (4096, 10_000_000 // 4096)
    assert (sp(256, 16).splits, sp(256, 16).chunk_len) == (2, 128)
    assert (sp(255, 8).splits, sp(255, 8).chunk_len) == (3, 85)
    assert sp(0) is None
    assert status_of(sp, 512, 0) == 22


def test_strategy_boundary_is_the_plane_width():
    inp, out = reduced([32, 3], 0)
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.UNIT, out, 3, inp, 96, 0, 32) == 0
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.PLANE, out, 3, inp, 96, 0, 32) == 0
    inp, out = reduced([31, 3], 0)
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.PLANE, out, 3, inp, 93, 0, 32) == 21
    inp, out = reduced([33, 3], 0)
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.UNIT, out, 3, inp, 99, 0, 32) == 21
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.PLANE, out, 3, inp, 99, 0, 32) == 0
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.PLANE, out, 3, inp, 99, 0, 24) == 22


def test_reduction_shapes_are_validated():
    inp, _ = reduced([4, 64], 1)
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.PLANE, abi.layout([4]), 4, inp, 256, 1, 32) == 2
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.PLANE, abi.layout([5, 1]), 5, inp, 256, 1, 32) == 16
    zin, zout = reduced([4, 0], 1)
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.UNIT, zout, 4, zin, 0, 1, 32) == 4
    ein, eout = reduced([0, 64], 1)
    assert t4.plan_reduce(abi.F32, abi.SUM, abi.PLANE, eout, 0, ein, 0, 1, 32).is_empty()
    # Spans: an input allocation one element short is refused.
    inp, out = reduced([64, 4], 0)
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.PLANE, out, 4, inp, 255, 0, 32) == 7
    # A broadcast destination axis is refused.
    bad_out = abi.layout([1, 4], [1, 0])
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.PLANE, bad_out, 4, inp, 256, 0, 32) == 8
    assert status_of(t4.plan_reduce, abi.F32, abi.SUM, abi.PLANE, out, 4, inp, 256, 2, 32) == 13


def test_dtype_gates_follow_the_operation():
    inp, out = reduced([64, 2], 0)
    assert status_of(t4.plan_reduce, abi.C64, abi.MAX, abi.PLANE, out, 2, inp, 128, 0, 32) == 9
    assert status_of(t4.plan_reduce, abi.I32, abi.SUM_SQUARES, abi.PLANE, out, 2, inp, 128, 0, 32) == 9
    assert status_of(t4.plan_reduce, abi.C64, abi.PROD, abi.PLANE, out, 2, inp, 128, 0, 32) == 0
    assert status_of(t4.plan_reduce, abi.BOOL, abi.SUM, abi.PLANE, out, 2, inp, 128, 0, 32) == 9


def test_auto_policy():
    inp, out = reduced([64, 4], 0)
    plan = t4.plan_reduction(abi.F64, abi.SUM, out, 4, inp, 256, 0)
    assert plan.is_split == 0 and plan.strategy == abi.PLANE and not plan.launch.is_empty()
    inp, out = reduced([512, 4], 0)
    plan = t4.plan_reduction(abi.F64, abi.SUM, out, 4, inp, 2048, 0)
    assert plan.is_split == 1 and (plan.split.splits, plan.split.chunk_len) == (2, 256)
    assert plan.combine_strategy == abi.UNIT and plan.combine_op == abi.SUM
    inp, out = reduced([8448, 2], 0)
    plan = t4.plan_reduction(abi.F32, abi.SUM_SQUARES, out, 2, inp, 16896, 0)
    assert plan.split.splits == 33 and plan.combine_strategy == abi.PLANE and plan.combine_op == abi.SUM
    # Many partials widen the combine block unless the op is PROD.
    inp, out = reduced([65536 * 8, 1], 0)
    plan = t4.plan_reduction(abi.F32, abi.SUM, out, 1, inp, 65536 * 8, 0)
    assert plan.split.splits == 2048 and plan.pass2.block[0] == 256
    plan = t4.plan_reduction(abi.F32, abi.PROD, out, 1, inp, 65536 * 8, 0)
    assert plan.pass2.block[0] == 32


def test_partials_plans_enforce_the_floor_split():
    inp, _ = reduced([512, 4], 0)
    partials = abi.layout([2, 4])

    def plan(splits, chunk):
        launch = t4.Launch()
        return t4.lib().t4a_plan_reduce_partials(abi.F32, abi.SUM, ctypes.byref(partials), 8, ctypes.byref(inp),
                                                 2048, 0, t4.Split(splits, chunk), 32, ctypes.byref(launch))

    assert plan(2, 256) == 0
    assert plan(64, 1) == 23
    assert plan(2, 255) == 23
    assert plan(1, 512) == 23


def test_partials_layout_is_compact_with_the_split_axis():
    inp = abi.layout([4096, 4096, 32][::-1])
    p = t4.reduction_partials_layout(inp, 2, 16)
    assert p.extents_list() == [32, 4096, 16] and p.strides_list() == [1, 32, 131072]


@pytest.mark.parametrize("numpy_axis", [0, 1, 2])
def test_config3_reductions_plan_the_coalesced_paths(numpy_axis):
    shape = [4096, 4096, 32]
    inp = abi.numpy_layout(shape)
    out_shape = list(shape)
    out_shape[numpy_axis] = 1
    out = abi.numpy_layout(out_shape)
    axis = 2 - numpy_axis
    plan = t4.plan_reduction(abi.F32, abi.SUM, out, out.count(), inp, inp.count(), axis)
    if numpy_axis == 2:
        assert plan.is_split == 0 and plan.strategy == abi.UNIT and plan.launch.variant == 18
    else:
        assert plan.is_split == 1 and plan.split.splits == 16 and plan.pass1.variant == 17


# ---- gather / scatter_add planners (src/lib.rs:2867-3029) ------------------------

def test_gather_planner_errors():
    op_l, idx_l = abi.layout([4, 3]), abi.layout([2, 1])
    plan = abi.gather_plan([1], [1], [0], [1, 3], 1, 2)
    ok = t4.plan_gather(abi.F64, abi.I64, abi.layout([2, 3]), 6, op_l, 12, idx_l, 2, plan)
    assert ok[1] == 6
    cases = [
        (abi.F64, abi.BOOL, abi.layout([2, 3]), plan, idx_l, 9),                        # index dtype
        (abi.F64, abi.I64, abi.layout([2, 4]), plan, idx_l, 16),                        # derived extents
        (abi.F64, abi.I64, abi.layout([2, 3]), abi.gather_plan([1], [1], [0], [1, 4], 1, 2), idx_l, 16),  # slice > extent
        (abi.F64, abi.I64, abi.layout([2, 3]), abi.gather_plan([1], [1], [0], [2, 3], 1, 2), idx_l, 16),  # collapsed != 1
        (abi.F64, abi.I64, abi.layout([2, 3]), abi.gather_plan([1], [1], [0, 1], [1, 3], 1, 2), idx_l, 24),  # vector size
        (abi.F64, abi.I64, abi.layout([2, 3]), abi.gather_plan([1], [1], [0], [1, 3], 1, 2), abi.layout([2, 1], [2, 1]), 15),
        (abi.F64, abi.I64, abi.layout([2, 3]), abi.gather_plan([1], [1], [5], [1, 3], 1, 2), idx_l, 13),  # invalid axis
        (abi.F64, abi.I64, abi.layout([2, 3]), abi.gather_plan([1, 1], [1, 0], [0], [1, 3], 1, 2), idx_l, 14),  # duplicate
    ]
    for dtype, idt, out_l, p, il, code in cases:
        with pytest.raises(t4.T4AError) as err:
            t4.plan_gather(dtype, idt, out_l, out_l.count(), op_l, 12, il, 4, p)
        assert err.value.status == code, (p, code)


def test_gather_config4_plans_a_grid_stride_launch():
    rows, cols, n = 1 << 20, 128, 1 << 22
    plan = abi.gather_plan([0], [0], [1], [cols, 1], 1, 2)
    launch, count = t4.plan_gather(abi.F32, abi.I64, abi.numpy_layout([n, cols]), n * cols,
                                   abi.numpy_layout([rows, cols]), rows * cols, abi.layout([n, 1]), n, plan)
    assert count == n * cols
    assert 0 < launch.grid[0] <= 2 ** 31 - 1 and launch.block[0] == 256


def test_scatter_planner_errors():
    out_l, idx_l, upd_l = abi.layout([6]), abi.layout([4]), abi.layout([4, 2])
    plan = abi.scatter_plan([0], [1], [0], 1, 1, 2)
    t4.plan_scatter_add(abi.F64, abi.I64, out_l, 6, idx_l, 4, upd_l, 8, plan)
    cases = [
        (abi.I32, abi.I64, upd_l, plan, idx_l, 9),                       # data dtype
        (abi.F64, abi.I64, abi.layout([5, 2]), plan, idx_l, 16),         # batch mismatch
        (abi.F64, abi.I64, upd_l, abi.scatter_plan([0], [1], [0, 0], 1, 1, 2), abi.layout([4, 2]), 14),
        (abi.F64, abi.I64, upd_l, abi.scatter_plan([0], [1], [0], 0, 1, 2), idx_l, 24),  # vector size
        (abi.F64, abi.I64, upd_l, plan, abi.layout([4], [2]), 15),      # not compact
    ]
    for dtype, idt, ul, p, il, code in cases:
        with pytest.raises(t4.T4AError) as err:
            t4.plan_scatter_add(dtype, idt, out_l, 6, il, il.count() * 2, ul, ul.count(), p)
        assert err.value.status == code, (p, code)


def test_scatter_plans_nothing_when_no_window_fits():
    plan = abi.scatter_plan([0], [1], [0], 1, 1, 2)
    launch = t4.plan_scatter_add(abi.F64, abi.I64, abi.layout([6]), 6, abi.layout([2, 1]), 2,
                                 abi.layout([2, 7]), 14, plan)
    assert launch.grid[0] == 0


def rrqr_status(dtype, layout, work_len, steps, work=0x10000, status=0x20000, ws=0x30000, ws_bytes=None,
                perm=0x40000, coeff=0x50000, piv=0x60000):
    """t4a_rrqr's status for arguments it rejects before any launch (addresses are
    never dereferenced on these paths)."""
    if ws_bytes is None:
        n = ctypes.c_size_t(0)
        rc = t4.lib().t4a_rrqr_workspace_bytes(dtype, ctypes.byref(layout), ctypes.byref(n))
        ws_bytes = n.value if rc == 0 else 1 << 20
    vp = lambda a: ctypes.c_void_p(a) if a else None  # noqa: E731
    return t4.lib().t4a_rrqr(None, dtype, vp(work), ctypes.byref(layout), work_len, steps, vp(perm), vp(coeff),
                             vp(piv), vp(status), vp(ws), ctypes.c_size_t(ws_bytes))


def test_rrqr_driver_rejects_bad_arguments_before_launching():
    good = abi.layout([600, 40])
    n = ctypes.c_size_t(0)
    assert t4.lib().t4a_rrqr_workspace_bytes(abi.F64, ctypes.byref(good), ctypes.byref(n)) == 0 and n.value > 0
    assert rrqr_status(abi.F64, good, 600 * 40, 41) == 16                    # steps > min(m, n)
    assert rrqr_status(abi.F64, good, 600 * 40, -1) == 16
    assert rrqr_status(abi.C64, good, 600 * 40, 40) == 9                     # F32/F64 only
    assert rrqr_status(abi.F64, abi.layout([600, 40, 2]), 48000, 40) == 1    # one matrix
    assert rrqr_status(abi.F64, abi.layout([600, 40], [40, 1]), 24000, 40) == 20  # row stride 1
    assert rrqr_status(abi.F64, abi.layout([600, 40], [1, 599]), 24000, 40) == 20  # columns overlap
    assert rrqr_status(abi.F64, good, 100, 40) == 7                          # span past the buffer
    assert rrqr_status(abi.F64, good, 600 * 40, 40, ws_bytes=16) == 65       # workspace too small
    assert rrqr_status(abi.F64, good, 600 * 40, 40, ws=0) == 65
    assert rrqr_status(abi.F64, good, 600 * 40, 40, work=0x10004) == 20      # not 8-byte aligned
    assert rrqr_status(abi.F32, good, 600 * 40, 40, work=0x10002) == 20      # not 4-byte aligned
    assert rrqr_status(abi.F64, good, 600 * 40, 40, status=0x20004) == 20    # status word alignment
    assert rrqr_status(abi.F64, good, 600 * 40, 40, work=0) == 66            # NULL arguments
    assert rrqr_status(abi.F64, good, 600 * 40, 40, piv=0) == 66
    assert rrqr_status(abi.F64, abi.layout([0, 40]), 0, 0) == 0              # nothing to do


def test_reduce_any_geometry_and_host_checks():
    g = t4.reduce_any_geometry(abi.UNIT, 32, 1000)
    assert (g.block[0], g.grid[0]) == (256, 4)
    g = t4.reduce_any_geometry(abi.PLANE, 16, 100, 3)
    assert (g.block[0], g.block[1], g.grid[0]) == (16, 16, 19)
    g = t4.reduce_any_geometry(abi.PLANE, 128, 70)
    assert (g.block[0], g.grid[0]) == (128, 70)
    assert t4.reduce_any_geometry(abi.PLANE, 32, 0).grid[0] == 0
    for args, code in [((abi.PLANE, 128, 70, 2), 22), ((abi.PLANE, 24, 10), 22), ((abi.UNIT, 32, -1), 4),
                       ((7, 32, 10), 25)]:
        with pytest.raises(t4.T4AError) as err:
            t4.reduce_any_geometry(*args)
        assert err.value.status == code, args
    # host-side refusals of the general-rank launchers (no device access on these paths)
    launch = t4.reduce_any_geometry(abi.UNIT, 32, 10)
    good = abi.LayoutAny(3, 0, 0, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000))
    bad_reserved = abi.LayoutAny(3, 1, 0, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000))
    null_arrays = abi.LayoutAny(3, 0, 0, None, None)
    lib = t4.lib()
    p = ctypes.c_void_p(0x3000)
    assert lib.t4a_launch_reduce_any(ctypes.byref(launch), None, p, p, abi.F32, abi.SUM, abi.UNIT, good,
                                     bad_reserved, 0, ctypes.c_longlong(10)) == 1
    assert lib.t4a_launch_reduce_any(ctypes.byref(launch), None, p, p, abi.F32, abi.SUM, abi.UNIT, null_arrays,
                                     good, 0, ctypes.c_longlong(10)) == 66
    assert lib.t4a_launch_reduce_any(ctypes.byref(launch), None, p, p, abi.F32, abi.SUM, abi.UNIT, good, good, 3,
                                     ctypes.c_longlong(10)) == 13
    assert lib.t4a_launch_reduce_partials_any(ctypes.byref(launch), None, p, p, abi.F32, abi.SUM, good, good, 0,
                                              ctypes.c_longlong(10), ctypes.c_longlong(0),
                                              ctypes.c_longlong(1)) == 23


def test_movement_any_geometry_and_host_checks():
    g = t4.movement_any_geometry(1000)
    assert (g.block[0], g.grid[0]) == (256, 4)
    assert t4.movement_any_geometry(0).grid[0] == 0
    with pytest.raises(t4.T4AError) as err:
        t4.movement_any_geometry(-1)
    assert err.value.status == 4
    lib = t4.lib()
    launch = t4.movement_any_geometry(10)
    p = ctypes.c_void_p(0x3000)
    good = abi.LayoutAny(3, 0, 0, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000))
    rank2 = abi.LayoutAny(2, 0, 0, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000))
    bad = abi.LayoutAny(3, 7, 0, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000))
    nulls = abi.LayoutAny(3, 0, 0, None, None)
    n = ctypes.c_longlong(10)
    assert lib.t4a_launch_materialize_strided_any(ctypes.byref(launch), None, p, p, abi.F32, bad, n) == 1
    assert lib.t4a_launch_contiguous_to_view_any(ctypes.byref(launch), None, p, p, abi.F32, nulls, n) == 66
    assert lib.t4a_launch_strided_to_strided_any(ctypes.byref(launch), None, p, p, abi.F32, good, rank2, n) == 2
    assert lib.t4a_launch_fill_zero_view_any(ctypes.byref(launch), None, p, 99, good, n) == 9
    dims = abi.AxisValuesAny(2, 0, ctypes.c_void_p(0x4000))
    assert lib.t4a_launch_broadcast_in_dim_any(ctypes.byref(launch), None, p, p, abi.F32, good, good, dims, n) == 2
    assert lib.t4a_launch_fill_zero_view_any(ctypes.byref(launch), None, None, abi.F32, good,
                                             ctypes.c_longlong(0)) == 0


def test_rrqr_any_geometry_and_host_checks():
    g = t4.rrqr_any_geometry(20, False)
    assert (g.block[0], g.grid[0]) == (256, 3)  # eight tasks (warps) per block
    g = t4.rrqr_any_geometry(1000, True)
    assert (g.block[0], g.grid[0]) == (256, 4)
    assert t4.rrqr_any_geometry(10 ** 12, True).grid[0] == 148 * 64
    assert t4.rrqr_any_geometry(0, True).grid[0] == 0
    with pytest.raises(t4.T4AError) as err:
        t4.rrqr_any_geometry(-1, False)
    assert err.value.status == 4
    lib = t4.lib()
    launch = t4.rrqr_any_geometry(4, False)
    lp = ctypes.byref(launch)
    p = ctypes.c_void_p(0x3000)
    mat = abi.LayoutAny(2, 0, 0, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000))
    vec = abi.LayoutAny(1, 0, 0, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000))
    bad = abi.LayoutAny(2, 7, 0, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000))
    nulls = abi.LayoutAny(2, 0, 0, None, None)
    st = ctypes.c_longlong(0)
    assert lib.t4a_launch_column_norms_any(lp, None, p, p, abi.F64, vec, vec, st) == 1  # work needs rank 2
    assert lib.t4a_launch_column_norms_any(lp, None, p, p, abi.I32, mat, vec, st) == 9
    assert lib.t4a_launch_select_pivot_any(lp, None, p, p, p, p, abi.C64, vec, vec, st) == 9
    assert lib.t4a_launch_swap_columns_any(lp, None, p, p, p, abi.F64, nulls, vec, st) == 66
    assert lib.t4a_launch_reflector_any(lp, None, p, p, abi.F64, bad, vec, st) == 1
    assert lib.t4a_launch_apply_reflector_any(lp, None, p, p, p, abi.F64, mat, vec, vec, st, st, st) == 1
    assert lib.t4a_launch_extract_r_any(lp, None, p, p, abi.F64, mat, vec) == 1
    assert lib.t4a_launch_prefix_rank_any(lp, None, p, p, p, abi.F64, vec, ctypes.c_double(0.0),
                                          ctypes.c_double(0.0)) == 1
    assert lib.t4a_launch_prefix_rank_any(None, None, p, p, p, abi.F64, mat, ctypes.c_double(0.0),
                                          ctypes.c_double(0.0)) == 66
    empty = t4.rrqr_any_geometry(0, True)
    assert lib.t4a_launch_extract_r_any(ctypes.byref(empty), None, p, p, abi.F64, mat, mat) == 0


def test_gather_scatter_any_geometry_and_host_checks():
    g = t4.gather_scatter_any_geometry(1000)
    assert (g.block[0], g.grid[0]) == (256, 4)
    assert t4.gather_scatter_any_geometry(10 ** 12).grid[0] == 148 * 64
    assert t4.gather_scatter_any_geometry(0).grid[0] == 0
    with pytest.raises(t4.T4AError) as err:
        t4.gather_scatter_any_geometry(-5)
    assert err.value.status == 4
    lib = t4.lib()
    lp = ctypes.byref(t4.gather_scatter_any_geometry(10))
    p = ctypes.c_void_p(0x3000)
    a = ctypes.c_void_p(0x1000)

    def lay(rank, reserved=0, arrays=True):
        return abi.LayoutAny(rank, reserved, 0, a if arrays else None, a if arrays else None)

    def gplan(operand_rank, out_rank, ivd, window_rank, start_len, reserved=0, arrays=True):
        x = a if arrays else None
        return abi.GatherPlanAny(operand_rank, out_rank, ivd, window_rank, start_len, reserved, x, x, x, x)

    def splan(operand_rank, updates_rank, ivd, window_rank, map_len, reserved=0):
        return abi.ScatterPlanAny(operand_rank, updates_rank, ivd, window_rank, map_len, reserved, a, a, a)

    n = ctypes.c_longlong(10)
    # Row gather: operand [cols, rows], out [cols, n], indices [n, 1] (vector axis 1).
    good = (lay(2), lay(2), lay(2), gplan(2, 2, 1, 1, 1))
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, abi.F32, abi.I64, *good, ctypes.c_longlong(0)) == 0
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, 99, abi.I64, *good, n) == 9
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, abi.F32, abi.C32, *good, n) == 9
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, abi.F32, abi.I64, *good, ctypes.c_longlong(-1)) == 4
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, abi.F32, abi.I64, lay(2, 3), lay(2), lay(2),
                                     gplan(2, 2, 1, 1, 1), n) == 1
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, abi.F32, abi.I64, lay(2), lay(2, arrays=False), lay(2),
                                     gplan(2, 2, 1, 1, 1), n) == 66
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, abi.F32, abi.I64, lay(2), lay(2), lay(2),
                                     gplan(3, 2, 1, 1, 1), n) == 2  # operand rank differs from the plan's
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, abi.F32, abi.I64, lay(2), lay(2), lay(2),
                                     gplan(2, 2, 1, 1, 1, reserved=1), n) == 1
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, abi.F32, abi.I64, lay(2), lay(2), lay(2),
                                     gplan(2, 2, 1, 1, 1, arrays=False), n) == 66
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, abi.F32, abi.I64, lay(2), lay(2), lay(2),
                                     gplan(2, 2, 3, 1, 1), n) == 13  # index_vector_dim past the indices
    assert lib.t4a_launch_gather_any(lp, None, p, p, p, abi.F32, abi.I64, lay(2), lay(2), lay(3),
                                     gplan(2, 2, 1, 1, 1), n) == 24  # index rank does not match
    assert lib.t4a_launch_gather_any(lp, None, None, p, p, abi.F32, abi.I64, *good, n) == 66
    # Row scatter: destination [cols, rows], updates [cols, n], indices [n, 1].
    sgood = (lay(2), lay(2), lay(2), splan(2, 2, 1, 1, 1))
    assert lib.t4a_launch_scatter_add_any(lp, None, p, p, p, abi.F64, abi.I32, *sgood, ctypes.c_longlong(0)) == 0
    assert lib.t4a_launch_scatter_add_any(lp, None, p, p, p, abi.I32, abi.I32, *sgood, n) == 9
    assert lib.t4a_launch_scatter_add_any(lp, None, p, p, p, abi.F64, abi.I32, lay(2), lay(2), lay(2),
                                          splan(2, 3, 1, 1, 1), n) == 2
    assert lib.t4a_launch_scatter_add_any(lp, None, p, p, p, abi.F64, abi.I32, lay(2), lay(3), lay(2),
                                          splan(2, 2, 1, 1, 1), n) == 24
    assert lib.t4a_launch_scatter_add_any(lp, None, p, p, p, abi.F64, abi.I32, lay(2), lay(2), lay(2),
                                          splan(2, 2, 1, 3, 1), n) == 1  # window wider than the ranks
    assert lib.t4a_launch_scatter_add_any(None, None, p, p, p, abi.F64, abi.I32, *sgood, n) == 66


def test_plan_identity_shifted_validation():
    """plan_identity_shifted (reference src/lib.rs:2158): numeric dtypes, a matrix
    destination without aliasing, start >= 0 and a span that covers the layout."""
    lib = t4.lib()
    launch = t4.Launch()
    lp = ctypes.byref(launch)
    lay = abi.layout([4, 3], [1, 5], 1)
    assert lib.t4a_plan_identity_shifted(abi.F64, ctypes.byref(lay), 15, 0, lp) == 0
    assert (launch.grid[0], launch.block[0]) == (1, 256)
    assert lib.t4a_plan_identity_shifted(abi.F64, ctypes.byref(lay), 14, 0, lp) == 7  # span too short
    assert lib.t4a_plan_identity_shifted(abi.F64, ctypes.byref(lay), 15, -1, lp) == 4
    assert lib.t4a_plan_identity_shifted(abi.BOOL, ctypes.byref(lay), 15, 0, lp) == 9
    assert lib.t4a_plan_identity_shifted(abi.F64, ctypes.byref(abi.layout([4])), 4, 0, lp) == 1
    assert lib.t4a_plan_identity_shifted(abi.F64, ctypes.byref(abi.layout([4, 3], [1, 0])), 4, 0, lp) == 8
    assert lib.t4a_plan_identity_shifted(abi.I32, ctypes.byref(abi.layout([4, 3])), 12, 2 ** 63 - 2, lp) == 5
    assert lib.t4a_plan_identity_shifted(abi.C64, ctypes.byref(abi.layout([0, 3], [1, 4])), 0, 0, lp) == 0
    assert launch.grid[0] == 0
    # Q formation plans every step before launching: a bad coefficient span launches nothing.
    wl, ql, cl = abi.layout([10, 4]), abi.layout([10, 4]), abi.layout([4])
    p = ctypes.c_void_p(0x1000)
    assert lib.t4a_rrqr_form_q(None, abi.F64, p, ctypes.byref(wl), 40, p, ctypes.byref(cl), 3, p,
                               ctypes.byref(ql), 40, None) == 7
    assert lib.t4a_rrqr_form_q(None, abi.I32, p, ctypes.byref(wl), 40, p, ctypes.byref(cl), 4, p,
                               ctypes.byref(ql), 40, None) == 9
