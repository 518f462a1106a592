"""Host-side refusals of the movement and RRQR planners, restated from the reference's
planning tests (reference tests/planning.rs) as t4a_status codes.

The reference's planners return `Err(Error::...)`; this library's return the code of the
same variant (t4a_status, in the order of the Rust enum, src/lib.rs:219-270).  Launch
geometry is this library's own (one warp or one block per task), so only the refusals
and the task counts are compared, not the reference's grid shapes.  No GPU is needed."""
import ctypes

import pytest

import t4a_b200 as t4
from t4a_b200 import abi

OK = 0
COUNT_MISMATCH = 6
OFFSET_OUT_OF_SPAN = 7
UNSUPPORTED_DTYPE = 9
INVALID_TRANSPOSE_CONFIG = 12
INVALID_AXIS = 13
DUPLICATE_AXIS = 14
SHAPE_MISMATCH = 16
INVALID_STRIDE = 20
WORKSPACE = 65
NEGATIVE_COUNT = 4
LAUNCH_LIMIT = 11


def status(fn, *args):
    """The t4a_status of a planner call (0 when it plans)."""
    try:
        fn(*args)
        return OK
    except t4.T4AError as exc:
        return exc.status


def compact(*extents):
    return abi.layout(list(extents))


# ---- strided movement (tests/planning.rs:159) -----------------------------------------

def test_strided_to_strided_requires_equal_extents():
    assert status(t4.plan_strided_to_strided, abi.F32, compact(2, 2), 4, compact(4), 4) == COUNT_MISMATCH
    assert status(t4.plan_strided_to_strided, abi.F32, compact(2, 2), 4, compact(2, 2), 4) == OK
    # either side's span is checked
    assert status(t4.plan_strided_to_strided, abi.F32, compact(2, 2), 3, compact(2, 2), 4) == OFFSET_OUT_OF_SPAN
    assert status(t4.plan_strided_to_strided, abi.F32, compact(2, 2), 4, compact(2, 2), 3) == OFFSET_OUT_OF_SPAN


# ---- the transpose configuration (tests/planning.rs:195, :205, :227) --------------------

@pytest.mark.parametrize("tile,rows,pad,vec,ok", [
    (12, 8, 1, 1, False), (16, 3, 1, 1, False), (16, 8, 2, 1, False), (16, 8, 1, 8, False),
    (8, 16, 0, 4, True), (16, 8, 1, 1, True), (32, 8, 1, 2, True)])
def test_transpose_configuration_range(tile, rows, pad, vec, ok):
    cfg = abi.transpose_config(tile, rows, pad, vec)
    got = status(t4.plan_tiled_transpose, abi.F32, cfg, 0, 6, 2, 3, 1, 6, 6)
    assert (got == OK) == ok
    if not ok:
        assert got == INVALID_TRANSPOSE_CONFIG


def test_transpose_plans_batches_and_ragged_extents():
    cfg = abi.transpose_config()
    span = 512 * 1024 * 3
    launch = t4.plan_tiled_transpose(abi.F64, cfg, 0, 512 * 1024, 512, 1024, 3, span, span)
    assert not launch.is_empty()
    launch = t4.plan_tiled_transpose(abi.F32, cfg, 0, 5 * 7, 5, 7, 1, 35, 35)
    assert not launch.is_empty()


def test_transpose_rejects_bad_batches_and_limits():
    cfg = abi.transpose_config()
    # batch_stride must be the matrix product
    assert status(t4.plan_tiled_transpose, abi.F32, cfg, 0, 5, 2, 3, 1, 6, 6) == INVALID_TRANSPOSE_CONFIG
    assert status(t4.plan_tiled_transpose, abi.F32, cfg, -1, 6, 2, 3, 1, 6, 6) == NEGATIVE_COUNT
    # the source span must include every batch
    assert status(t4.plan_tiled_transpose, abi.F32, cfg, 1, 6, 2, 3, 1, 6, 6) == OFFSET_OUT_OF_SPAN
    # a zero extent plans no launch
    assert t4.plan_tiled_transpose(abi.F32, cfg, 0, 0, 0, 8, 4, 0, 0).is_empty()


# ---- broadcast_in_dim's rank map (tests/planning.rs:3105) -------------------------------

def test_broadcast_in_dim_plans_the_rank_map():
    out = compact(2, 3)
    assert status(t4.plan_broadcast_in_dim, abi.F64, out, 6, compact(2), 2, [0]) == OK
    assert status(t4.plan_broadcast_in_dim, abi.F64, out, 6, compact(2), 2, [2]) == INVALID_AXIS
    assert status(t4.plan_broadcast_in_dim, abi.F64, out, 6, compact(2, 2), 4, [0, 0]) == DUPLICATE_AXIS
    assert status(t4.plan_broadcast_in_dim, abi.F64, out, 6, compact(2), 2, [1]) == SHAPE_MISMATCH
    assert status(t4.plan_broadcast_in_dim, abi.F64, out, 6, compact(3), 3, [1]) == OK
    assert status(t4.plan_broadcast_in_dim, abi.F64, out, 6, compact(1), 1, [1]) == OK  # extent 1 broadcasts


# ---- a reversed layout (tests/planning.rs:3198) ------------------------------------------

def test_a_reversed_layout_is_a_strided_movement_plan():
    extents, strides = [3, 4], [1, 3]
    offset = sum((e - 1) * s for e, s in zip(extents, strides))
    reversed_l = abi.layout(extents, [-s for s in strides], offset)
    assert status(t4.plan_materialize_strided, abi.F64, reversed_l, 12) == OK
    assert status(t4.plan_contiguous_to_view, abi.F64, reversed_l, 12) == OK
    # the view visits the compact elements in reverse order along every axis
    visited = []
    for flat in range(12):
        i0, i1 = flat % 3, flat // 3
        visited.append(offset - i0 - 3 * i1)
    assert visited == list(range(11, -1, -1))
    # one element short of the span is refused
    assert status(t4.plan_materialize_strided, abi.F64, reversed_l, 11) == OFFSET_OUT_OF_SPAN


# ---- RRQR primitives (tests/planning.rs:2496-2745) ---------------------------------------

def rrqr(name, *args):
    return status(t4.plan_rrqr, name, *args)


def tasks_of(launch):
    """Tasks a plane geometry covers: one per warp (or per block on the column engine)."""
    per_block = 1 if launch.variant == 66 else launch.block[0] // 32
    return launch.grid[0] * per_block


def test_column_norms_maps_one_task_per_trailing_column():
    work, norms = compact(5, 4, 2), compact(4, 2)
    launch = t4.plan_rrqr("column_norms", abi.C32, work, 40, norms, 8, 1)
    assert tasks_of(launch) >= 6  # step 1 leaves three columns per batch
    # the norms carry the component type, so a shorter capacity is caught
    assert rrqr("column_norms", abi.C64, work, 40, norms, 7, 1) == OFFSET_OUT_OF_SPAN
    # the norms must drop exactly the row axis
    assert rrqr("column_norms", abi.F64, work, 40, compact(4, 2), 8, 0) == OK
    assert rrqr("column_norms", abi.F64, work, 40, compact(5, 4, 2), 40, 0) == SHAPE_MISMATCH
    assert rrqr("column_norms", abi.F64, work, 40, norms, 8, 5) == SHAPE_MISMATCH
    assert rrqr("column_norms", abi.F64, work, 40, norms, 8, -1) == SHAPE_MISMATCH
    assert rrqr("column_norms", abi.I32, work, 40, norms, 8, 0) == UNSUPPORTED_DTYPE
    # a step past the rows would leave every lane without an accumulator
    assert rrqr("column_norms", abi.F32, compact(2, 3), 6, compact(3), 3, 2) == SHAPE_MISMATCH
    assert t4.plan_rrqr("column_norms", abi.F32, compact(2, 3), 6, compact(3), 3, 3).is_empty()


def test_select_pivot_requires_matching_arrays_and_capacities():
    norms, perm = compact(6, 2), compact(6, 2)
    launch = t4.plan_rrqr("select_pivot", abi.F32, norms, 12, perm, 12, 2, 2, 1)
    assert tasks_of(launch) >= 2
    assert rrqr("select_pivot", abi.F32, norms, 12, perm, 12, 1, 2, 1) == SHAPE_MISMATCH
    assert rrqr("select_pivot", abi.F32, norms, 12, perm, 12, 2, 1, 1) == SHAPE_MISMATCH
    # the permutation is int64 whatever the norm type is
    assert rrqr("select_pivot", abi.F64, norms, 12, perm, 11, 2, 2, 1) == OFFSET_OUT_OF_SPAN
    assert rrqr("select_pivot", abi.F32, norms, 12, compact(6, 3), 18, 2, 2, 1) == SHAPE_MISMATCH
    assert rrqr("select_pivot", abi.F32, norms, 12, perm, 12, 2, 2, 7) == SHAPE_MISMATCH
    assert rrqr("select_pivot", abi.C64, norms, 12, perm, 12, 2, 2, 1) == UNSUPPORTED_DTYPE


def test_swap_columns_bounds_the_step_and_the_permutation():
    work, perm = compact(4, 3, 2), compact(3, 2)
    assert rrqr("swap_columns", abi.F64, work, 24, perm, 6, 2, 1) == OK
    big = t4.plan_rrqr("swap_columns", abi.F64, compact(20, 20, 20), 8000, compact(20, 20), 400, 20, 3)
    assert big.grid[0] * big.block[0] >= 400  # 20 rows times 20 batches
    assert rrqr("swap_columns", abi.F64, work, 24, perm, 6, 2, 3) == SHAPE_MISMATCH
    assert rrqr("swap_columns", abi.F64, work, 24, perm, 6, 2, -1) == SHAPE_MISMATCH
    assert rrqr("swap_columns", abi.F64, work, 24, compact(2, 2), 4, 2, 0) == SHAPE_MISMATCH
    # one pivot word per batch
    assert rrqr("swap_columns", abi.F64, work, 24, perm, 6, 1, 1) == SHAPE_MISMATCH


def test_reflector_bounds_the_step_and_the_coefficients():
    work, coeff = compact(5, 4, 2), compact(4, 2)
    launch = t4.plan_rrqr("reflector", abi.C64, work, 40, coeff, 8, 3)
    assert tasks_of(launch) >= 2
    assert rrqr("reflector", abi.C64, work, 40, compact(2, 2), 4, 2) == SHAPE_MISMATCH
    assert rrqr("reflector", abi.C64, work, 40, coeff, 8, 4) == SHAPE_MISMATCH
    assert rrqr("reflector", abi.C64, work, 40, coeff, 8, -1) == SHAPE_MISMATCH
    assert rrqr("reflector", abi.C64, work, 40, compact(4), 4, 0) == SHAPE_MISMATCH


def test_apply_reflector_checks_the_target_window():
    packed, coeff, target = compact(5, 4, 2), compact(4, 2), compact(5, 6, 2)
    launch = t4.plan_rrqr("apply_reflector", abi.F64, packed, 40, target, 60, coeff, 8, 1, 2, 3)
    assert tasks_of(launch) >= 6  # two batches times three columns
    assert rrqr("apply_reflector", abi.F64, packed, 40, target, 60, coeff, 8, 1, 4, 3) == SHAPE_MISMATCH
    assert rrqr("apply_reflector", abi.F64, packed, 40, target, 60, coeff, 8, 1, -1, 3) == NEGATIVE_COUNT
    assert rrqr("apply_reflector", abi.F64, packed, 40, target, 60, coeff, 8, 1, 0, -3) == NEGATIVE_COUNT
    assert rrqr("apply_reflector", abi.F64, packed, 40, compact(4, 6, 2), 48, coeff, 8, 1, 0, 1) == SHAPE_MISMATCH
    assert rrqr("apply_reflector", abi.F64, packed, 40, target, 60, coeff, 8, 4, 0, 1) == SHAPE_MISMATCH
    # the reflector lives in packed column `step`: a step outside the columns is refused
    assert rrqr("apply_reflector", abi.F64, compact(5, 1, 2), 10, compact(5, 2, 2), 20, compact(4, 2), 8, 1, 0,
                1) == SHAPE_MISMATCH


def test_extract_r_copies_the_upper_triangle_only():
    work = compact(5, 4, 2)
    assert rrqr("extract_r", abi.C32, work, 40, compact(3, 4, 2), 24) == OK
    assert rrqr("extract_r", abi.C32, work, 40, compact(6, 4, 2), 48) == SHAPE_MISMATCH
    assert rrqr("extract_r", abi.C32, work, 40, compact(3, 5, 2), 30) == SHAPE_MISMATCH


def test_prefix_rank_bounds_the_diagonal_domain():
    r = compact(3, 4, 2)
    launch = t4.plan_rrqr("prefix_rank", abi.F64, r, 24, 2, 2, 1e-12, 0.0)
    assert tasks_of(launch) >= 2
    assert rrqr("prefix_rank", abi.F64, r, 24, 1, 2, 1e-12, 0.0) == SHAPE_MISMATCH
    assert rrqr("prefix_rank", abi.F64, r, 24, 2, 1, 1e-12, 0.0) == SHAPE_MISMATCH
    # more rows than columns would read past the matrix on the diagonal
    assert rrqr("prefix_rank", abi.F64, compact(5, 3, 2), 30, 2, 2, 1e-12, 0.0) == SHAPE_MISMATCH
    assert rrqr("prefix_rank", abi.F64, compact(0, 3), 0, 1, 1, 1e-12, 0.0) == SHAPE_MISMATCH


def test_engine_geometry_for_long_real_columns():
    """F32/F64 columns of at least 2048 rows from the step are planned one block per task
    on the column engine (variant 66); shorter or strided ones one warp per task."""
    long_l, short_l = compact(4096, 8), compact(1000, 8)
    n_long = t4.plan_rrqr("column_norms", abi.F64, long_l, 4096 * 8, compact(8), 8, 0)
    n_short = t4.plan_rrqr("column_norms", abi.F64, short_l, 1000 * 8, compact(8), 8, 0)
    assert n_long.variant == 66 and n_long.grid[0] == 8 and n_long.block[0] == 384
    assert n_short.variant != 66
    strided = abi.layout([4096, 8], [2, 8192])
    assert t4.plan_rrqr("column_norms", abi.F64, strided, 8192 * 8, compact(8), 8, 0).variant != 66
    assert t4.plan_rrqr("column_norms", abi.C64, long_l, 4096 * 8, compact(8), 8, 0).variant != 66
    refl = t4.plan_rrqr("reflector", abi.F32, long_l, 4096 * 8, compact(8), 8, 2)
    assert refl.variant == 66 and refl.grid[0] == 1
    app = t4.plan_rrqr("apply_reflector", abi.F64, long_l, 4096 * 8, long_l, 4096 * 8, compact(8), 8, 0, 1, 7)
    assert app.variant == 66 and app.grid[0] == 7


def test_scatter_range_refusals():
    """t4a_scatter_add_range's host checks, before any device access: a range end that
    cuts an update row, a range outside the destination, a destination that is not
    compact, and a missing workspace."""
    import ctypes
    lib = t4.lib()
    rows, cols, n = 100, 8, 10
    plan = abi.scatter_plan([0], [0], [1], 1, 2, 2)
    full = abi.layout([cols, rows], [1, cols])
    il, ul = abi.layout([n, 1]), abi.layout([cols, n], [1, cols])
    fake = ctypes.c_void_p(1 << 20)  # never dereferenced: every case is refused on the host

    def call(layout, begin, end, ws=fake, ws_bytes=1 << 20, out_len=rows * cols):
        return lib.t4a_scatter_add_range(None, abi.F64, abi.I64, fake, ctypes.byref(layout), out_len, begin, end,
                                         fake, ctypes.byref(il), n, fake, ctypes.byref(ul), n * cols, plan, ws,
                                         ws_bytes)

    assert call(full, 8, 12) == SHAPE_MISMATCH  # 12 cuts a row of 8
    assert call(full, 0, rows * cols + 8) == SHAPE_MISMATCH
    assert call(full, 16, 8) == SHAPE_MISMATCH
    assert call(abi.layout([cols, rows], [1, cols + 1]), 0, 8, out_len=rows * (cols + 1)) == INVALID_STRIDE
    assert call(full, 0, 8, None, 0) == WORKSPACE
