"""ctypes mirrors of the kernel-ABI structs in include/t4a_b200/abi.h.

These are the by-value metadata records of the t4a-cuda-kernels ABI
(reference cuda/include/t4a/abi.cuh:51-107, :240-245; Rust mirrors
src/lib.rs:4078-4303).  Axis 0 is the fastest-varying axis.
"""
import ctypes

MAX_RANK = 8
ABI_REVISION = 14

F32, F64, I32, I64, BOOL, C32, C64 = range(7)
DTYPE_SIZE = {F32: 4, F64: 8, I32: 4, I64: 8, BOOL: 1, C32: 8, C64: 16}
DTYPE_NAME = {F32: "F32", F64: "F64", I32: "I32", I64: "I64", BOOL: "Bool", C32: "C32", C64: "C64"}

SUM, PROD, SUM_SQUARES, MAX, MIN = range(5)
OP_NAME = {SUM: "Sum", PROD: "Prod", SUM_SQUARES: "SumSquares", MAX: "Max", MIN: "Min"}
UNIT, PLANE = 0, 1

_I64x8 = ctypes.c_longlong * MAX_RANK


class Layout(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int), ("reserved", ctypes.c_int), ("offset", ctypes.c_longlong),
                ("extents", _I64x8), ("strides", _I64x8)]

    def extents_list(self):
        return [self.extents[i] for i in range(self.rank)]

    def strides_list(self):
        return [self.strides[i] for i in range(self.rank)]

    def count(self):
        n = 1
        for e in self.extents_list():
            n *= e
        return n

    def __repr__(self):
        return f"Layout(extents={self.extents_list()}, strides={self.strides_list()}, offset={self.offset})"


class LayoutAny(ctypes.Structure):
    """t4a_cuda_layout_any: extents and strides in device memory (any rank)."""
    _fields_ = [("rank", ctypes.c_int), ("reserved", ctypes.c_int), ("offset", ctypes.c_longlong),
                ("extents", ctypes.c_void_p), ("strides", ctypes.c_void_p)]


class AxisValuesAny(ctypes.Structure):
    """t4a_cuda_axis_values_any: values in device memory (any rank)."""
    _fields_ = [("rank", ctypes.c_int), ("reserved", ctypes.c_int), ("values", ctypes.c_void_p)]


class GatherPlanAny(ctypes.Structure):
    """t4a_cuda_gather_plan_any: the gather maps in device memory (any rank)."""
    _fields_ = [("operand_rank", ctypes.c_int), ("out_rank", ctypes.c_int),
                ("index_vector_dim", ctypes.c_int), ("window_rank", ctypes.c_int),
                ("start_map_len", ctypes.c_int), ("reserved", ctypes.c_int),
                ("window_dims", ctypes.c_void_p), ("offset_dims", ctypes.c_void_p),
                ("start_index_map", ctypes.c_void_p), ("slice_sizes", ctypes.c_void_p)]


class ScatterPlanAny(ctypes.Structure):
    """t4a_cuda_scatter_plan_any: the scatter maps in device memory (any rank)."""
    _fields_ = [("operand_rank", ctypes.c_int), ("updates_rank", ctypes.c_int),
                ("index_vector_dim", ctypes.c_int), ("window_rank", ctypes.c_int),
                ("scatter_map_len", ctypes.c_int), ("reserved", ctypes.c_int),
                ("window_dims", ctypes.c_void_p), ("update_window_dims", ctypes.c_void_p),
                ("scatter_dims", ctypes.c_void_p)]


class AxisValues(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int), ("reserved", ctypes.c_int), ("values", _I64x8)]


class GatherPlan(ctypes.Structure):
    _fields_ = [("operand_rank", ctypes.c_int), ("out_rank", ctypes.c_int),
                ("index_vector_dim", ctypes.c_int), ("window_rank", ctypes.c_int),
                ("start_map_len", ctypes.c_int), ("reserved", ctypes.c_int),
                ("window_dims", _I64x8), ("offset_dims", _I64x8),
                ("start_index_map", _I64x8), ("slice_sizes", _I64x8)]


class ScatterPlan(ctypes.Structure):
    _fields_ = [("operand_rank", ctypes.c_int), ("updates_rank", ctypes.c_int),
                ("index_vector_dim", ctypes.c_int), ("window_rank", ctypes.c_int),
                ("scatter_map_len", ctypes.c_int), ("reserved", ctypes.c_int),
                ("window_dims", _I64x8), ("update_window_dims", _I64x8),
                ("scatter_dims", _I64x8)]


class TransposeConfig(ctypes.Structure):
    _fields_ = [("tile", ctypes.c_int), ("block_rows", ctypes.c_int),
                ("padding", ctypes.c_int), ("vector_width", ctypes.c_int)]


assert ctypes.sizeof(Layout) == 144 and Layout.offset.offset == 8 and Layout.strides.offset == 80
assert ctypes.sizeof(AxisValues) == 72
assert ctypes.sizeof(GatherPlan) == 280 and GatherPlan.window_dims.offset == 24
assert ctypes.sizeof(ScatterPlan) == 216 and ScatterPlan.window_dims.offset == 24
assert ctypes.sizeof(GatherPlanAny) == 56 and GatherPlanAny.slice_sizes.offset == 48
assert ctypes.sizeof(ScatterPlanAny) == 48 and ScatterPlanAny.scatter_dims.offset == 40
assert ctypes.sizeof(TransposeConfig) == 16


def layout(extents, strides=None, offset=0):
    """Layout over `extents` (axis 0 fastest); compact strides when `strides` is None."""
    extents = [int(e) for e in extents]
    if len(extents) > MAX_RANK:
        raise ValueError("rank exceeds 8")
    if strides is None:
        strides, s = [], 1
        for e in extents:
            strides.append(s)
            s *= e
    l = Layout()
    l.rank = len(extents)
    l.offset = int(offset)
    for i, (e, s) in enumerate(zip(extents, strides)):
        l.extents[i] = e
        l.strides[i] = int(s)
    return l


def numpy_layout(shape, strides_elems=None, offset=0):
    """Layout of a NumPy (row-major, last axis fastest) view: axes reversed."""
    shape = list(shape)
    if strides_elems is None:
        strides_elems, s = [], 1
        for e in reversed(shape):
            strides_elems.insert(0, s)
            s *= e
    return layout(list(reversed(shape)), list(reversed(list(strides_elems))), offset)


def axis_values(values):
    a = AxisValues()
    a.rank = len(values)
    for i, v in enumerate(values):
        a.values[i] = int(v)
    return a


def gather_plan(window_dims, offset_dims, start_index_map, slice_sizes, index_vector_dim, out_rank):
    p = GatherPlan()
    p.operand_rank = len(slice_sizes)
    p.out_rank = out_rank
    p.index_vector_dim = index_vector_dim
    p.window_rank = len(window_dims)
    p.start_map_len = len(start_index_map)
    for i, (w, o) in enumerate(zip(window_dims, offset_dims)):
        p.window_dims[i] = w
        p.offset_dims[i] = o
    for i, s in enumerate(start_index_map):
        p.start_index_map[i] = s
    for i, s in enumerate(slice_sizes):
        p.slice_sizes[i] = s
    return p


def scatter_plan(window_dims, update_window_dims, scatter_dims, index_vector_dim, operand_rank,
                 updates_rank):
    p = ScatterPlan()
    p.operand_rank = operand_rank
    p.updates_rank = updates_rank
    p.index_vector_dim = index_vector_dim
    p.window_rank = len(window_dims)
    p.scatter_map_len = len(scatter_dims)
    for i, (w, u) in enumerate(zip(window_dims, update_window_dims)):
        p.window_dims[i] = w
        p.update_window_dims[i] = u
    for i, s in enumerate(scatter_dims):
        p.scatter_dims[i] = s
    return p


def transpose_config(tile=16, block_rows=8, padding=1, vector_width=1):
    c = TransposeConfig()
    c.tile, c.block_rows, c.padding, c.vector_width = tile, block_rows, padding, vector_width
    return c
