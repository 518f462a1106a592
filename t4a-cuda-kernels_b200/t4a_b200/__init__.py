"""Python mirror of the t4a_b200 C ABI (include/t4a_b200.h).

Host-side counterpart of the reference's Rust facade (`t4a_cuda_kernels::plan_*`,
reference src/lib.rs): planners that validate metadata and return launch geometry,
launchers that run this library's sm_100a kernels on the caller's stream, and
one-call helpers over torch tensors.  Every call goes through libt4a_b200.so; there
is no CPU or PyTorch fallback, and a missing library raises at import of `lib()`.
"""
import ctypes
import os

from . import abi
from .abi import (F32, F64, I32, I64, BOOL, C32, C64, SUM, PROD, SUM_SQUARES, MAX, MIN, UNIT, PLANE,
                  Layout, layout, numpy_layout)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libt4a_b200.so")
MODULE_DIR = os.path.join(HERE, "lib")

_LIB = None


class T4AError(RuntimeError):
    """A planner refusal or launch failure; `status` is the t4a_status code."""

    def __init__(self, status, where=""):
        self.status = status
        msg = status_string(status) if _LIB is not None else str(status)
        super().__init__(f"{where}: {msg} (status {status})" if where else f"{msg} (status {status})")


class Launch(ctypes.Structure):
    _fields_ = [("grid", ctypes.c_uint * 3), ("block", ctypes.c_uint * 3),
                ("shared_bytes", ctypes.c_uint), ("variant", ctypes.c_int)]

    def is_empty(self):
        return 0 in tuple(self.grid)

    def __repr__(self):
        return (f"Launch(grid={tuple(self.grid)}, block={tuple(self.block)}, "
                f"shared_bytes={self.shared_bytes}, variant={self.variant})")


class Split(ctypes.Structure):
    _fields_ = [("splits", ctypes.c_longlong), ("chunk_len", ctypes.c_longlong)]


class ReductionPlan(ctypes.Structure):
    _fields_ = [("is_split", ctypes.c_int), ("strategy", ctypes.c_int), ("launch", Launch),
                ("split", Split), ("pass1", Launch), ("combine_strategy", ctypes.c_int),
                ("combine_op", ctypes.c_int), ("pass2", Launch)]


def lib():
    """The loaded libt4a_b200.so.  Raises when it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libt4a_b200.so is not built ({LIB_PATH}); run t4a-cuda-kernels_b200/build.py")
        _LIB = ctypes.CDLL(LIB_PATH)
        _declare(_LIB)
    return _LIB


def _declare(l):
    P, I, U, LL, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint, ctypes.c_longlong, ctypes.c_size_t
    LP = ctypes.POINTER(Layout)
    LB = Layout  # by value
    sig = {
        "t4a_status_string": (ctypes.c_char_p, [I]),
        "t4a_abi_revision": (I, []),
        "t4a_last_cuda_error": (I, []),
        "t4a_split_policy": (I, [LL, U, ctypes.POINTER(I), ctypes.POINTER(Split)]),
        "t4a_plan_reduce": (I, [I, I, I, LP, LL, LP, LL, U, U, ctypes.POINTER(Launch)]),
        "t4a_plan_reduce_partials": (I, [I, I, LP, LL, LP, LL, U, Split, U, ctypes.POINTER(Launch)]),
        "t4a_plan_reduction": (I, [I, I, LP, LL, LP, LL, U, U, ctypes.POINTER(ReductionPlan)]),
        "t4a_reduction_partials_layout": (I, [LP, U, LL, LP]),
        "t4a_launch_reduce": (I, [ctypes.POINTER(Launch), P, P, P, I, I, I, LB, LB, I, LL]),
        "t4a_launch_reduce_partials": (I, [ctypes.POINTER(Launch), P, P, P, I, I, LB, LB, I, LL, LL, LL]),
        "t4a_reduce_workspace_bytes": (I, [I, I, LP, LL, LP, LL, U, U, ctypes.POINTER(SZ)]),
        "t4a_reduce": (I, [P, I, I, P, LP, LL, P, LP, LL, U, U, P, SZ]),
        "t4a_plan_materialize_strided": (I, [I, LP, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_contiguous_to_view": (I, [I, LP, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_strided_to_strided": (I, [I, LP, LL, LP, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_copy_exact": (I, [I, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_fill_zero": (I, [I, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_fill_zero_view": (I, [I, LP, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_tiled_transpose": (I, [I, abi.TransposeConfig, LL, LL, LL, LL, LL, LL, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_broadcast_in_dim": (I, [I, LP, LL, LP, LL, ctypes.POINTER(LL), I, ctypes.POINTER(Launch)]),
        "t4a_launch_materialize_strided": (I, [ctypes.POINTER(Launch), P, P, P, I, LB, LL]),
        "t4a_launch_contiguous_to_view": (I, [ctypes.POINTER(Launch), P, P, P, I, LB, LL]),
        "t4a_launch_strided_to_strided": (I, [ctypes.POINTER(Launch), P, P, P, I, LB, LB, LL]),
        "t4a_launch_copy_exact": (I, [ctypes.POINTER(Launch), P, P, P, I, LL]),
        "t4a_launch_tiled_transpose": (I, [ctypes.POINTER(Launch), P, P, P, I, LL, LL, LL, LL, abi.TransposeConfig]),
        "t4a_launch_broadcast_in_dim": (I, [ctypes.POINTER(Launch), P, P, P, I, LB, LB, abi.AxisValues, LL]),
        "t4a_launch_fill_zero": (I, [ctypes.POINTER(Launch), P, P, I, LL]),
        "t4a_launch_fill_zero_view": (I, [ctypes.POINTER(Launch), P, P, I, LB, LL]),
        "t4a_copy_strided": (I, [P, I, P, LP, LL, P, LP, LL]),
        "t4a_plan_gather": (I, [I, I, LP, LL, LP, LL, LP, LL, ctypes.POINTER(abi.GatherPlan),
                                ctypes.POINTER(Launch), ctypes.POINTER(LL)]),
        "t4a_plan_scatter_add": (I, [I, I, LP, LL, LP, LL, LP, LL, ctypes.POINTER(abi.ScatterPlan),
                                     ctypes.POINTER(Launch)]),
        "t4a_launch_gather": (I, [ctypes.POINTER(Launch), P, P, P, P, I, I, LP, LP, LP,
                                  ctypes.POINTER(abi.GatherPlan), LL]),
        "t4a_launch_scatter_add": (I, [ctypes.POINTER(Launch), P, P, P, P, I, I, LP, LP, LP,
                                       ctypes.POINTER(abi.ScatterPlan), LL]),
        "t4a_gather": (I, [P, I, I, P, LP, LL, P, LP, LL, P, LP, LL, ctypes.POINTER(abi.GatherPlan)]),
        "t4a_plan_initialize_permutation": (I, [LL, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_column_norms": (I, [I, LP, LL, LP, LL, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_select_pivot": (I, [I, LP, LL, LP, LL, LL, LL, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_swap_columns": (I, [I, LP, LL, LP, LL, LL, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_reflector": (I, [I, LP, LL, LP, LL, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_apply_reflector": (I, [I, LP, LL, LP, LL, LP, LL, LL, LL, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_extract_r": (I, [I, LP, LL, LP, LL, ctypes.POINTER(Launch)]),
        "t4a_plan_prefix_rank": (I, [I, LP, LL, LL, LL, ctypes.c_double, ctypes.c_double, ctypes.POINTER(Launch)]),
        "t4a_launch_initialize_permutation": (I, [ctypes.POINTER(Launch), P, P, LL, LL]),
        "t4a_launch_column_norms": (I, [ctypes.POINTER(Launch), P, P, P, I, LB, LB, LL]),
        "t4a_launch_select_pivot": (I, [ctypes.POINTER(Launch), P, P, P, P, P, I, LB, LB, LL]),
        "t4a_launch_swap_columns": (I, [ctypes.POINTER(Launch), P, P, P, P, I, LB, LB, LL]),
        "t4a_launch_reflector": (I, [ctypes.POINTER(Launch), P, P, P, I, LB, LB, LL]),
        "t4a_launch_apply_reflector": (I, [ctypes.POINTER(Launch), P, P, P, P, I, LB, LB, LB, LL, LL, LL]),
        "t4a_launch_extract_r": (I, [ctypes.POINTER(Launch), P, P, P, I, LB, LB]),
        "t4a_launch_prefix_rank": (I, [ctypes.POINTER(Launch), P, P, P, P, I, LB, ctypes.c_double, ctypes.c_double]),
        "t4a_rrqr_workspace_bytes": (I, [I, LP, ctypes.POINTER(SZ)]),
        "t4a_rrqr_primitive_faults": (I, [ctypes.POINTER(ctypes.c_ulonglong)]),
        "t4a_dist_unique_id": (I, [P]),
        "t4a_dist_comm_init": (I, [ctypes.POINTER(P), P, I, I]),
        "t4a_dist_comm_destroy": (I, [P]),
        "t4a_dist_rrqr_workspace_bytes": (I, [I, LL, I, ctypes.POINTER(SZ)]),
        "t4a_dist_rrqr": (I, [P, P, I, P, LP, LL, LL, LL, LL, P, P, P, P, P, SZ]),
        "t4a_p2p_region_bytes": (I, [LL, I, ctypes.POINTER(SZ)]),
        "t4a_p2p_create": (I, [LL, I, I, ctypes.POINTER(P), P]),
        "t4a_p2p_open": (I, [P, P]),
        "t4a_p2p_destroy": (I, [P]),
        "t4a_dist_rrqr_p2p": (I, [P, P, I, P, LP, LL, LL, LL, LL, P, P, P, P]),
        "t4a_rrqr": (I, [P, I, P, LP, LL, LL, P, P, P, P, P, SZ]),
        "t4a_rrqr_form_q": (I, [P, I, P, LP, LL, P, LP, LL, P, LP, LL, P]),
        "t4a_plan_identity_shifted": (I, [I, LP, LL, LL, ctypes.POINTER(Launch)]),
        "t4a_launch_identity_shifted": (I, [ctypes.POINTER(Launch), P, P, I, LB, LL]),
        "t4a_scatter_add": (I, [P, I, I, P, LP, LL, P, LP, LL, P, LP, LL, ctypes.POINTER(abi.ScatterPlan), P, SZ]),
        "t4a_scatter_add_range": (I, [P, I, I, P, LP, LL, LL, LL, P, LP, LL, P, LP, LL,
                                      ctypes.POINTER(abi.ScatterPlan), P, SZ]),
        "t4a_scatter_add_cyclic": (I, [P, I, I, P, LP, LL, LL, LL, LL, P, LP, LL, P, LP, LL,
                                       ctypes.POINTER(abi.ScatterPlan), P, SZ]),
        "t4a_scatter_add_workspace_bytes": (I, [I, I, LP, LP, LP, ctypes.POINTER(abi.ScatterPlan),
                                                ctypes.POINTER(SZ)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(l, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    _declare_more(l)


_EXTRA_DECLS = []


def _declare_more(l):
    for decl in _EXTRA_DECLS:
        decl(l)


def status_string(status):
    return lib().t4a_status_string(status).decode()


def check(status, where=""):
    if status != 0:
        raise T4AError(status, where)


# ---- torch interop ------------------------------------------------------------

def torch_dtype_tag(t):
    import torch
    return {torch.float32: F32, torch.float64: F64, torch.int32: I32, torch.int64: I64,
            torch.bool: BOOL, torch.uint8: BOOL, torch.complex64: C32, torch.complex128: C64}[t.dtype]


def tensor_layout(t):
    """Layout of a torch tensor relative to its data_ptr (NumPy axes reversed)."""
    return numpy_layout(list(t.shape), list(t.stride()), 0)


def span(t):
    """Elements reachable from data_ptr for a non-negative-stride tensor (the span length)."""
    if t.numel() == 0:
        return 0
    return 1 + sum((e - 1) * s for e, s in zip(t.shape, t.stride()))


def stream_handle(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


# ---- reductions (reference src/lib.rs:3033-3557) ----------------------------------

def split_policy(reduce_len, plane_width=32):
    has = ctypes.c_int()
    sp = Split()
    check(lib().t4a_split_policy(reduce_len, plane_width, ctypes.byref(has), ctypes.byref(sp)), "split_policy")
    return sp if has.value else None


def plan_reduction(dtype, op, out_layout, out_len, in_layout, in_len, axis, plane_width=32):
    plan = ReductionPlan()
    check(lib().t4a_plan_reduction(dtype, op, ctypes.byref(out_layout), out_len, ctypes.byref(in_layout),
                                   in_len, axis, plane_width, ctypes.byref(plan)), "plan_reduction")
    return plan


def plan_reduce(dtype, op, strategy, out_layout, out_len, in_layout, in_len, axis, plane_width=32):
    launch = Launch()
    check(lib().t4a_plan_reduce(dtype, op, strategy, ctypes.byref(out_layout), out_len, ctypes.byref(in_layout),
                                in_len, axis, plane_width, ctypes.byref(launch)), "plan_reduce")
    return launch


def reduction_partials_layout(in_layout, axis, splits):
    out = Layout()
    check(lib().t4a_reduction_partials_layout(ctypes.byref(in_layout), axis, splits, ctypes.byref(out)),
          "reduction_partials_layout")
    return out


def reduce_workspace_bytes(dtype, op, out_layout, out_len, in_layout, in_len, axis, plane_width=32):
    n = ctypes.c_size_t()
    check(lib().t4a_reduce_workspace_bytes(dtype, op, ctypes.byref(out_layout), out_len, ctypes.byref(in_layout),
                                           in_len, axis, plane_width, ctypes.byref(n)), "reduce_workspace_bytes")
    return n.value


def reduce_raw(stream, dtype, op, out_ptr, out_layout, out_len, in_ptr, in_layout, in_len, axis, plane_width=32,
               workspace_ptr=None, workspace_bytes=0):
    check(lib().t4a_reduce(stream, dtype, op, out_ptr, ctypes.byref(out_layout), out_len, in_ptr,
                           ctypes.byref(in_layout), in_len, axis, plane_width, workspace_ptr, workspace_bytes),
          "reduce")


def reduce(inp, axis, op=SUM, plane_width=32, out=None, workspace=None, stream=None):
    """Keepdims reduction of a CUDA tensor along NumPy axis `axis`."""
    import torch
    nd = inp.dim()
    ref_axis = nd - 1 - axis
    if out is None:
        shape = list(inp.shape)
        shape[axis] = 1
        out = torch.empty(shape, dtype=inp.dtype, device=inp.device)
    dtype = torch_dtype_tag(inp)
    il, ol = tensor_layout(inp), tensor_layout(out)
    n_in, n_out = span(inp), span(out)
    need = reduce_workspace_bytes(dtype, op, ol, n_out, il, n_in, ref_axis, plane_width)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=inp.device)
    reduce_raw(stream_handle(stream), dtype, op, ctypes.c_void_p(out.data_ptr()), ol, n_out,
               ctypes.c_void_p(inp.data_ptr()), il, n_in, ref_axis, plane_width,
               ctypes.c_void_p(workspace.data_ptr()) if need else None, need)
    return out


# ---- strided movement (reference src/lib.rs:1465-1737) -----------------------------

def _plan(fn, *args):
    launch = Launch()
    check(getattr(lib(), fn)(*args, ctypes.byref(launch)), fn)
    return launch


def plan_materialize_strided(dtype, src_layout, src_len):
    return _plan("t4a_plan_materialize_strided", dtype, ctypes.byref(src_layout), src_len)


def plan_strided_to_strided(dtype, src_layout, src_len, dst_layout, dst_len):
    return _plan("t4a_plan_strided_to_strided", dtype, ctypes.byref(src_layout), src_len, ctypes.byref(dst_layout),
                 dst_len)


def plan_contiguous_to_view(dtype, dst_layout, dst_len):
    return _plan("t4a_plan_contiguous_to_view", dtype, ctypes.byref(dst_layout), dst_len)


def plan_tiled_transpose(dtype, config, src_offset, batch_stride, dst_fast_extent, src_fast_extent, batches,
                         src_len, dst_len):
    return _plan("t4a_plan_tiled_transpose", dtype, config, src_offset, batch_stride, dst_fast_extent,
                 src_fast_extent, batches, src_len, dst_len)


def plan_broadcast_in_dim(dtype, out_layout, out_len, in_layout, in_len, dims):
    arr = (ctypes.c_longlong * max(1, len(dims)))(*dims)
    return _plan("t4a_plan_broadcast_in_dim", dtype, ctypes.byref(out_layout), out_len, ctypes.byref(in_layout),
                 in_len, arr, len(dims))


def copy_strided_raw(stream, dtype, dst_ptr, dst_layout, dst_len, src_ptr, src_layout, src_len):
    check(lib().t4a_copy_strided(stream, dtype, dst_ptr, ctypes.byref(dst_layout), dst_len, src_ptr,
                                 ctypes.byref(src_layout), src_len), "copy_strided")


def materialize(view, out=None, stream=None):
    """Compact copy of a (permuted, sliced, expanded) CUDA tensor view."""
    import torch
    if out is None:
        out = torch.empty(view.shape, dtype=view.dtype, device=view.device)
    dtype = torch_dtype_tag(view)
    base = view.storage_offset()
    src_l = numpy_layout(list(view.shape), list(view.stride()), 0)
    src_len = view.untyped_storage().nbytes() // view.element_size() - base
    copy_strided_raw(stream_handle(stream), dtype, ctypes.c_void_p(out.data_ptr()), tensor_layout(out), span(out),
                     ctypes.c_void_p(view.data_ptr()), src_l, src_len)
    return out


# ---- gather and additive scatter (reference src/lib.rs:2779-3029) ----------------

def plan_gather(dtype, index_dtype, out_layout, out_len, operand_layout, operand_len, indices_layout, indices_len,
                plan):
    """plan_gather: returns (launch, output element count)."""
    launch, count = Launch(), ctypes.c_longlong(0)
    check(lib().t4a_plan_gather(dtype, index_dtype, ctypes.byref(out_layout), out_len, ctypes.byref(operand_layout),
                                operand_len, ctypes.byref(indices_layout), indices_len, ctypes.byref(plan),
                                ctypes.byref(launch), ctypes.byref(count)), "plan_gather")
    return launch, count.value


def plan_scatter_add(dtype, index_dtype, out_layout, out_len, indices_layout, indices_len, updates_layout,
                     updates_len, plan):
    launch = Launch()
    check(lib().t4a_plan_scatter_add(dtype, index_dtype, ctypes.byref(out_layout), out_len,
                                     ctypes.byref(indices_layout), indices_len, ctypes.byref(updates_layout),
                                     updates_len, ctypes.byref(plan), ctypes.byref(launch)), "plan_scatter_add")
    return launch


def gather_raw(stream, dtype, index_dtype, out_ptr, out_layout, out_len, operand_ptr, operand_layout, operand_len,
               indices_ptr, indices_layout, indices_len, plan):
    check(lib().t4a_gather(stream, dtype, index_dtype, out_ptr, ctypes.byref(out_layout), out_len, operand_ptr,
                           ctypes.byref(operand_layout), operand_len, indices_ptr, ctypes.byref(indices_layout),
                           indices_len, ctypes.byref(plan)), "gather")


def scatter_add_workspace_bytes(dtype, index_dtype, out_layout, indices_layout, updates_layout, plan):
    n = ctypes.c_size_t(0)
    check(lib().t4a_scatter_add_workspace_bytes(dtype, index_dtype, ctypes.byref(out_layout),
                                                ctypes.byref(indices_layout), ctypes.byref(updates_layout),
                                                ctypes.byref(plan), ctypes.byref(n)), "scatter_add_workspace_bytes")
    return n.value


def scatter_add_raw(stream, dtype, index_dtype, out_ptr, out_layout, out_len, indices_ptr, indices_layout,
                    indices_len, updates_ptr, updates_layout, updates_len, plan, workspace=None, workspace_bytes=0):
    """t4a_scatter_add: the two-kernel path with a workspace pointer, else one kernel."""
    check(lib().t4a_scatter_add(stream, dtype, index_dtype, out_ptr, ctypes.byref(out_layout), out_len,
                                indices_ptr, ctypes.byref(indices_layout), indices_len, updates_ptr,
                                ctypes.byref(updates_layout), updates_len, ctypes.byref(plan), workspace,
                                workspace_bytes), "scatter_add")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def layout_any(extents, strides=None, offset=0, device="cuda"):
    """(t4a_cuda_layout_any, keep-alive tensor) with the arrays on `device`; strides
    default to compact (axis 0 fastest)."""
    import torch
    extents = list(extents)
    if strides is None:
        strides, acc = [], 1
        for e in extents:
            strides.append(acc)
            acc *= e
    arrays = torch.tensor(list(extents) + list(strides), dtype=torch.int64, device=device)
    rank = len(extents)
    lay = abi.LayoutAny(rank, 0, offset, ctypes.c_void_p(arrays.data_ptr()),
                        ctypes.c_void_p(arrays.data_ptr() + 8 * rank))
    return lay, arrays


def axis_values_any(values, device="cuda"):
    """(t4a_cuda_axis_values_any, keep-alive tensor) with the values on `device`."""
    import torch
    arr = torch.tensor(list(values) or [0], dtype=torch.int64, device=device)
    return abi.AxisValuesAny(len(values), 0, ctypes.c_void_p(arr.data_ptr())), arr


def gather_plan_any(window_dims, offset_dims, start_index_map, slice_sizes, index_vector_dim, out_rank,
                    device="cuda"):
    """(t4a_cuda_gather_plan_any, keep-alive tensor): the gather maps in device memory."""
    import torch
    vals = list(window_dims) + list(offset_dims) + list(start_index_map) + list(slice_sizes)
    arr = torch.tensor(vals or [0], dtype=torch.int64, device=device)
    base, w, k = arr.data_ptr(), len(window_dims), len(start_index_map)
    plan = abi.GatherPlanAny(len(slice_sizes), out_rank, index_vector_dim, w, k, 0, ctypes.c_void_p(base),
                             ctypes.c_void_p(base + 8 * w), ctypes.c_void_p(base + 16 * w),
                             ctypes.c_void_p(base + 16 * w + 8 * k))
    return plan, arr


def scatter_plan_any(window_dims, update_window_dims, scatter_dims, index_vector_dim, operand_rank, updates_rank,
                     device="cuda"):
    """(t4a_cuda_scatter_plan_any, keep-alive tensor): the scatter maps in device memory."""
    import torch
    vals = list(window_dims) + list(update_window_dims) + list(scatter_dims)
    arr = torch.tensor(vals or [0], dtype=torch.int64, device=device)
    base, w = arr.data_ptr(), len(window_dims)
    plan = abi.ScatterPlanAny(operand_rank, updates_rank, index_vector_dim, w, len(scatter_dims), 0,
                              ctypes.c_void_p(base), ctypes.c_void_p(base + 8 * w), ctypes.c_void_p(base + 16 * w))
    return plan, arr


def gather_scatter_any_geometry(elements):
    launch = Launch()
    check(lib().t4a_gather_scatter_any_geometry(ctypes.c_longlong(elements), ctypes.byref(launch)),
          "gather_scatter_any_geometry")
    return launch


def movement_any_geometry(length):
    launch = Launch()
    check(lib().t4a_movement_any_geometry(ctypes.c_longlong(length), ctypes.byref(launch)), "movement_any_geometry")
    return launch


def launch_movement_any(name, launch, stream, *args):
    """t4a_launch_<name>_any(&launch, stream, *args): the kernel's own argument list."""
    check(getattr(lib(), "t4a_launch_" + name + "_any")(ctypes.byref(launch), stream, *args), "launch_" + name + "_any")


def reduce_any_geometry(strategy, plane_width, output_len, splits=1):
    launch = Launch()
    check(lib().t4a_reduce_any_geometry(strategy, plane_width, output_len, splits, ctypes.byref(launch)),
          "reduce_any_geometry")
    return launch


def launch_reduce_any(launch, stream, out_ptr, in_ptr, dtype, op, strategy, out_layout, in_layout, axis, output_len):
    check(lib().t4a_launch_reduce_any(ctypes.byref(launch), stream, out_ptr, in_ptr, dtype, op, strategy, out_layout,
                                      in_layout, axis, ctypes.c_longlong(output_len)), "launch_reduce_any")


def launch_reduce_partials_any(launch, stream, part_ptr, in_ptr, dtype, op, part_layout, in_layout, axis, output_len,
                               splits, chunk):
    check(lib().t4a_launch_reduce_partials_any(ctypes.byref(launch), stream, part_ptr, in_ptr, dtype, op, part_layout,
                                               in_layout, axis, ctypes.c_longlong(output_len),
                                               ctypes.c_longlong(splits), ctypes.c_longlong(chunk)),
          "launch_reduce_partials_any")


def gather_rows(table, indices, out=None, stream=None):
    """out[i, :] = table[clamp(indices[i]), :] for a row-major CUDA table [rows, cols]
    (the XLA gather of whole rows; starts clamp as the reference's)."""
    import torch
    rows, cols = table.shape
    n = indices.numel()
    if out is None:
        out = torch.empty((n, cols), dtype=table.dtype, device=table.device)
    plan = abi.gather_plan([0], [0], [1], [cols, 1], 1, 2)
    gather_raw(stream_handle(stream), torch_dtype_tag(table), torch_dtype_tag(indices), _ptr(out),
               tensor_layout(out), span(out), _ptr(table), tensor_layout(table), span(table), _ptr(indices),
               abi.layout([n, 1]), n, plan)
    return out


def scatter_add_rows(dest, indices, updates, workspace=None, stream=None):
    """dest[clamp(indices[i]), :] += updates[i, :] in place, for a row-major CUDA
    destination [rows, cols] (the XLA additive scatter of whole rows).  `workspace`: a
    CUDA uint8 tensor of scatter_add_workspace_bytes for the two-kernel path, or None."""
    n, cols = updates.shape
    plan = abi.scatter_plan([0], [0], [1], 1, 2, 2)
    ws, nbytes = (None, 0) if workspace is None else (_ptr(workspace), workspace.numel())
    scatter_add_raw(stream_handle(stream), torch_dtype_tag(dest), torch_dtype_tag(indices), _ptr(dest),
                    tensor_layout(dest), span(dest), _ptr(indices), abi.layout([n, 1]), n, _ptr(updates),
                    tensor_layout(updates), span(updates), plan, ws, nbytes)
    return dest


def scatter_add_rows_range(shard, rows, row0, indices, updates, workspace, stream=None):
    """Rows [row0, row0 + shard_rows) of a row-major destination [rows, cols] scatter,
    held by the CUDA tensor `shard` [shard_rows, cols]: shard[clamp(indices[i]) - row0, :]
    += updates[i, :] for the updates whose clamped row falls in the slice
    (t4a_scatter_add_range).  `workspace`: scatter_rows_workspace of the whole scatter."""
    n, cols = updates.shape
    plan = abi.scatter_plan([0], [0], [1], 1, 2, 2)
    full = abi.layout([cols, rows], [1, cols])
    begin = row0 * cols
    check(lib().t4a_scatter_add_range(stream_handle(stream), torch_dtype_tag(shard), torch_dtype_tag(indices),
                                      _ptr(shard), ctypes.byref(full), rows * cols, begin,
                                      begin + shard.shape[0] * cols, _ptr(indices), ctypes.byref(abi.layout([n, 1])),
                                      n, _ptr(updates), ctypes.byref(tensor_layout(updates)), span(updates), plan,
                                      _ptr(workspace), workspace.numel()), "scatter_add_range")
    return shard


def scatter_add_rows_cyclic(shard, rows, owners, owner, indices, updates, workspace, stream=None):
    """Rows r of a row-major destination [rows, cols] with r % owners == owner, held by
    the CUDA tensor `shard` (its row k is row k * owners + owner):
    shard[(clamp(indices[i]) - owner) / owners, :] += updates[i, :] for the updates whose
    clamped row this owner holds (t4a_scatter_add_cyclic).  `workspace`:
    scatter_rows_workspace of the whole scatter."""
    n, cols = updates.shape
    plan = abi.scatter_plan([0], [0], [1], 1, 2, 2)
    full = abi.layout([cols, rows], [1, cols])
    check(lib().t4a_scatter_add_cyclic(stream_handle(stream), torch_dtype_tag(shard), torch_dtype_tag(indices),
                                       _ptr(shard), ctypes.byref(full), rows * cols, cols, owners, owner,
                                       _ptr(indices), ctypes.byref(abi.layout([n, 1])), n, _ptr(updates),
                                       ctypes.byref(tensor_layout(updates)), span(updates), plan, _ptr(workspace),
                                       workspace.numel()), "scatter_add_cyclic")
    return shard


def scatter_rows_workspace(dest, indices, updates):
    """A CUDA workspace for scatter_add_rows' two-kernel path."""
    import torch
    n, cols = updates.shape
    plan = abi.scatter_plan([0], [0], [1], 1, 2, 2)
    nbytes = scatter_add_workspace_bytes(torch_dtype_tag(dest), torch_dtype_tag(indices), tensor_layout(dest),
                                         abi.layout([n, 1]), tensor_layout(updates), plan)
    return torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dest.device)


# ---- RRQR primitives (reference src/lib.rs:2460-2774) -----------------------------

def plan_rrqr(name, *args):
    """t4a_plan_<name>(*args, &launch) for the RRQR planners; layouts by reference."""
    conv = [ctypes.byref(a) if isinstance(a, abi.Layout) else a for a in args]
    return _plan("t4a_plan_" + name, *conv)


def launch_rrqr(name, launch, stream, *args):
    """t4a_launch_<name>(&launch, stream, *args): the kernel's own argument list."""
    check(getattr(lib(), "t4a_launch_" + name)(ctypes.byref(launch), stream, *args), "launch_" + name)


def rrqr_any_geometry(tasks, flat):
    launch = Launch()
    check(lib().t4a_rrqr_any_geometry(ctypes.c_longlong(tasks), int(bool(flat)), ctypes.byref(launch)),
          "rrqr_any_geometry")
    return launch


def rrqr_form_q(work, coeff, k=None, q=None, stream=None, status=None):
    """Q formation after rrqr(work): q [m, k] (column-major, k default the coefficients
    given) = identity_shifted(0), then apply_reflector for step = k-1 .. 0 over all k
    columns with the reflectors in `work` and `coeff` (the reference bench's epilogue).
    Returns (q, status); status bit 1 means a bounded wait of the column pass ran out."""
    import torch
    m, n = work.shape
    k = coeff.numel() if k is None else k
    if q is None:
        q = torch.empty((k, m), dtype=work.dtype, device=work.device).t()
    if status is None:
        status = torch.zeros(1, dtype=torch.int64, device=work.device)
    wl = abi.layout([m, n], [work.stride(0), work.stride(1)])
    ql = abi.layout([m, k], [q.stride(0), q.stride(1)])
    cl = abi.layout([coeff.numel()])
    check(lib().t4a_rrqr_form_q(stream_handle(stream), torch_dtype_tag(work), _ptr(work), ctypes.byref(wl), span(work),
                                _ptr(coeff), ctypes.byref(cl), coeff.numel(), _ptr(q), ctypes.byref(ql), span(q),
                                _ptr(status)),
          "rrqr_form_q")
    return q, status


def rrqr_primitive_faults():
    """Faults of the column-engine primitives since the last call (bit 1: a bounded wait
    ran out and a task's outputs were left unwritten); reading clears them."""
    f = ctypes.c_ulonglong(0)
    check(lib().t4a_rrqr_primitive_faults(ctypes.byref(f)), "rrqr_primitive_faults")
    return f.value


def rrqr_workspace_bytes(dtype, work_layout):
    n = ctypes.c_size_t(0)
    check(lib().t4a_rrqr_workspace_bytes(dtype, ctypes.byref(work_layout), ctypes.byref(n)), "rrqr_workspace_bytes")
    return n.value


def rrqr(work, steps=None, stream=None, workspace=None):
    """Tall-skinny RRQR of a CUDA F32/F64 matrix in place: `work` is a torch tensor
    whose transpose is contiguous (column-major [m, n]).  Runs `steps` (default
    min(m, n)) steps of the reference loop; returns (perm, coeff, pivots, status)."""
    import torch
    m, n = work.shape
    steps = min(m, n) if steps is None else steps
    layout = abi.layout([m, n], [work.stride(0), work.stride(1)])
    dev = work.device
    perm = torch.empty(n, dtype=torch.int64, device=dev)
    coeff = torch.zeros(max(steps, 1), dtype=work.dtype, device=dev)
    pivots = torch.zeros(max(steps, 1), dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int64, device=dev)
    nbytes = rrqr_workspace_bytes(torch_dtype_tag(work), layout)
    if workspace is None:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    check(lib().t4a_rrqr(stream_handle(stream), torch_dtype_tag(work), _ptr(work), ctypes.byref(layout),
                         span(work), steps, _ptr(perm), _ptr(coeff), _ptr(pivots), _ptr(status), _ptr(workspace),
                         workspace.numel()), "rrqr")
    return perm, coeff, pivots, status
