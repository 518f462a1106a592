"""ctypes access to the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, the smoke check and the CPU
baseline leg of bench.py, never by the shipped library.  Build the library with
`make -C oracle`.
"""
import ctypes
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "t4a-cuda-kernels_b200"))
from t4a_b200 import abi  # noqa: E402  (the shared ABI struct definitions)

_LIB = None


def build():
    subprocess.check_call(["make", "-s", "-C", HERE, "all"])


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        _LIB = ctypes.CDLL(path)
        _declare(_LIB)
    return _LIB


class Topology(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("direct_strategy", ctypes.c_int),
                ("splits", ctypes.c_longlong), ("chunk_len", ctypes.c_longlong),
                ("combine_strategy", ctypes.c_int), ("combine_width", ctypes.c_int),
                ("combine_op", ctypes.c_int)]

    def plan_string(self):
        if self.kind == 0:
            return "direct=" + ("Unit" if self.direct_strategy == 0 else "Plane")
        strategy = "Unit" if self.combine_strategy == 0 else "Plane"
        return f"splits={self.splits} chunk={self.chunk_len} combine={strategy}/{self.combine_width}"


def _declare(l):
    P, L, I, LL, D = ctypes.c_void_p, ctypes.POINTER(abi.Layout), ctypes.c_int, ctypes.c_longlong, ctypes.c_double
    LP = ctypes.POINTER(ctypes.c_longlong)
    sig = {
        "t4a_oracle_reduce_topology_for": (I, [I, LL, I, ctypes.POINTER(Topology)]),
        "t4a_oracle_reduce": (I, [I, I, P, L, P, L, I, I, P, ctypes.POINTER(Topology)]),
        "t4a_oracle_reduce_threaded": (I, [I, I, P, L, P, L, I, I, I]),
        "t4a_oracle_set_complex_contraction": (I, [I]),
        "t4a_oracle_strided_to_strided": (I, [I, P, P, L, L, I]),
        "t4a_oracle_materialize_strided": (I, [I, P, P, L, I]),
        "t4a_oracle_contiguous_to_view": (I, [I, P, P, L, I]),
        "t4a_oracle_tiled_transpose": (I, [I, P, P, LL, LL, LL, LL, LL, I]),
        "t4a_oracle_broadcast_in_dim": (I, [I, P, P, L, L, ctypes.POINTER(abi.AxisValues), I]),
        "t4a_oracle_gather": (I, [I, I, P, P, P, L, L, L, ctypes.POINTER(abi.GatherPlan), I]),
        "t4a_oracle_scatter_add": (I, [I, I, P, P, P, L, L, L, ctypes.POINTER(abi.ScatterPlan), I]),
        "t4a_oracle_initialize_permutation": (I, [LP, LL, LL]),
        "t4a_oracle_column_norms": (I, [I, P, P, L, L, LL, I]),
        "t4a_oracle_select_pivot": (I, [I, P, LP, LP, LP, L, L, LL]),
        "t4a_oracle_swap_columns": (I, [I, P, LP, LP, L, L, LL]),
        "t4a_oracle_reflector": (I, [I, P, P, L, L, LL]),
        "t4a_oracle_apply_reflector": (I, [I, P, P, P, L, L, L, LL, LL, LL, I]),
        "t4a_oracle_extract_r": (I, [I, P, P, L, L]),
        "t4a_oracle_identity_shifted": (I, [I, P, L, LL]),
        "t4a_oracle_prefix_rank": (I, [I, P, LP, LP, L, D, D]),
        "t4a_oracle_rrqr_f64": (LL, [P, LL, LL, LL, LP, P, D, D, I]),
        "t4a_oracle_dist_norm_parts": (I, [P, LL, LL, LL, LL, LL, LL, P]),
        "t4a_oracle_dist_select_swap": (I, [P, LL, LL, LL, LL, LL, P, I, LP, P, LP, LP]),
        "t4a_oracle_dist_dot_parts": (I, [P, LL, LL, LL, LL, LL, P]),
        "t4a_oracle_dist_update": (I, [P, LL, LL, LL, LL, LL, P, I, P]),
        "t4a_oracle_rrqr_rows_sharded_f64": (LL, [P, LL, LL, LL, I, LP, P, LP]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(l, name)
        fn.restype = res
        fn.argtypes = args


def ptr(array):
    """Data pointer of a NumPy array."""
    return ctypes.c_void_p(array.ctypes.data)


def lptr(array):
    return array.ctypes.data_as(ctypes.POINTER(ctypes.c_longlong))


def reduce(dtype, op, out, out_layout, inp, in_layout, axis, width=32, partials=None):
    topo = Topology()
    rc = lib().t4a_oracle_reduce(dtype, op, ptr(out), ctypes.byref(out_layout), ptr(inp),
                                 ctypes.byref(in_layout), axis, width,
                                 ptr(partials) if partials is not None else None, ctypes.byref(topo))
    if rc != 0:
        raise ValueError("oracle reduce refused the case")
    return topo


def topology(op, reduce_len, width=32):
    topo = Topology()
    if lib().t4a_oracle_reduce_topology_for(op, reduce_len, width, ctypes.byref(topo)) != 0:
        raise ValueError("bad plane width")
    return topo
