"""Shared helpers of the reduction tests: golden case inputs and comparisons."""
import numpy as np

import reduce_inputs as ri
from t4a_b200 import abi

DT = {"F32": abi.F32, "F64": abi.F64, "C32": abi.C32, "C64": abi.C64}
OP = {"Sum": abi.SUM, "Prod": abi.PROD, "Max": abi.MAX, "Min": abi.MIN, "SumSquares": abi.SUM_SQUARES}


def golden_case(shape, w, dtype, op, klass):
    """(input components, in layout, out layout, axis, ftype, comps, splits)."""
    extents, axis = ri.SHAPES[shape]
    width, comps = ri.DTYPES[dtype]
    splits = ri.split_count(extents[axis], w)
    arr = ri.input_array(shape, dtype, op, klass, splits)
    in_l = abi.layout(extents)
    oe = list(extents)
    oe[axis] = 1
    out_l = abi.layout(oe)
    ftype = np.float32 if width == 4 else np.float64
    return arr, in_l, out_l, axis, ftype, comps, splits


def same_bits_or_nan(golden_hex, got_bytes, ftype, variant_hex=""):
    """Bit-identical, or identical except in the payload of components NaN in both."""
    got_hex = got_bytes.hex()
    if got_hex == golden_hex or (variant_hex and got_hex == variant_hex):
        return True
    a = np.frombuffer(bytes.fromhex(golden_hex), dtype=ftype)
    b = np.frombuffer(got_bytes, dtype=ftype)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    if not (na == nb).all():
        return False
    return bool((((a == b) & (np.signbit(a) == np.signbit(b))) | na).all())


def partials_hash_matches(partials_bytes, nbytes, fnv_hex, ftype):
    """Partials hash equality, checked only when no partial is NaN (payloads are not contractual)."""
    if np.isnan(np.frombuffer(partials_bytes, dtype=ftype)).any():
        return None
    return len(partials_bytes) == nbytes and f"{ri.fnv1a64(partials_bytes):016x}" == fnv_hex
