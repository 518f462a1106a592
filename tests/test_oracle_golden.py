"""Pins the CPU oracle to the reference's split-reduction golden.

The fixture tests/golden/reduce_golden.tsv holds, per case, the reference kernels'
split plan, the FNV-1a hash of their pass-1 partials and the bytes of their final
outputs (reference tests/data/reduce-golden.tsv, captured on sm_80).  The inputs are
regenerated bit for bit (tests/golden/reduce_inputs.py).  The oracle must reproduce
every plan, every NaN-free partials buffer and every final output; NaN payloads are
not part of the ABI contract, so a final that differs only in the payload of a NaN
component passes.

identity_shifted is pinned to the reference's own test cases
(tests/gpu_linalg_aux.rs:1153-1185) restated as expectations.
"""
import os

import numpy as np
import pytest

import oracle
import reduce_inputs as ri
from reduce_cases import DT, OP, golden_case, partials_hash_matches, same_bits_or_nan

FIXTURE = ri.load_fixture(os.path.join(os.path.dirname(__file__), "golden", "reduce_golden.tsv"))
CASES = ri.cases()


def test_fixture_covers_every_case():
    assert len(CASES) == 666
    assert sorted(FIXTURE) == sorted("|".join([s, f"w{w}", d, o, k]) for s, w, d, o, k in CASES)


@pytest.mark.parametrize("shape", list(ri.SHAPES))
def test_oracle_reproduces_golden(shape):
    bad, partial_bad, exact = [], [], 0
    for case in [c for c in CASES if c[0] == shape]:
        s, w, d, o, k = case
        key = f"{s}|w{w}|{d}|{o}|{k}"
        plan, nbytes, fnv, finals, variant = FIXTURE[key]
        arr, in_l, out_l, axis, ftype, comps, splits = golden_case(*case)
        out = np.zeros(out_l.count() * comps, dtype=ftype)
        pe = in_l.extents_list()
        pe[axis] = splits
        part = np.zeros(int(np.prod(pe)) * comps, dtype=ftype)
        topo = oracle.reduce(DT[d], OP[o], out, out_l, arr, in_l, axis, w, part)
        assert topo.plan_string() == plan, key
        if partials_hash_matches(part.tobytes(), nbytes, fnv, ftype) is False:
            partial_bad.append(key)
        if out.tobytes().hex() == finals:
            exact += 1
        elif not same_bits_or_nan(finals, out.tobytes(), ftype, variant):
            bad.append(key)
    assert not partial_bad, partial_bad[:5]
    assert not bad, bad[:5]
    assert exact > 0


# identity_shifted: the reference's own cases (tests/gpu_linalg_aux.rs:1153-1185, its
# expectation: the element at flat position f of the layout holds one exactly when
# row(f) == start + column(f)), written into a sentinel-filled buffer so that the
# holes of the strided layout must stay untouched.
@pytest.mark.parametrize("dtype,extents,strides,offset,start", [
    ("F64", [4, 3], [1, 5], 1, 0),
    ("F64", [3, 2], [1, 3], 0, 2),
    ("F32", [3, 2], [1, 3], 0, 2),
    ("I32", [3, 2], [1, 3], 0, 0),
    ("I64", [3, 2], [1, 3], 0, 1),
    ("C32", [5, 3, 2], [1, 5, 15], 0, 1),
    ("C64", [4, 4, 3], [2, 8, 40], 1, 0),
])
def test_oracle_identity_shifted_reference_cases(dtype, extents, strides, offset, start):
    import ctypes
    from t4a_b200 import abi
    tag = getattr(abi, dtype)
    npdt = {"F32": np.float32, "F64": np.float64, "I32": np.int32, "I64": np.int64, "C32": np.complex64,
            "C64": np.complex128}[dtype]
    span = offset + sum((e - 1) * s for e, s in zip(extents, strides)) + 1
    sentinel = np.full(span, 7, dtype=npdt)
    want = sentinel.copy()
    count = int(np.prod(extents))
    for f in range(count):
        row, col, rest = f % extents[0], (f // extents[0]) % extents[1], f // (extents[0] * extents[1])
        at = offset + row * strides[0] + col * strides[1]
        for e, s in zip(extents[2:], strides[2:]):
            at += (rest % e) * s
            rest //= e
        want[at] = 1 if row == start + col else 0
    got = sentinel.copy()
    lay = abi.layout(extents, strides, offset)
    assert oracle.lib().t4a_oracle_identity_shifted(tag, oracle.ptr(got), ctypes.byref(lay), start) == 0
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))


def test_oracle_q_formation_is_orthonormal():
    """The oracle's own epilogue, which the GPU Q-formation tests compare against:
    after its RRQR loop (t4a_oracle_rrqr_f64), the identity and apply_reflector for
    step = k-1 .. 0 give an orthonormal Q with Q R = A P on the factorized columns."""
    import ctypes
    from t4a_b200 import abi
    rng = np.random.default_rng(7)
    m, n = 120, 16
    a = np.asfortranarray(rng.standard_normal((m, n)))
    work = a.copy(order="F")
    perm, coeff = np.zeros(n, np.int64), np.zeros(n)
    oracle.lib().t4a_oracle_rrqr_f64(oracle.ptr(work.ravel(order="K")), m, n, n, oracle.lptr(perm),
                                     oracle.ptr(coeff), 1e-8, 0.0, 1)
    q = np.zeros((m, n), order="F")
    wl, ql, cl = abi.layout([m, n]), abi.layout([m, n]), abi.layout([n])
    assert oracle.lib().t4a_oracle_identity_shifted(abi.F64, oracle.ptr(q.ravel(order="K")), ctypes.byref(ql), 0) == 0
    for step in range(n - 1, -1, -1):
        assert oracle.lib().t4a_oracle_apply_reflector(abi.F64, oracle.ptr(work.ravel(order="K")),
                                                       oracle.ptr(q.ravel(order="K")), oracle.ptr(coeff),
                                                       ctypes.byref(wl), ctypes.byref(ql), ctypes.byref(cl), step, 0,
                                                       n, 1) == 0
    assert np.abs(q.T @ q - np.eye(n)).max() < 1e-12
    assert np.abs(q @ np.triu(work[:n, :]) - a[:, perm]).max() < 1e-12 * np.abs(a).max() * m
