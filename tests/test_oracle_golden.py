"""Pins the CPU oracle to the reference's split-reduction golden.

The fixture tests/golden/reduce_golden.tsv holds, per case, the reference kernels'
split plan, the FNV-1a hash of their pass-1 partials and the bytes of their final
outputs (reference tests/data/reduce-golden.tsv, captured on sm_80).  The inputs are
regenerated bit for bit (tests/golden/reduce_inputs.py).  The oracle must reproduce
every plan, every NaN-free partials buffer and every final output; NaN payloads are
not part of the ABI contract, so a final that differs only in the payload of a NaN
component passes.
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
