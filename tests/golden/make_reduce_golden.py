"""Extract the reference's split-reduction golden into a committed fixture.

Reads the reference project's `tests/data/reduce-golden.tsv` (1332 cases captured
from the reference kernels on sm_80: partials FNV-1a hash and final output bytes per
case) and `tests/data/reduce-golden-nan-payload.tsv`, and writes
`tests/golden/reduce_golden.tsv`: the 666 fast-entry rows (the `_any` twins repeat
them byte for byte), with the NaN-payload exception bytes appended as a sixth
column where the reference lists one.

Run once, from the repository root, in a tree where the reference is present:
    python tests/golden/make_reduce_golden.py /path/to/reference
The test suite reads only the committed output.
"""
import os
import sys


def main(reference: str) -> None:
    src = os.path.join(reference, "tests", "data", "reduce-golden.tsv")
    payload = os.path.join(reference, "tests", "data", "reduce-golden-nan-payload.tsv")
    listed = {}
    with open(payload) as fh:
        for line in fh:
            if line.startswith("#") or not line.strip():
                continue
            key, finals = line.rstrip("\n").split("\t")
            listed[key] = finals
    out_rows = []
    header = []
    with open(src) as fh:
        for line in fh:
            if line.startswith("#"):
                header.append(line.rstrip("\n"))
                continue
            key, plan, nbytes, fnv, finals = line.rstrip("\n").split("\t")
            if not key.endswith("|fast"):
                continue
            out_rows.append("\t".join([key[: -len("|fast")], plan, nbytes, fnv, finals,
                                       listed.get(key, "")]))
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reduce_golden.tsv")
    with open(dst, "w") as fh:
        fh.write("# extracted from the reference tests/data/reduce-golden.tsv by make_reduce_golden.py\n")
        fh.write("# " + header[0].lstrip("# ") + "\n")
        fh.write("# key\tplan\tpartials_bytes\tpartials_fnv1a64\tfinals_hex\tnan_payload_variant_hex\n")
        for row in out_rows:
            fh.write(row + "\n")
    print(f"wrote {len(out_rows)} cases to {dst}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_reduce_golden.py <reference checkout>")
    main(sys.argv[1])
