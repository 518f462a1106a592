"""Inputs of the reference's split-reduction golden, regenerated bit for bit.

Restates the reference test generator (tests/gpu_reduce_golden.rs:49-65 SplitMix64
and FNV-1a, :121-190 classes and shapes, :216-330 `input_bytes`, :460-480 case set)
with vectorised NumPy, so the committed fixture `reduce_golden.tsv` can be checked
against the same inputs the reference kernels reduced.
"""
import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)

SHAPES = {
    "n1048576": ([1_048_576], 0),
    "n1000003": ([1_000_003], 0),
    "n4194304": ([4_194_304], 0),
    "n65541": ([65_541], 0),
    "n8195": ([8_195], 0),
    "3x100003-axis1": ([3, 100_003], 1),
    "131075x3-axis0": ([131_075, 3], 0),
}
CLASSES = ["Random", "NanPayloads", "Infs", "SignedZeros", "NegZeros", "Overflow"]
DTYPES = {"F32": (4, 1), "F64": (8, 1), "C32": (4, 2), "C64": (8, 2)}


def fnv1a64(data: bytes) -> int:
    h = 0xCBF29CE484222325
    for b in data:
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def splitmix_units(seed: int, count: int) -> np.ndarray:
    """The first `count` draws of `SplitMix::unit` from state `seed`."""
    with np.errstate(over="ignore"):
        k = np.arange(1, count + 1, dtype=np.uint64)
        z = np.uint64(seed) + k * GAMMA
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
        z = z ^ (z >> np.uint64(31))
    return (z >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 52)) - 1.0


def compact_strides(extents):
    out, s = [], 1
    for e in extents:
        out.append(s)
        s *= e
    return out


def line_base(extents, axis, o):
    strides = compact_strides(extents)
    base = 0
    for d, e in enumerate(extents):
        if d == axis:
            continue
        base += (o % e) * strides[d]
        o //= e
    return base


def nan_positions(axis_len, splits, chunk):
    out = [0, 1, 33] + [32 * k for k in range(1, 32)]
    for k in [5, 37, 69, 133, 517, 1029]:
        if k < splits:
            out.append(k * chunk + 7)
    out.append(axis_len - 1)
    return sorted(set(p for p in out if p < axis_len))


def _nan_bits(width, k):
    if width == 4:
        sign = 0x80000000 if k % 2 == 1 else 0
        return sign | 0x7FC00000 | (0x100 + k * 0x11)
    sign = 1 << 63 if k % 2 == 1 else 0
    return sign | 0x7FF8000000000000 | (0x1000 + k * 0x111)


def input_array(shape_name, dtype, op, klass, splits):
    """Input components as a flat float array (f32 or f64, `comps` per element),
    plus its raw bytes, exactly as `input_bytes` writes them."""
    extents, axis = SHAPES[shape_name]
    width, comps = DTYPES[dtype]
    count = int(np.prod(extents))
    seed = fnv1a64(f"{shape_name}|{dtype}|{op}|{klass}".encode())
    prod = op == "Prod"
    n = count * comps
    if klass == "Overflow":
        draws = splitmix_units(seed, 2 * n).reshape(n, 2)
        u, mag = draws[:, 0], 2.0 + 0.5 * draws[:, 1]
        vals = np.where(u < 0.0, -mag, mag)
    else:
        u = splitmix_units(seed, n)
        if klass == "SignedZeros":
            vals = np.where(u < 0.0, -0.0, 0.0)
        elif klass == "NegZeros":
            vals = np.full(n, -0.0)
        elif prod:
            c = np.arange(n) % comps
            vals = np.where(c == 0, 1.0 + u * (1.0 / 512.0), u * (1.0 / 512.0))
        else:
            vals = u
    ftype = np.float32 if width == 4 else np.float64
    itype = np.uint32 if width == 4 else np.uint64
    arr = vals.astype(ftype)
    bits = arr.view(itype)

    axis_len = extents[axis]
    axis_stride = compact_strides(extents)[axis]
    outputs = count // axis_len
    chunk = axis_len // max(splits, 1)
    lines = [0] + ([outputs - 1] if outputs > 1 else [])
    k = 0
    for line in lines:
        base = line_base(extents, axis, line)

        def put(position, comp, value=None, nan_k=None):
            at = (base + position * axis_stride) * comps + comp
            if nan_k is not None:
                bits[at] = itype(_nan_bits(width, nan_k))
            else:
                arr[at] = ftype(value)

        if klass == "NanPayloads":
            for position in nan_positions(axis_len, splits, chunk):
                put(position, k % comps, nan_k=k)
                k += 1
        elif klass == "Infs":
            late = 41 * chunk + 2 if 41 < splits else min(40, axis_len - 1)
            put(min(9 * chunk + 2, axis_len - 1), 0, np.inf)
            put(late, 0, -np.inf)
            if prod:
                put(min(3 * chunk + 1, axis_len - 1), 0, 0.0)
        elif klass == "Overflow":
            put(min(3 * chunk + 1, axis_len - 1), 0, 0.0)
    return arr


def cases():
    """(shape, width, dtype, op, class) of every golden case, in the reference's order."""
    pairs = []
    for dtype in ["F32", "F64"]:
        for op in ["Sum", "Prod", "Max", "Min", "SumSquares"]:
            pairs.append((dtype, op))
    for dtype in ["C32", "C64"]:
        for op in ["Sum", "Prod"]:
            pairs.append((dtype, op))
    out = []
    for shape in SHAPES:
        widths = [32, 16, 8] if shape == "n1000003" else [32]
        for w in widths:
            for dtype, op in pairs:
                for klass in CLASSES:
                    if klass == "Overflow" and op != "Prod":
                        continue
                    out.append((shape, w, dtype, op, klass))
    return out


def split_count(axis_len, width):
    splits = max(1, min(axis_len // (width * 8), 4096))
    return splits


def load_fixture(path):
    rows = {}
    with open(path) as fh:
        for line in fh:
            if line.startswith("#"):
                continue
            key, plan, nbytes, fnv, finals, variant = line.rstrip("\n").split("\t")
            rows[key] = (plan, int(nbytes), fnv, finals, variant)
    return rows
