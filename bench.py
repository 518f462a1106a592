"""Benchmark of the t4a_b200 hot path on B200 (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--op all|movement|reduce|gather|rrqr|rrqr-loop] [--only TAGS] [--no-cpu-baseline]

One step runs every operation of the BASELINE configurations once, back to back on one
stream (the default `--op all`):
  config 1  F64 [256,1024,64] uniform(-1,1): sum and max over NumPy axis 1;
  config 2  F32 [64]^4 permuted (3,1,0,2), C64 [16]^6 permuted (5,0,4,1,3,2), F32 [64]^4
            with axis 2 reversed (strided_to_strided);
  config 3  F32 [4096,4096,32] normal: sum, sum_squares and max over each NumPy axis;
            C64 [8192,8192] sum over axis 1 (split reductions: partials + combine);
  config 4  gather of 4,194,304 rows of an F32 [1048576,128] table by uniform I64
            indices; scatter_add of F64 [4194304,128] updates into [1048576,128] with
            Zipf(1.1) indices;
  config 5  F64 RRQR of [65536,256] = U V^T + 1e-10 N, 256 steps (t4a_rrqr).
`--op rrqr-loop` (one GPU, not in the default step) times config 5 through the
reference bench's loop of RRQR primitives, launched one call at a time.
Inputs are seeded synthetic values (SplitMix64 streams; NumPy generators for config 5);
no dataset is involved.

`value` is algorithmic HBM bytes (each logical input element read once, each output
element written once; workspace excluded) over kernel time: the sum over ops of the
bytes of the whole job (all ranks) divided by the max over ranks of the summed CUDA-event
time of the ops.  Timing is steady state: the ops of a step run back to back with no L2
flush; a step touches about 12 GB, so every op starts with its inputs evicted from L2 by
the ops before it and pays for the write-back of the previous op's dirty lines.  A
second, shorter pass flushes L2 (a 256 MiB read) before every op and reports each op's
cold figure beside the steady one.

At `--gpus N` (torchrun, one rank per GPU) every op is sharded (strong scaling: the
global problem stays the same):
  reductions  slabs of a non-reduced axis, one per rank, resident on that rank;
  movement    destination parts along the axis slowest in both destination and source
              (so both sides stream long runs), each written from the strided view of
              the (replicated) source that feeds it;
  gather      index batches, table replicated;
  scatter_add destination rows, cyclic (row r on rank r mod N; owner computes): every
              rank holds the whole index list and the updates, and applies the updates
              whose row it owns (t4a_scatter_add_cyclic), so no collective is needed;
  RRQR        row blocks, with the per-step exchange of column norms and reflector dots
              fused into the step kernels (stores into every rank's memory over NVLink).
Before timing, every rank checks its shard against the single-GPU result of the same
library (computed on that rank from the full input): bit for bit for reductions,
movement and gather; for scatter_add (atomic, so its summation order is not fixed)
within the bound on reordering a sum of n terms, 2 (n - 1) 2^-53 sum|x| per element; for
RRQR the pivots over the rank-revealing prefix and the factorization residual.  A
mismatch exits non-zero.

`e2e` is the same bytes through the public C ABI with this rank's inputs copied from
pinned host memory every step and each op's results copied back, on three streams as a
caller pipelines them.  `cpu_baseline` (rank 0, N=1) and `--impl reference` time the
path's CPU implementation on this box's host cores: the reference library has no CPU
path of its own (its Rust crate only plans), so both run the C++ restatement under
oracle/ on a bounded sample of every op.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "t4a-cuda-kernels_b200"))

MIB = 1 << 20
METRIC = "achieved HBM GB/s (% of B200 peak) per op at 1/2/4/8 GPUs vs CPU baseline"


def _oracle():
    """The CPU restatement (oracle/), used only by the CPU-baseline leg and --impl reference."""
    if os.path.join(ROOT, "oracle") not in sys.path:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    return oracle


def read_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            data = json.load(fh)
        return float(data["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profile_traffic(tag):
    """Per-launch DRAM bytes of an op from a committed ncu summary, or None."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for name in sorted(os.listdir(pdir)):
        if not name.endswith((".md", ".txt")):
            continue
        with open(os.path.join(pdir, name)) as fh:
            for line in fh:
                if line.startswith(f"traffic_per_launch[{tag}]"):
                    try:
                        return int(line.split("=")[1].split()[0])
                    except (IndexError, ValueError):
                        return None
    return None


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, device_index):
        self.device_index = device_index
        self.samples = []
        self._stop = threading.Event()
        self._thread = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.samples.append([x.strip() for x in out.stdout.strip().split(",")])
            except (OSError, subprocess.SubprocessError):
                return
            self._stop.wait(0.2)

    def __enter__(self):
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        smax = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for i, n in enumerate(names):
                if len(s) > 5 + i and s[5 + i].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# Seeded inputs (counter-based SplitMix64, so any slice of a stream is generated
# directly).  torch int64 arithmetic wraps like uint64.
# ---------------------------------------------------------------------------

def _srl(z, n):
    """Logical right shift of an int64 tensor holding uint64 bits."""
    return (z >> n) & ((1 << (64 - n)) - 1)


def _i64(x):
    return x - (1 << 64) if x >= 1 << 63 else x


def _splitmix_bits(seed, start, count, device):
    import torch
    k = torch.arange(start + 1, start + count + 1, dtype=torch.int64, device=device)
    z = _i64(seed) + k * _i64(0x9E3779B97F4A7C15)
    z = (z ^ _srl(z, 30)) * _i64(0xBF58476D1CE4E5B9)
    z = (z ^ _srl(z, 27)) * _i64(0x94D049BB133111EB)
    return z ^ _srl(z, 31)


def gen_normal(seed, count, dtype, device, start=0, chunk=1 << 24):
    """Values start .. start+count-1 of the seeded normal(0,1) stream: Box-Muller over
    SplitMix64 (draws 2i, 2i+1 make value i)."""
    import math
    import torch
    out = torch.empty(count, dtype=dtype, device=device)
    for lo in range(0, count, chunk):
        n = min(chunk, count - lo)
        z = _splitmix_bits(seed, 2 * (start + lo), 2 * n, device)
        u = (_srl(z, 11).double() + 0.5) * (1.0 / (1 << 53))
        out[lo:lo + n] = (torch.sqrt(-2.0 * torch.log(u[0::2])) * torch.cos(2 * math.pi * u[1::2])).to(dtype)
    return out


def gen_uniform(seed, count, dtype, device, start=0, chunk=1 << 24):
    """Values of the seeded uniform(-1,1) stream on a 2^-52 grid: (next >> 11) 2^-52 - 1."""
    import torch
    out = torch.empty(count, dtype=dtype, device=device)
    for lo in range(0, count, chunk):
        n = min(chunk, count - lo)
        z = _splitmix_bits(seed, start + lo, n, device)
        out[lo:lo + n] = (_srl(z, 11).double() * (1.0 / (1 << 52)) - 1.0).to(dtype)
    return out


def gen_complex(seed, count, device, start=0):
    """complex128 values: real parts from stream `seed`, imaginary from `seed + 1000`."""
    import torch
    return torch.complex(gen_normal(seed, count, torch.float64, device, start),
                         gen_normal(seed + 1000, count, torch.float64, device, start))


def gen_rows_uniform(seed, n, rows, device, start=0):
    import torch
    z = _splitmix_bits(seed, start, n, device)
    u = _srl(z, 11).double() * (1.0 / (1 << 53))
    return (u * rows).to(torch.int64)


def gen_rows_zipf(seed, n, rows, s, device, start=0):
    """Zipf(s) ranks 1..rows by inverse CDF (row = rank - 1)."""
    import torch
    w = torch.arange(1, rows + 1, dtype=torch.float64, device=device) ** -s
    cdf = torch.cumsum(w, 0)
    cdf /= cdf[-1].clone()
    z = _splitmix_bits(seed, start, n, device)
    u = _srl(z, 11).double() * (1.0 / (1 << 53))
    return torch.clamp(torch.searchsorted(cdf, u, right=True), max=rows - 1).to(torch.int64)


def gen_device():
    """A GPU to generate inputs on when one is visible, else the CPU."""
    import torch
    return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")


def pinned(t):
    """A pinned host copy of a tensor (plain host copy without a GPU)."""
    import torch
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=torch.cuda.is_available())
    h.copy_(t)
    return h


def vp(t):
    return ctypes.c_void_p(t.data_ptr())


def numpy_view(t):
    """NumPy array over a host tensor (complex tensors as their float pairs)."""
    import torch
    if t.is_complex():
        return torch.view_as_real(t).numpy()
    return t.numpy()


class CheckFailed(RuntimeError):
    pass


def same_bits(got, want, what):
    import torch
    g, w = got.contiguous(), want.contiguous()
    if g.shape != w.shape:
        raise CheckFailed(f"{what}: shape {tuple(g.shape)} != {tuple(w.shape)}")
    if g.is_complex():
        g, w = torch.view_as_real(g), torch.view_as_real(w)
    ib = {1: torch.uint8, 4: torch.int32, 8: torch.int64}[g.element_size()]
    if not torch.equal(g.view(ib), w.view(ib)):
        bad = int((g.view(ib) != w.view(ib)).sum())
        raise CheckFailed(f"{what}: {bad} elements differ from the single-GPU result")


def close_rel(got, want, tol, what):
    import torch
    err = ((got - want).abs() / torch.clamp(want.abs(), min=1.0)).max().item()
    if not err <= tol:
        raise CheckFailed(f"{what}: relative error {err:.3e} > {tol:.0e}")
    return err


# ---------------------------------------------------------------------------
# Configurations.  Each holds this rank's device inputs and outputs and a list of
# ops; an op is a dict with
#   tag, config, bytes (whole job), local_bytes (this rank), launches,
#   run(stream_handle), inputs / outputs (names in self.dev / self.host),
#   optional prepare() (untimed, before the op), cpu(threads) -> sample bytes.
# setup() builds the rank's shards; check() compares them with the single-GPU result.
# ---------------------------------------------------------------------------

class Config:
    """Shared machinery: device tensors in self.dev, pinned host copies in self.host."""

    def __init__(self, rank, world, device, host_only=False):
        import t4a_b200 as t4
        from t4a_b200 import abi
        self.t4, self.abi = t4, abi
        self.rank, self.world, self.device = rank, world, device
        self.host_only = host_only
        self.dev, self.host, self.ops, self.expect = {}, {}, [], {}
        self.checks = {}

    def keep(self, name, t, host=True):
        """Registers a tensor: on the device (unless host_only) and, for e2e or the CPU
        leg, as a pinned host copy."""
        if not self.host_only:
            self.dev[name] = t if t.device.type == "cuda" else t.to(self.device)
        if host:
            self.host[name] = pinned(t)

    def shard(self, n):
        from t4a_b200 import dist as t4dist
        return t4dist.shard_range(n, self.world, self.rank)

    def group_bytes(self):
        return sum(op["bytes"] for op in self.ops)

    def after_timing(self):
        """Checks of status words after the timed steps (none by default)."""

    def close(self):
        """Releases what outlives the run (communicators); nothing by default."""


class ReduceConfigs(Config):
    """single-axis reductions through t4a_reduce
    (a direct pass, or pass 1 into the caller's partials workspace plus the combine pass).

    Sharding: axis-1 and axis-2 reductions of the F32 tensor, the C64 reduction and the
    config-1 reductions shard NumPy axis 0; axis-0 reductions of the F32 tensor shard
    axis 1.  Every rank holds its slabs (a compact copy made once) and reduces them."""

    name = "reduce"

    def setup(self):
        import torch
        t4, abi = self.t4, self.abi
        gdev = gen_device()
        n0 = 4096
        a0, a1 = self.shard(n0)
        specs = []
        # config 1
        full1 = gen_uniform(0, 256 * 1024 * 64, torch.float64, gdev).reshape(256, 1024, 64)
        c0, c1 = self.shard(256)
        self.keep("c1", full1[c0:c1].contiguous())
        specs += [("sum-f64-256x1024x64-axis1", 1, "c1", full1, (c0, c1), 0, 1, abi.SUM),
                  ("max-f64-256x1024x64-axis1", 1, "c1", full1, (c0, c1), 0, 1, abi.MAX)]
        # config 3 F32
        big = gen_normal(4, n0 * 4096 * 32, torch.float32, gdev).reshape(n0, 4096, 32)
        self.keep("x_rows", big[a0:a1].contiguous())  # axis-0 slab: reduced over axes 1 and 2
        b0, b1 = self.shard(4096)
        if self.world == 1:
            self.dev.setdefault("x_cols", self.dev.get("x_rows"))
            self.host["x_cols"] = self.host["x_rows"]
        else:
            self.keep("x_cols", big[:, b0:b1].contiguous())  # axis-1 slab: reduced over axis 0
        for ax in (0, 1, 2):
            for op, tag in ((abi.SUM, "sum"), (abi.SUM_SQUARES, "sumsq"), (abi.MAX, "max")):
                if ax == 0:
                    specs.append((f"{tag}-f32-4096x4096x32-axis0", 3, "x_cols", big, (b0, b1), 1, 0, op))
                else:
                    specs.append((f"{tag}-f32-4096x4096x32-axis{ax}", 3, "x_rows", big, (a0, a1), 0, ax, op))
        # config 3 C64
        cplx = gen_complex(5, 8192 * 8192, gdev).reshape(8192, 8192)
        z0, z1 = self.shard(8192)
        self.keep("z", cplx[z0:z1].contiguous())
        specs.append(("sum-c64-8192x8192-axis1", 3, "z", cplx, (z0, z1), 0, 1, abi.SUM))
        need_ws = 16
        for j, (tag, cfg, name, full, (s0, s1), shard_axis, ax, op) in enumerate(specs):
            local = self.dev.get(name) if not self.host_only else self.host[name]
            shape = list(local.shape)
            oshape = list(shape)
            oshape[ax] = 1
            gshape = list(full.shape)
            gshape[ax] = 1
            dt = t4.torch_dtype_tag(local)
            in_l, out_l = abi.numpy_layout(shape), abi.numpy_layout(oshape)
            n_out = 1
            for e in oshape:
                n_out *= e
            ref_axis = len(shape) - 1 - ax
            ws = t4.reduce_workspace_bytes(dt, op, out_l, n_out, in_l, local.numel(), ref_axis)
            need_ws = max(need_ws, ws)
            es = local.element_size()
            out_name = f"out{j}"
            if not self.host_only:
                self.dev[out_name] = torch.empty(oshape, dtype=local.dtype, device=self.device)
                # the single-GPU result of the whole tensor, this rank's slab of it
                want = t4.reduce(full.to(self.device) if full.device != self.device else full, ax, op)
                self.expect[out_name] = want.narrow(shard_axis, s0, s1 - s0).clone()
            self.host[out_name] = pinned(torch.empty(oshape, dtype=local.dtype))
            gl = full.numel()
            gout = 1
            for e in gshape:
                gout *= e
            self.ops.append(dict(tag=tag, config=cfg, bytes=(gl + gout) * es, local_bytes=(local.numel() + n_out) * es,
                                 launches=2 if ws else 1, inputs=[name], outputs=[out_name], dtype=dt, op=op,
                                 in_l=in_l, out_l=out_l, n_in=local.numel(), n_out=n_out, axis=ref_axis, ws=ws,
                                 src=name, dst=out_name, full_shape=list(full.shape), np_axis=ax))
        del big, cplx, full1
        if not self.host_only:
            self.workspace = torch.empty(need_ws, dtype=torch.uint8, device=self.device)
        for op in self.ops:
            op["run"] = self._runner(op)
            op["cpu"] = self._cpu(op)

    def _runner(self, op):
        def run(sh):
            self.t4.reduce_raw(sh, op["dtype"], op["op"], vp(self.dev[op["dst"]]), op["out_l"], op["n_out"],
                               vp(self.dev[op["src"]]), op["in_l"], op["n_in"], op["axis"], 32,
                               vp(self.workspace), op["ws"])
        return run

    def _cpu(self, op):
        """The oracle on a slab of the op: the whole op for config 1, 1/16 of the rows of
        a non-reduced axis for config 3 (axis-0 reductions: 256 of the 4096 columns of
        NumPy axis 1, a strided view)."""
        def cpu(threads):
            oracle = _oracle()
            abi = self.abi
            src = self.host[op["src"]]
            dst = self.host[op["dst"]]
            shape = list(src.shape)
            es = src.element_size()
            ax = op["np_axis"]
            if op["config"] == 1:
                in_l, out_l, nbytes = op["in_l"], op["out_l"], (op["n_in"] + op["n_out"]) * es
            else:
                cut = 1 if ax == 0 else 0
                keep = shape[cut] // 16
                sub = list(shape)
                sub[cut] = keep
                st, s = [], 1
                for e in reversed(shape):
                    st.insert(0, s)
                    s *= e
                in_l = abi.numpy_layout(sub, st)
                osub = list(sub)
                osub[ax] = 1
                out_l = abi.numpy_layout(osub)
                n_in = 1
                for e in sub:
                    n_in *= e
                nbytes = (n_in + n_in // sub[ax]) * es
            rc = oracle.lib().t4a_oracle_reduce_threaded(op["dtype"], op["op"], oracle.ptr(numpy_view(dst)),
                                                         ctypes.byref(out_l), oracle.ptr(numpy_view(src)),
                                                         ctypes.byref(in_l), op["axis"], 32, threads)
            assert rc == 0
            return nbytes
        return cpu

    def check(self):
        for op in self.ops:
            op["run"](self.t4.stream_handle())
            same_bits(self.dev[op["dst"]], self.expect[op["dst"]], op["tag"])


class MovementConfig(Config):
    """permutations and a reversal through the strided-copy entry.

    Sharding: the destination is split along the axis that is slowest in both it and the
    source view (t4a_b200.dist.movement_shard_axis); every rank writes its part, stored
    compactly, from the matching strided view of the source (replicated)."""

    name = "movement"

    def setup(self):
        import torch
        from t4a_b200 import dist as t4dist
        abi = self.abi
        gdev = gen_device()
        a = gen_normal(2, 64 ** 4, torch.float32, gdev)
        b = gen_complex(3, 16 ** 6, gdev).view(torch.float64)  # interleaved (re, im) pairs
        c = gen_normal(4, 64 ** 4, torch.float32, gdev)

        def perm_layout(shape, perm):
            st, s = [], 1
            for e in reversed(shape):
                st.insert(0, s)
                s *= e
            return abi.numpy_layout([shape[p] for p in perm], [st[p] for p in perm])

        specs = [
            ("perm-f32-64^4", abi.F32, a, perm_layout([64] * 4, (3, 1, 0, 2)), 4),
            ("perm-c64-16^6", abi.C64, b, perm_layout([16] * 6, (5, 0, 4, 1, 3, 2)), 16),
            ("reverse-f32-64^4", abi.F32, c, abi.numpy_layout([64] * 4, [64 ** 3, 64 ** 2, -64, 1], 63 * 64), 4),
        ]
        for i, (tag, dt, src, full_l, es) in enumerate(specs):
            n_full = full_l.count()
            src_l, dst_l, axis, start = t4dist.movement_slab(full_l, self.world, self.rank)
            n_local = dst_l.count()
            name, out = f"src{i}", f"dst{i}"
            self.keep(name, src)
            flat_len = src.numel() * src.element_size() // es
            if not self.host_only:
                self.dev[out] = torch.empty(n_local * es // src.element_size(), dtype=src.dtype, device=self.device)
                # single-GPU result of the whole permutation, this rank's slab
                whole = torch.empty_like(self.dev[name])
                self.t4.copy_strided_raw(self.t4.stream_handle(), dt, vp(whole), abi.layout(full_l.extents_list()),
                                         n_full, vp(self.dev[name]), full_l, flat_len)
                # the same part of the whole destination (t4a axis `axis` = NumPy axis rank-1-axis)
                np_shape = list(reversed(full_l.extents_list()))
                per = es // src.element_size()
                view = whole.view(np_shape + ([per] if per > 1 else []))
                part = view.narrow(full_l.rank - 1 - axis, start, dst_l.extents[axis]).contiguous()
                self.expect[out] = part.view(-1)
            self.host[out] = pinned(torch.empty(n_local * es // src.element_size(), dtype=src.dtype))
            self.ops.append(dict(tag=tag, config=2, bytes=2 * n_full * es, local_bytes=2 * n_local * es, launches=1,
                                 inputs=[name], outputs=[out], dtype=dt, src_l=src_l, dst_l=dst_l, n=n_local,
                                 flat_len=flat_len, src=name, dst=out, full_l=full_l, n_full=n_full, es=es))
        for op in self.ops:
            op["run"] = self._runner(op)
            op["cpu"] = self._cpu(op)

    def _runner(self, op):
        def run(sh):
            self.t4.copy_strided_raw(sh, op["dtype"], vp(self.dev[op["dst"]]), op["dst_l"], op["n"],
                                     vp(self.dev[op["src"]]), op["src_l"], op["flat_len"])
        return run

    def _cpu(self, op):
        def cpu(threads):
            oracle = _oracle()
            rc = oracle.lib().t4a_oracle_strided_to_strided(op["dtype"], oracle.ptr(numpy_view(self.host[op["dst"]])),
                                                            oracle.ptr(numpy_view(self.host[op["src"]])),
                                                            ctypes.byref(op["src_l"]), ctypes.byref(op["dst_l"]),
                                                            threads)
            assert rc == 0
            return 2 * op["n"] * op["es"]
        return cpu

    def check(self):
        for op in self.ops:
            op["run"](self.t4.stream_handle())
            same_bits(self.dev[op["dst"]], self.expect[op["dst"]], op["tag"])


class GatherScatterConfig(Config):
    """XLA gather of 4,194,304 rows from an F32 table
    [1048576,128] with I64 indices uniform in [0, 1048576) (seeds 6, 7), and scatter_add
    of F64 updates [4194304,128] normal(0,1) (seed 8) into a zeroed [1048576,128]
    destination with Zipf(s=1.1) row indices (seed 9).  Algorithmic bytes: gather =
    output + gathered rows + indices; scatter = updates + indices + destination read
    and write.

    Sharding: gather by index batches (rows shard_range of the 4M), the table
    replicated; scatter_add by destination rows, cyclically (row r on rank r mod N, so
    the Zipf-hot low rows spread over the ranks; contiguous slabs would give rank 0 about
    98% of the updates), every rank holding the whole index list and the updates and
    applying, with t4a_scatter_add_cyclic, only the updates whose row it owns.  Each
    rank then reads the indices and its rows' update rows, and no collective is
    needed."""

    name = "gather"
    ROWS, COLS, N = 1 << 20, 128, 1 << 22
    SAMPLE = 1 << 18

    def setup(self):
        import torch
        t4, abi = self.t4, self.abi
        R, C, N = self.ROWS, self.COLS, self.N
        gdev = gen_device()
        lo, hi = self.shard(N)
        n = hi - lo
        self.lo, self.n = lo, n
        table = gen_normal(6, R * C, torch.float32, gdev).reshape(R, C)
        self.keep("table", table)
        gidx_full = gen_rows_uniform(7, N, R, gdev)
        self.keep("gidx", gidx_full[lo:hi].contiguous())
        # scatter_add is sharded by destination rows (owner computes): every rank holds the
        # whole index list and every update row, and applies the updates of its own rows
        upd = gen_normal(8, N * C, torch.float64, gdev).reshape(N, C)
        sidx_full = gen_rows_zipf(9, N, R, 1.1, gdev)
        self.keep("upd", upd)
        self.keep("sidx", sidx_full)
        self.sharded = self.world > 1
        self.gplan = abi.gather_plan([0], [0], [1], [C, 1], 1, 2)
        self.splan = abi.scatter_plan([0], [0], [1], 1, 2, 2)
        own = R // self.world
        if not self.host_only:
            d = self.dev
            d["gout"] = torch.empty((n, C), dtype=torch.float32, device=self.device)
            if self.sharded:
                d["shard_out"] = torch.zeros((own, C), dtype=torch.float64, device=self.device)
            else:
                d["dest"] = torch.zeros((R, C), dtype=torch.float64, device=self.device)
            self.ws_bytes = t4.scatter_add_workspace_bytes(abi.F64, abi.I64, abi.numpy_layout([R, C]),
                                                           abi.layout([N, 1]), abi.numpy_layout([N, C]), self.splan)
            self.ws = torch.empty(max(self.ws_bytes, 16), dtype=torch.uint8, device=self.device)
            # single-GPU results of the whole ops (this rank's rows)
            full_gout = torch.empty((N, C), dtype=torch.float32, device=self.device)
            t4.gather_raw(t4.stream_handle(), abi.F32, abi.I64, vp(full_gout), abi.numpy_layout([N, C]), N * C,
                          vp(d["table"]), abi.numpy_layout([R, C]), R * C, vp(gidx_full.to(self.device)),
                          abi.layout([N, 1]), N, self.gplan)
            self.expect["gout"] = full_gout[lo:hi].clone()
            del full_gout
            full_upd = gen_normal(8, N * C, torch.float64, self.device).reshape(N, C)
            full_dest = torch.zeros((R, C), dtype=torch.float64, device=self.device)
            d_sidx = sidx_full.to(self.device)
            t4.scatter_add_rows(full_dest, d_sidx, full_upd)
            rows = slice(self.rank, R, self.world)  # this rank's rows (cyclic ownership)
            self.expect["dest"] = full_dest[rows].clone()
            # Two summation orders of the same n terms differ by at most 2 (n - 1) u sum|x|
            # (u = 2^-53, recursive summation): the per-element bound for the check.
            absum = torch.zeros((R, C), dtype=torch.float64, device=self.device).index_add_(0, d_sidx, full_upd.abs())
            count = torch.zeros(R, dtype=torch.float64, device=self.device).index_add_(
                0, d_sidx, torch.ones(N, dtype=torch.float64, device=self.device))
            self.expect["dest_bound"] = (2.0 * torch.clamp(count - 1, min=0) * 2.0 ** -53)[rows, None] * absum[rows]
            del full_upd, full_dest, absum, count
        self.host["gout"] = pinned(torch.empty((n, C), dtype=torch.float32))
        self.host["dest"] = pinned(torch.empty((own, C), dtype=torch.float64))
        self.ops = [
            dict(tag="gather-f32-4Mx128-of-1Mx128", config=4, kind="gather", launches=1,
                 bytes=N * C * 4 * 2 + N * 8, local_bytes=n * C * 4 * 2 + n * 8,
                 inputs=["table", "gidx"], outputs=["gout"]),
            dict(tag="scatter-add-f64-4Mx128-zipf-into-1Mx128", config=4, kind="scatter",
                 launches=3 if self.sharded else 2,
                 bytes=N * C * 8 + N * 8 + 2 * R * C * 8,
                 local_bytes=N * C * 8 // self.world + N * 8 + 2 * own * C * 8,
                 inputs=["sidx", "upd"], outputs=["shard_out" if self.sharded else "dest"]),
        ]
        if self.sharded:
            self.host["shard_out"] = self.host.pop("dest")
        for op in self.ops:
            op["run"] = self._runner(op)
            op["cpu"] = self._cpu(op)

    def _runner(self, op):
        t4, abi, d = self.t4, self.abi, self.dev
        R, C, n = self.ROWS, self.COLS, self.n

        def run(sh):
            if op["kind"] == "gather":
                t4.gather_raw(sh, abi.F32, abi.I64, vp(d["gout"]), abi.numpy_layout([n, C]), n * C, vp(d["table"]),
                              abi.numpy_layout([R, C]), R * C, vp(d["gidx"]), abi.layout([n, 1]), n, self.gplan)
                return
            N = self.N
            if self.sharded:
                # this rank's destination rows (r % world == rank), from the whole index list
                t4.check(t4.lib().t4a_scatter_add_cyclic(
                    sh, abi.F64, abi.I64, vp(d["shard_out"]), ctypes.byref(abi.numpy_layout([R, C])), R * C, C,
                    self.world, self.rank, vp(d["sidx"]), ctypes.byref(abi.layout([N, 1])), N, vp(d["upd"]),
                    ctypes.byref(abi.numpy_layout([N, C])), N * C, self.splan, vp(self.ws), self.ws_bytes),
                    "scatter_add_cyclic")
                return
            t4.scatter_add_raw(sh, abi.F64, abi.I64, vp(d["dest"]), abi.numpy_layout([R, C]), R * C, vp(d["sidx"]),
                               abi.layout([N, 1]), N, vp(d["upd"]), abi.numpy_layout([N, C]), N * C, self.splan,
                               vp(self.ws), self.ws_bytes)
        return run

    def _cpu(self, op):
        """The oracle on the first SAMPLE index rows of the op."""
        def cpu(threads):
            oracle = _oracle()
            abi = self.abi
            R, C, S = self.ROWS, self.COLS, self.SAMPLE
            h = self.host
            if op["kind"] == "gather":
                rc = oracle.lib().t4a_oracle_gather(abi.F32, abi.I64, oracle.ptr(h["gout"].numpy()),
                                                    oracle.ptr(h["table"].numpy()), oracle.ptr(h["gidx"].numpy()),
                                                    ctypes.byref(abi.numpy_layout([S, C])),
                                                    ctypes.byref(abi.numpy_layout([R, C])),
                                                    ctypes.byref(abi.layout([S, 1])), ctypes.byref(self.gplan),
                                                    threads)
                assert rc == 0
                return S * C * 4 * 2 + S * 8
            if "cpu_dest" not in h:
                import torch
                h["cpu_dest"] = torch.zeros((R, C), dtype=torch.float64)
            rc = oracle.lib().t4a_oracle_scatter_add(abi.F64, abi.I64, oracle.ptr(h["cpu_dest"].numpy()),
                                                     oracle.ptr(h["sidx"].numpy()), oracle.ptr(h["upd"].numpy()),
                                                     ctypes.byref(abi.numpy_layout([R, C])),
                                                     ctypes.byref(abi.layout([S, 1])),
                                                     ctypes.byref(abi.numpy_layout([S, C])),
                                                     ctypes.byref(self.splan), threads)
            assert rc == 0
            return S * C * 8 + S * 8 + 2 * R * C * 8 * S // self.N
        return cpu

    def after_timing(self):
        status = int(self.ws[:4].view(__import__("torch").int32).item())
        self.checks["scatter_status"] = status
        if status != 0:
            raise CheckFailed(f"scatter_add status {status}: a bounded wait of the fold ran out")

    def reset_scatter(self):
        """Untimed: the destination (or this rank's rows of it) back to zeros."""
        self.dev["shard_out" if self.sharded else "dest"].zero_()

    def check(self):
        import torch
        self.ops[0]["run"](self.t4.stream_handle())
        same_bits(self.dev["gout"], self.expect["gout"], "gather")
        self.reset_scatter()
        scatter = self.ops[1]
        scatter["run"](self.t4.stream_handle())
        got = self.dev["shard_out"] if self.sharded else self.dev["dest"]
        want, bound = self.expect["dest"], self.expect["dest_bound"]
        err = (got - want).abs()
        excess = (err - bound).max().item()
        self.checks["scatter_max_abs_err"] = err.max().item()
        self.checks["scatter_max_rel_err"] = (err / torch.clamp(want.abs(), min=1.0)).max().item()
        if excess > 0:
            raise CheckFailed(f"{scatter['tag']}: an element differs from the single-GPU sum by more than the "
                              f"reordering bound 2 (n-1) 2^-53 sum|x| (excess {excess:.3e})")
        self.reset_scatter()


class RrqrConfig(Config):
    """tall-skinny F64 RRQR of A = U V^T + 1e-10 N, U [65536,64],
    V [256,64], N [65536,256] normal(0,1) (NumPy generators seeded 10, 11, 12), 256
    steps of column_norms -> select_pivot -> swap_columns -> reflector ->
    apply_reflector.  One GPU: the fused driver t4a_rrqr (bit-identical to that loop of
    primitives).  N GPUs: row blocks of m/N rows with the per-step exchange of the
    column norms and reflector dots fused into the step kernels, as stores into every
    rank's memory over NVLink (t4a_b200.dist.RrqrRowsSharded, t4a_dist_rrqr_p2p).  Algorithmic
    bytes per factorization: sum over steps s of norms 8(m-s)(n-s) + apply
    16(m-s)(n-s-1) + swap 32m + reflector 16(m-s).  A is restored from a pristine device
    copy before every factorization, outside the op's events; in the end-to-end leg the
    timed host-to-device copy of A is the restore."""

    name = "rrqr"
    M, N, RANK = 65536, 256, 64
    CPU_STEPS = 16

    @classmethod
    def step_bytes(cls, s):
        m, n = cls.M, cls.N
        return 8 * (m - s) * (n - s) + 16 * (m - s) * (n - s - 1) + 32 * m + 16 * (m - s)

    def setup(self):
        import numpy as np
        import torch
        t4, abi = self.t4, self.abi
        m, n, k = self.M, self.N, self.RANK
        u = np.random.default_rng(10).standard_normal((m, k))
        v = np.random.default_rng(11).standard_normal((n, k))
        noise = np.random.default_rng(12).standard_normal((m, n))
        a = torch.from_numpy(np.asfortranarray(u @ v.T + 1e-10 * noise).ravel(order="K").copy())  # column-major
        from t4a_b200 import dist as t4dist
        self.sharded = self.world > 1
        r0, r1 = self.shard(m)
        self.rows = r1 - r0
        self.r0 = r0
        local = a.view(n, m)[:, r0:r1].contiguous().view(-1)  # this rank's rows, column-major
        self.keep("a", local)
        self.a_full = a
        bytes_all = sum(self.step_bytes(s) for s in range(n))
        if not self.host_only:
            d = self.dev
            d["pristine"] = d["a"].clone()
            d["perm"] = torch.empty(n, dtype=torch.int64, device=self.device)
            d["coeff"] = torch.empty(n, dtype=torch.float64, device=self.device)
            d["pivots"] = torch.empty(n, dtype=torch.int64, device=self.device)
            d["status"] = torch.zeros(1, dtype=torch.int64, device=self.device)
            if self.sharded:
                from t4a_b200 import dist as t4dist
                self.driver = t4dist.RrqrRowsSharded(d["a"], m, n, r0, n, exchange="p2p")
            else:
                self.layout = abi.layout([m, n])
                self.ws = torch.empty(t4.rrqr_workspace_bytes(abi.F64, self.layout), dtype=torch.uint8,
                                      device=self.device)
        for name in ("perm", "coeff", "pivots"):
            self.host[name] = pinned(torch.empty(n, dtype=torch.float64 if name == "coeff" else torch.int64))
        # the factorized block comes back into its own host buffer (the input stays pristine)
        self.host["a_out"] = pinned(torch.empty_like(local))
        if not self.host_only:
            self.dev["a_out"] = self.dev["a"]
        self.ops = [dict(tag="rrqr-f64-65536x256-256steps", config=5, bytes=bytes_all,
                         local_bytes=bytes_all * self.rows // m, inputs=["a"],
                         outputs=["a_out", "perm", "coeff", "pivots"], launches=None, e2e_restores=True)]
        op = self.ops[0]
        op["run"] = self._run
        op["prepare"] = self._prepare
        op["cpu"] = self._cpu
        op["launches"] = self.driver.launches if (self.sharded and not self.host_only) else 2 * n + 1

    def _prepare(self):
        self.dev["a"].copy_(self.dev["pristine"])

    def after_timing(self):
        status = int(self.dev["status"].item())
        self.checks["rrqr_status"] = status
        if status != 0:
            raise CheckFailed(f"RRQR status {status} after the timed factorizations")

    def close(self):
        if self.sharded and not self.host_only:
            self.driver.close()

    def _run(self, sh):
        t4, abi, d = self.t4, self.abi, self.dev
        if self.sharded:
            self.driver.run(sh, d["perm"], d["coeff"], d["pivots"], d["status"])
            return
        t4.check(t4.lib().t4a_rrqr(sh, abi.F64, vp(d["a"]), ctypes.byref(self.layout), self.M * self.N, self.N,
                                   vp(d["perm"]), vp(d["coeff"]), vp(d["pivots"]), vp(d["status"]), vp(self.ws),
                                   self.ws.numel()), "rrqr")

    def _cpu(self, threads):
        """The oracle's factorization loop for the first CPU_STEPS steps."""
        import numpy as np
        oracle = _oracle()
        work = self.a_full.numpy().copy()
        perm = np.zeros(self.N, np.int64)
        coeff = np.zeros(self.N)
        oracle.lib().t4a_oracle_rrqr_f64(oracle.ptr(work), self.M, self.N, self.CPU_STEPS, oracle.lptr(perm),
                                         oracle.ptr(coeff), 1e-8, 0.0, threads)
        return sum(self.step_bytes(s) for s in range(self.CPU_STEPS))

    def check(self):
        """One GPU: status 0 and the rank-revealing prefix (prefix_rank of R is 64).
        Sharded: pivots over the first 64 steps equal the single-GPU driver's, and the
        gathered factorization satisfies |Q R - A P| <= 1e-8 |A|."""
        import torch
        t4, abi, d = self.t4, self.abi, self.dev
        m, n = self.M, self.N
        self._prepare()
        self._run(t4.stream_handle())
        torch.cuda.synchronize()
        if int(d["status"].item()) != 0:
            raise CheckFailed(f"RRQR status {int(d['status'].item())}")
        if self.sharded:
            import torch.distributed as tdist
            from t4a_b200 import dist as t4dist
            work = t4dist.gather_rows_colmajor(d["a"], m, n, self.r0)
            ref_a = self.a_full.to(self.device)
            ref_layout = abi.layout([m, n])
            ref_ws = torch.empty(t4.rrqr_workspace_bytes(abi.F64, ref_layout), dtype=torch.uint8, device=self.device)
            rp, rc_, rv, rs = (torch.empty(n, dtype=torch.int64, device=self.device),
                               torch.empty(n, dtype=torch.float64, device=self.device),
                               torch.empty(n, dtype=torch.int64, device=self.device),
                               torch.zeros(1, dtype=torch.int64, device=self.device))
            t4.check(t4.lib().t4a_rrqr(t4.stream_handle(), abi.F64, vp(ref_a), ctypes.byref(ref_layout), m * n, n,
                                       vp(rp), vp(rc_), vp(rv), vp(rs), vp(ref_ws), ref_ws.numel()), "rrqr")
            piv, ref_piv = d["pivots"].cpu(), rv.cpu()
            diverge = next((i for i in range(n) if int(piv[i]) != int(ref_piv[i])), n)
            self.checks["rrqr_first_pivot_divergence"] = diverge
            if diverge < self.RANK:
                raise CheckFailed(f"RRQR pivots differ from the single-GPU driver at step {diverge} < {self.RANK}")
            wfull = work.view(n, m).t()
            q, qst = t4.rrqr_form_q(wfull, d["coeff"][:n])
            a_dev = self.a_full.to(self.device).view(n, m).t()
            resid = (torch.linalg.norm(q @ torch.triu(wfull[:n, :]) - a_dev[:, d["perm"]]) /
                     torch.linalg.norm(a_dev)).item()
            del q, wfull, a_dev
            self.checks["rrqr_residual_rel"] = resid
            if int(qst.item()) != 0:
                raise CheckFailed(f"RRQR Q formation status {int(qst.item())}")
            if not resid <= 1e-8:
                raise CheckFailed(f"RRQR residual |QR - AP| / |A| = {resid:.3e} > 1e-8")
            tdist.barrier()
        else:
            rank = torch.zeros(1, dtype=torch.int64, device=self.device)
            st = torch.zeros(1, dtype=torch.int64, device=self.device)
            rl = abi.layout([n, n], [1, m])
            launch = t4.plan_rrqr("prefix_rank", abi.F64, rl, m * n, 1, 1, 1e-8, 0.0)
            t4.launch_rrqr("prefix_rank", launch, t4.stream_handle(), vp(d["a"]), vp(rank), vp(st), abi.F64, rl,
                           1e-8, 0.0)
            self.checks["rrqr_prefix_rank"] = int(rank.item())
            if int(rank.item()) != self.RANK or int(st.item()) != 0:
                raise CheckFailed(f"RRQR prefix rank {int(rank.item())} (status {int(st.item())}), expected 64")


class RrqrLoopConfig(RrqrConfig):
    """Config 5 through the reference bench's loop of primitives instead of the fused
    driver (not in the default step; `--op rrqr-loop`, one GPU): initialize_permutation,
    then per step column_norms, select_pivot, swap_columns, reflector and, over the
    trailing columns, apply_reflector with the reflector column packed into its own
    buffer (t4a_copy_strided), each planned by this library's planner (plans made
    before timing) and launched through its launcher on the caller's stream.  This is the speed a caller
    that ports the reference one call at a time gets; the bits are the fused driver's.
    Same matrix, bytes, CPU leg and check as `rrqr`."""

    name = "rrqr-loop"

    def setup(self):
        import torch
        if self.world > 1:
            raise SystemExit("--op rrqr-loop runs on one GPU (the sharded RRQR is --op rrqr)")
        super().setup()
        t4, abi = self.t4, self.abi
        m, n = self.M, self.N
        op = self.ops[0]
        op["tag"] = "rrqr-loop-f64-65536x256-256steps"
        op["launches"] = 1 + 4 * n + 2 * (n - 1)
        if self.host_only:
            return
        wl, vl, cl = abi.layout([m, n]), abi.layout([n]), abi.layout([n])
        packed_l = abi.layout([m, n], [1, 0])
        self.loop_layouts = (wl, vl, cl, packed_l)
        span = m * n
        self.plans = dict(init=t4.plan_rrqr("initialize_permutation", n, n), steps=[])
        for step in range(n):
            self.plans["steps"].append(dict(
                norms=t4.plan_rrqr("column_norms", abi.F64, wl, span, vl, n, step),
                pivot=t4.plan_rrqr("select_pivot", abi.F64, vl, n, vl, n, 1, 1, step),
                swap=t4.plan_rrqr("swap_columns", abi.F64, wl, span, vl, n, 1, step),
                reflector=t4.plan_rrqr("reflector", abi.F64, wl, span, cl, n, step),
                apply=(t4.plan_rrqr("apply_reflector", abi.F64, packed_l, m, wl, span, cl, n, step, step + 1,
                                    n - step - 1) if n - step - 1 > 0 else None)))
        self.dev["norms"] = torch.empty(n, dtype=torch.float64, device=self.device)
        self.dev["packed"] = torch.empty(m, dtype=torch.float64, device=self.device)
        self.packed_dst = abi.layout([m])
        self.packed_src = [abi.layout([m], [1], step * m) for step in range(n)]

    def _run(self, sh):
        t4, abi, d = self.t4, self.abi, self.dev
        m, n = self.M, self.N
        wl, vl, cl, packed_l = self.loop_layouts
        dt = ctypes.c_int(abi.F64)
        t4.launch_rrqr("initialize_permutation", self.plans["init"], sh, vp(d["perm"]), ctypes.c_longlong(n),
                       ctypes.c_longlong(n))
        for step, p in enumerate(self.plans["steps"]):
            st = ctypes.c_longlong(step)
            t4.launch_rrqr("column_norms", p["norms"], sh, vp(d["a"]), vp(d["norms"]), dt, wl, vl, st)
            t4.launch_rrqr("select_pivot", p["pivot"], sh, vp(d["norms"]), vp(d["perm"]), vp(d["pivots"][step:]),
                           vp(d["status"]), dt, vl, vl, st)
            t4.launch_rrqr("swap_columns", p["swap"], sh, vp(d["a"]), vp(d["perm"]), vp(d["pivots"][step:]), dt,
                           wl, vl, st)
            t4.launch_rrqr("reflector", p["reflector"], sh, vp(d["a"]), vp(d["coeff"]), dt, wl, cl, st)
            if p["apply"] is not None:
                t4.copy_strided_raw(sh, abi.F64, vp(d["packed"]), self.packed_dst, m, vp(d["a"]),
                                    self.packed_src[step], m * n)
                t4.launch_rrqr("apply_reflector", p["apply"], sh, vp(d["packed"]), vp(d["a"]), vp(d["coeff"]), dt,
                               packed_l, wl, cl, st, ctypes.c_longlong(step + 1), ctypes.c_longlong(n - step - 1))

    def after_timing(self):
        super().after_timing()
        faults = self.t4.rrqr_primitive_faults()
        self.checks["rrqr_primitive_faults"] = faults
        if faults:
            raise CheckFailed(f"RRQR primitives: a bounded wait ran out (fault word {faults})")


CONFIGS = {"reduce": ReduceConfigs, "movement": MovementConfig, "gather": GatherScatterConfig, "rrqr": RrqrConfig,
           "rrqr-loop": RrqrLoopConfig}
ORDER = ["reduce", "movement", "gather", "rrqr"]


def build_configs(args, rank, world, device, host_only=False):
    names = ORDER if args.op == "all" else [args.op]
    groups = []
    for name in names:
        g = CONFIGS[name](rank, world, device, host_only)
        g.setup()
        if args.only:
            keep = set(args.only.split(","))
            g.ops = [op for op in g.ops if op["tag"] in keep]
        if g.ops:
            groups.append(g)
    return groups


def workload_config(groups, world):
    """The `config` object of the JSON line (identical in both arms)."""
    ops = [op for g in groups for op in g.ops]
    return {"workload": "BASELINE configs 1-5: " + ", ".join(sorted({g.name for g in groups})) if len(groups) > 1
            else f"BASELINE {groups[0].name}",
            "ops": [op["tag"] for op in ops],
            "bytes_per_step": sum(op["bytes"] for op in ops),
            "parallelism": f"sharded x{world}" if world > 1 else "1 gpu",
            "l2": "steady state: ops back to back, each op's inputs evicted by the ~12 GB step; "
                  "a flushed pass (256 MiB read before every op) is reported per op",
            "timing": "CUDA events per op on the launching stream, max over ranks"}


def dtype_string(groups):
    names = {"reduce": "f32,f64,c64", "movement": "f32,c64", "gather": "f32,f64,i64", "rrqr": "f64", "rrqr-loop": "f64"}
    return ";".join(names[g.name] for g in groups)


def run_ours(args, rank, world, local_rank):
    import torch
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist_on = world > 1

    def barrier():
        if dist_on:
            torch.distributed.barrier()

    groups = build_configs(args, rank, world, device)
    ops = [(g, op) for g in groups for op in g.ops]
    stream = torch.cuda.current_stream()
    sh = ctypes.c_void_p(stream.cuda_stream)
    torch.cuda.synchronize()

    # Every rank checks its shards against the single-GPU result before timing.
    # Ranks agree on every group's outcome before the next group runs, so no rank goes on
    # launching kernels that store into another rank's memory (the sharded RRQR) after
    # that rank has stopped.
    checks = {}
    if not args.no_check:
        for g in groups:
            err = None
            try:
                g.check()
            except CheckFailed as e:
                err = e
            torch.cuda.synchronize()
            if dist_on:
                flag = torch.tensor([0 if err is None else 1], dtype=torch.int32, device=device)
                torch.distributed.all_reduce(flag)
                if int(flag.item()) and err is None:
                    err = CheckFailed(f"another rank's check of the {g.name} ops failed")
            if err is not None:
                raise err
            checks.update(g.checks)
        torch.cuda.synchronize()
    for g in groups:
        g.expect.clear()
    torch.cuda.empty_cache()
    barrier()

    def one_step(events=None, flush=None):
        for j, (g, op) in enumerate(ops):
            if op.get("prepare"):
                op["prepare"]()
            if flush is not None:
                flush.sum(dtype=torch.int64)
            if events is not None:
                events[j][0].record(stream)
            op["run"](sh)
            if events is not None:
                events[j][1].record(stream)

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    barrier()

    # Timed region: K steady-state steps.
    events = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in ops]
              for _ in range(args.steps)]
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    with sampler:
        # Hold the stream with a bounded sleep kernel while the first steps are enqueued,
        # so each event pair brackets GPU work, not the host's launch latency.
        torch.cuda._sleep(int(2e8))
        r0.record(stream)
        for k in range(args.steps):
            one_step(events[k])
        r1.record(stream)
        torch.cuda.synchronize()
    barrier()
    wall = time.perf_counter() - wall0
    per_op = [[events[k][j][0].elapsed_time(events[k][j][1]) for k in range(args.steps)] for j in range(len(ops))]
    totals = [sum(x) for x in per_op]
    stats = torch.tensor([sum(totals), r0.elapsed_time(r1)] + totals, device=device, dtype=torch.float64)
    if dist_on:
        torch.distributed.all_reduce(stats, op=torch.distributed.ReduceOp.MAX)
    kernel_ms, region_ms = stats[0].item(), stats[1].item()
    totals_max = stats[2:].tolist()
    job_bytes = sum(op["bytes"] for _, op in ops)
    value = job_bytes * args.steps / (kernel_ms / 1e3) / 1e9

    # Status words of the timed steps: a bounded wait that ran out fails the run.
    for g in groups:
        g.after_timing()

    # Cold pass: L2 flushed (256 MiB read) before every op.
    flush = torch.ones(256 * MIB, dtype=torch.uint8, device=device)
    cold_steps = min(args.steps, 3)
    cold_events = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in ops]
                   for _ in range(cold_steps)]
    barrier()
    torch.cuda.synchronize()
    for k in range(cold_steps):
        one_step(cold_events[k], flush)
    torch.cuda.synchronize()
    cold = torch.tensor([sum(cold_events[k][j][0].elapsed_time(cold_events[k][j][1]) for k in range(cold_steps))
                         for j in range(len(ops))], device=device, dtype=torch.float64)
    if dist_on:
        torch.distributed.all_reduce(cold, op=torch.distributed.ReduceOp.MAX)
    cold = cold.tolist()
    del flush

    e2e = measure_e2e(args, groups, ops, stream, sh, device, world, barrier)

    peak, peak_kind = read_peaks()
    ops_detail = {}
    for j, (g, op) in enumerate(ops):
        ms = totals_max[j] / args.steps
        cms = cold[j] / cold_steps
        ops_detail[op["tag"]] = {
            "config": op["config"], "bytes": op["bytes"], "us": round(1e3 * ms, 2),
            "gbs": round(op["bytes"] / (ms / 1e3) / 1e9, 1), "frac": round(op["bytes"] / (ms / 1e3) / 1e9 / peak, 3),
            "us_flushed": round(1e3 * cms, 2),
            "frac_flushed": round(op["bytes"] / (cms / 1e3) / 1e9 / peak, 3)}
    dom = max(range(len(ops)), key=lambda j: totals_max[j])
    dom_op = ops[dom][1]
    dom_ms = totals_max[dom] / args.steps
    achieved = dom_op["bytes"] / (dom_ms / 1e3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(region_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong",  # the global problem is fixed; N ranks share it
        "vs_baseline": None,
        "dtype": dtype_string(groups),
        "data": "synthetic (seeded SplitMix64 normal/uniform/Zipf streams; NumPy generators for RRQR)",
        "config": workload_config(groups, world),
        "roofline": {"bound": "hbm", "kernel": dom_op["tag"], "achieved": round(achieved, 1), "peak": peak,
                     "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": profile_traffic(dom_op["tag"]) if world == 1 else None,
                     "unit_of_launch": "one whole op (RRQR: one 256-step factorization)"},
        "ops": ops_detail,
        "e2e": e2e,
        "gpu_launches": sum(op["launches"] for _, op in ops) * args.steps,
        "clocks": sampler.summary(),
        "checks": dict(checks, passed=not args.no_check, against="single-GPU result of the same library"),
        "kernel_ms_per_step": round(kernel_ms / args.steps, 4),
        "wall_s_timed_region": round(wall, 3),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(groups, args)
    torch.cuda.synchronize()
    for g in groups:
        g.close()
    return line


def measure_e2e(args, groups, ops, stream, sh, device, world, barrier):
    """Same ops through the C ABI from pinned host memory: every input tensor of a step is
    copied in before its first op, every op's outputs are copied out after it, on three
    streams (host-to-device copies, the ops, device-to-host copies) with buffer-level
    events, as a caller pipelines host data through the library."""
    import torch
    s_in = torch.cuda.Stream(device=device)
    s_out = torch.cuda.Stream(device=device)
    h2d = d2h = 0
    for g in groups:
        names_in = []
        for op in g.ops:
            for nm in op["inputs"]:
                if nm not in names_in:
                    names_in.append(nm)
        h2d += sum(g.host[nm].numel() * g.host[nm].element_size() for nm in names_in)
        d2h += sum(g.host[nm].numel() * g.host[nm].element_size() for op in g.ops for nm in op["outputs"])
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    read_done, copied_out = {}, {}
    for _ in range(args.steps):
        for g in groups:
            copied = set()
            for op in g.ops:
                with torch.cuda.stream(s_in):
                    for nm in op["inputs"]:
                        if nm in copied:
                            continue
                        d = g.dev[nm]
                        if d.data_ptr() in read_done:
                            s_in.wait_event(read_done[d.data_ptr()])
                        d.copy_(g.host[nm], non_blocking=True)
                        copied.add(nm)
                    arrived = torch.cuda.Event()
                    arrived.record(s_in)
                stream.wait_event(arrived)
                for nm in op["outputs"]:
                    d = g.dev[nm]
                    if d.data_ptr() in copied_out:
                        stream.wait_event(copied_out[d.data_ptr()])
                if op.get("prepare") and not op.get("e2e_restores"):
                    op["prepare"]()
                op["run"](sh)
                done = torch.cuda.Event()
                done.record(stream)
                for nm in op["inputs"]:
                    read_done[g.dev[nm].data_ptr()] = done
                s_out.wait_event(done)
                with torch.cuda.stream(s_out):
                    for nm in op["outputs"]:
                        g.host[nm].copy_(g.dev[nm], non_blocking=True)
                    out_done = torch.cuda.Event()
                    out_done.record(s_out)
                for nm in op["outputs"]:
                    copied_out[g.dev[nm].data_ptr()] = out_done
    tail_in, tail_out = torch.cuda.Event(), torch.cuda.Event()
    tail_in.record(s_in)
    tail_out.record(s_out)
    stream.wait_event(tail_in)
    stream.wait_event(tail_out)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], device=device, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    ms = ms.item()
    job_bytes = sum(op["bytes"] for g in groups for op in g.ops)
    return {"value": round(job_bytes * args.steps / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms / args.steps, 3),
            "per_rank": world > 1}


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample_text(groups):
    parts = []
    for g in groups:
        if g.name == "reduce":
            parts.append("config 1 whole, config 3 on 1/16 of a non-reduced axis")
        elif g.name == "movement":
            parts.append("config 2 whole")
        elif g.name == "gather":
            parts.append(f"config 4 on the first {GatherScatterConfig.SAMPLE} of {GatherScatterConfig.N} index rows")
        elif g.name in ("rrqr", "rrqr-loop"):
            parts.append(f"config 5's first {RrqrConfig.CPU_STEPS} of {RrqrConfig.N} factorization steps")
    return "; ".join(parts)


def cpu_step(groups, threads):
    nbytes = 0
    for g in groups:
        for op in g.ops:
            nbytes += op["cpu"](threads)
    return nbytes


def cpu_baseline(groups, args, steps=3):
    """The oracle port over every host core on a bounded sample of every op, `steps` times."""
    threads = host_threads()
    cpu_step(groups, threads)  # warm-up (page faults of the output buffers)
    t0 = time.perf_counter()
    nbytes = 0
    for _ in range(steps):
        nbytes += cpu_step(groups, threads)
    dt = time.perf_counter() - t0
    return {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{steps} steps of: {cpu_sample_text(groups)} "
                      f"({nbytes / steps / MIB:.0f} MiB algorithmic per step), {dt:.2f} s"}


def run_reference(args, rank, world):
    """CPU implementation of the path on the host cores (see module docstring)."""
    if rank != 0:
        return None
    import torch
    device = gen_device()
    groups = build_configs(args, 0, 1, device, host_only=True)
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    threads = host_threads()
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_step(groups, threads)
    t0 = time.perf_counter()
    nbytes = 0
    for _ in range(args.steps):
        nbytes += cpu_step(groups, threads)
    dt = time.perf_counter() - t0
    value = nbytes / dt / 1e9
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * dt / args.steps, 3), "higher_is_better": True,
        "scaling": "strong",  # the global problem is fixed; N ranks share it
        "vs_baseline": None, "dtype": dtype_string(groups),
        "data": "synthetic (seeded SplitMix64 normal/uniform/Zipf streams; NumPy generators for RRQR)",
        "config": workload_config(groups, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps of: {cpu_sample_text(groups)} "
                                   f"({nbytes / args.steps / MIB:.0f} MiB algorithmic per step)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--op", default="all", choices=["all"] + ORDER + ["rrqr-loop"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true", help="skip the per-rank check against the single-GPU result")
    ap.add_argument("--only", default=None, help="comma-separated op tags to run (profiling)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    import torch
    # Libraries may print to the process's stdout (NCCL's version banner at communicator
    # set-up); send file descriptor 1 to stderr while they run, so that stdout carries
    # the one JSON line only.
    sys.stdout.flush()
    saved_stdout = os.dup(1)
    os.dup2(2, 1)
    line = None
    failed = None
    try:
        if world > 1:
            import datetime
            torch.cuda.set_device(local_rank)
            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                                 device_id=torch.device("cuda", local_rank))
        try:
            line = run_ours(args, rank, world, local_rank)
        except CheckFailed as exc:
            failed = f"rank {rank}: {exc}"
        finally:
            if world > 1:
                torch.distributed.destroy_process_group()
    finally:
        sys.stdout.flush()
        os.dup2(saved_stdout, 1)
        os.close(saved_stdout)
    if failed:
        print(json.dumps({"metric": METRIC, "error": failed}), flush=True)
        sys.exit(3)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
