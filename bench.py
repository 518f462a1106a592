"""Benchmark of the t4a_b200 hot path on B200 (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--op NAME]

Headline workload ("Permutation movement"): one step is
  * F32 [64,64,64,64] materialized in permutation (3,1,0,2),
  * C64 [16]^6 materialized in permutation (5,0,4,1,3,2),
  * F32 [64,64,64,64] with axis 2 reversed (negated stride, rebased offset),
through the library's strided-copy entry (t4a_copy_strided / the strided_to_strided
plan).  Inputs are seeded normal(0,1) values (synthetic; no dataset is involved).
`value` is the algorithmic HBM traffic (each element read once and written once)
per second of kernel time, summed over all ranks; each rank copies its own full
workload (weak scaling, no collective: the movement ops shard by independent
tensors).  L2 is flushed before every op (a 256 MiB read, outside the timed events),
so every kernel streams from HBM and starts without another kernel's dirty lines.

`--op` selects another BASELINE config as the workload (reduce; gather = gather and
scatter_add; rrqr) for the secondary lines; the driver's runs use the default.

`--impl reference` times the reference path's CPU implementation on this box's host
cores: the reference library has no CPU path of its own (its Rust crate only plans),
so the arm runs the C++ restatement under oracle/ (the same semantics, the same
inputs), multi-threaded over the host cores, on a bounded sample per step.
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


def _oracle():
    """The CPU restatement (oracle/), used only by the CPU-baseline leg and --impl reference."""
    if os.path.join(ROOT, "oracle") not in sys.path:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    return oracle

MIB = 1 << 20


def read_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            data = json.load(fh)
        return float(data["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profile_traffic(kernel_tag):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary, or None."""
    for name in sorted(os.listdir(os.path.join(ROOT, "profiles"))) if os.path.isdir(os.path.join(ROOT, "profiles")) else []:
        if not name.endswith((".md", ".txt")):
            continue
        with open(os.path.join(ROOT, "profiles", name)) as fh:
            for line in fh:
                if line.startswith(f"traffic_per_launch[{kernel_tag}]"):
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
# Workloads.  Each builds its device inputs and returns a list of ops; an op is
# (tag, algorithmic bytes, launch(stream), host_inputs, device_inputs, device_outputs).
# ---------------------------------------------------------------------------

def gen_device():
    """A GPU to generate inputs on when one is visible (the reference arm times only host
    work), else None."""
    import torch
    return torch.device("cuda", 0) if torch.cuda.is_available() else None


def _splitmix_bits(seed, start, count):
    """Draws start+1 .. start+count of a SplitMix64 stream from state `seed` (counter-based)."""
    import numpy as np
    with np.errstate(over="ignore"):
        k = np.arange(start + 1, start + count + 1, dtype=np.uint64)
        z = np.uint64(seed) + k * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def _srl(z, n):
    """Logical right shift of an int64 tensor holding uint64 bits."""
    return (z >> n) & ((1 << (64 - n)) - 1)


def _i64(x):
    return x - (1 << 64) if x >= 1 << 63 else x


def _splitmix_bits_torch(seed, start, count, device):
    import torch
    k = torch.arange(start + 1, start + count + 1, dtype=torch.int64, device=device)
    z = _i64(seed) + k * _i64(0x9E3779B97F4A7C15)
    z = (z ^ _srl(z, 30)) * _i64(0xBF58476D1CE4E5B9)
    z = (z ^ _srl(z, 27)) * _i64(0x94D049BB133111EB)
    return z ^ _srl(z, 31)


def gen_normal(seed, count, np_dtype, device=None, chunk=1 << 24):
    """Seeded normal(0,1) values: Box-Muller over a SplitMix64 stream (draws 2i, 2i+1
    make value i).  On `device` when given (torch int64 arithmetic wraps like uint64),
    else with NumPy; both produce the same values.  Returns a CPU torch tensor."""
    import numpy as np
    import torch
    if device is None or not torch.cuda.is_available():
        out = np.empty(count, dtype=np_dtype)
        for lo in range(0, count, chunk):
            n = min(chunk, count - lo)
            z = _splitmix_bits(seed, 2 * lo, 2 * n)
            u = ((z >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / (1 << 53))
            out[lo:lo + n] = np.sqrt(-2.0 * np.log(u[0::2])) * np.cos(2 * np.pi * u[1::2])
        return torch.from_numpy(out)
    tdt = {np.float32: torch.float32, np.float64: torch.float64}[np_dtype]
    out = torch.empty(count, dtype=tdt)
    for lo in range(0, count, chunk):
        n = min(chunk, count - lo)
        z = _splitmix_bits_torch(seed, 2 * lo, 2 * n, device)
        u = (_srl(z, 11).double() + 0.5) * (1.0 / (1 << 53))
        v = torch.sqrt(-2.0 * torch.log(u[0::2])) * torch.cos(2 * np.pi * u[1::2])
        out[lo:lo + n] = v.to(tdt).cpu()
    return out


def gen_uniform(seed, count, np_dtype, device=None, chunk=1 << 24):
    """Seeded uniform(-1,1) values on a 2^-52 grid: (next >> 11) * 2^-52 - 1."""
    import numpy as np
    import torch
    if device is None or not torch.cuda.is_available():
        out = np.empty(count, dtype=np_dtype)
        for lo in range(0, count, chunk):
            n = min(chunk, count - lo)
            z = _splitmix_bits(seed, lo, n)
            out[lo:lo + n] = (z >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 52)) - 1.0
        return torch.from_numpy(out)
    tdt = {np.float32: torch.float32, np.float64: torch.float64}[np_dtype]
    out = torch.empty(count, dtype=tdt)
    for lo in range(0, count, chunk):
        n = min(chunk, count - lo)
        z = _splitmix_bits_torch(seed, lo, n, device)
        out[lo:lo + n] = (_srl(z, 11).double() * (1.0 / (1 << 52)) - 1.0).to(tdt).cpu()
    return out


class Workload:
    """Shared defaults: one input tensor (host_in[i] -> dev_in[i]) and one output
    (dev_out[j] -> host_out[j]) per op; the CPU leg runs the whole step."""

    def e2e_inputs(self, op):
        return [(self.host_in[op["i"]], self.dev_in[op["i"]])]

    def e2e_outputs(self, op):
        j = op.get("j", op["i"])
        return [(self.dev_out[j], self.host_out[j])]

    def cpu_units(self):
        return self.units()

    def cpu_sample(self):
        return f"the full {self.name} step"


class MovementWorkload(Workload):
    name = "config2-permutation-movement"
    dtype = "f32,c64"

    def __init__(self, device=None):
        import numpy as np
        import torch
        import t4a_b200 as t4
        from t4a_b200 import abi
        self.t4, self.abi = t4, abi
        self.device = device
        gdev = device if device is not None else gen_device()
        a = gen_normal(2, 64 ** 4, np.float32, gdev)
        b = torch.stack([gen_normal(3, 16 ** 6, np.float64, gdev), gen_normal(3 + 1000, 16 ** 6, np.float64, gdev)],
                        dim=1).reshape(-1)  # interleaved (re, im)
        c = gen_normal(4, 64 ** 4, np.float32, gdev)
        pin = device is not None
        host = [a, b, c]
        self.host_in = [h.pin_memory() for h in host] if pin else host
        self.host_out = [torch.empty_like(h).pin_memory() if pin else torch.empty_like(h) for h in host]
        if device is not None:
            self.dev_in = [h.to(device) for h in self.host_in]
            self.dev_out = [torch.empty_like(d) for d in self.dev_in]

        def perm_layout(shape, perm):
            st, s = [], 1
            for e in reversed(shape):
                st.insert(0, s)
                s *= e
            return abi.numpy_layout([shape[p] for p in perm], [st[p] for p in perm])

        self.ops = []
        specs = [
            ("perm-f32-64^4", abi.F32, perm_layout([64] * 4, (3, 1, 0, 2)), 64 ** 4, 4),
            ("perm-c64-16^6", abi.C64, perm_layout([16] * 6, (5, 0, 4, 1, 3, 2)), 16 ** 6, 16),
            ("reverse-f32-64^4", abi.F32, abi.numpy_layout([64] * 4, [64 ** 3, 64 ** 2, -64, 1], 63 * 64), 64 ** 4, 4),
        ]
        for i, (tag, dt, src_l, n, es) in enumerate(specs):
            dst_l = abi.layout(src_l.extents_list())
            self.ops.append(dict(tag=tag, dtype=dt, src_l=src_l, dst_l=dst_l, n=n, bytes=2 * n * es, i=i))

    def units(self):
        return sum(op["bytes"] for op in self.ops)

    def run_op(self, op, stream_handle, dev_in=None, dev_out=None):
        i = op["i"]
        src = (dev_in or self.dev_in)[i]
        dst = (dev_out or self.dev_out)[i]
        self.t4.copy_strided_raw(stream_handle, op["dtype"], ctypes.c_void_p(dst.data_ptr()), op["dst_l"], op["n"],
                                 ctypes.c_void_p(src.data_ptr()), op["src_l"], op["n"])

    def cpu_op(self, op, threads, srcs, dsts):
        oracle = _oracle()
        host_src, host_dst = srcs[op["i"]], dsts[op["i"]]
        rc = oracle.lib().t4a_oracle_strided_to_strided(op["dtype"], oracle.ptr(host_dst), oracle.ptr(host_src),
                                                        ctypes.byref(op["src_l"]), ctypes.byref(op["dst_l"]), threads)
        assert rc == 0

    def host_arrays(self):
        return [h.numpy() for h in self.host_in], [h.numpy() for h in self.host_out]



class ReduceWorkload(Workload):
    """BASELINE configs[2] (and configs[0]): single-axis reductions.

    F32 [4096,4096,32] normal(0,1): sum, sum_squares and max over each NumPy axis; C64
    [8192,8192] sum over axis 1; F64 [256,1024,64] uniform(-1,1) sum and max over axis 1.
    Each op is one whole reduction (t4a_reduce: pass 1 + combine, or a direct pass)."""

    name = "config3-reduction-sweep+config1"
    dtype = "f32,f64,c64"

    def __init__(self, device=None):
        import numpy as np
        import torch
        import t4a_b200 as t4
        from t4a_b200 import abi
        self.t4, self.abi = t4, abi
        self.device = device
        gdev = device if device is not None else gen_device()
        big = gen_normal(4, 4096 * 4096 * 32, np.float32, gdev).reshape(4096, 4096, 32)
        c = torch.complex(gen_normal(5, 8192 * 8192, np.float64, gdev),
                          gen_normal(5 + 1000, 8192 * 8192, np.float64, gdev)).reshape(8192, 8192)
        u = gen_uniform(0, 256 * 1024 * 64, np.float64, gdev).reshape(256, 1024, 64)
        self.host_in = [big, c, u]
        if device is not None:
            self.host_in = [h.pin_memory() for h in self.host_in]
            self.dev_in = [h.to(device) for h in self.host_in]
        specs = []
        for ax in (0, 1, 2):
            for op, tag in ((abi.SUM, "sum"), (abi.SUM_SQUARES, "sumsq"), (abi.MAX, "max")):
                specs.append((f"{tag}-f32-4096x4096x32-axis{ax}", 0, ax, op))
        specs.append(("sum-c64-8192x8192-axis1", 1, 1, abi.SUM))
        specs.append(("sum-f64-256x1024x64-axis1", 2, 1, abi.SUM))
        specs.append(("max-f64-256x1024x64-axis1", 2, 1, abi.MAX))
        self.ops = []
        self.dev_out, self.host_out, self.workspace = [], [], None
        need_ws = 0
        for j, (tag, i, ax, op) in enumerate(specs):
            x = self.host_in[i]
            shape = list(x.shape)
            oshape = list(shape)
            oshape[ax] = 1
            dt = t4.torch_dtype_tag(x)
            in_l = abi.numpy_layout(shape)
            out_l = abi.numpy_layout(oshape)
            n_out = int(np.prod(oshape))
            ws = t4.reduce_workspace_bytes(dt, op, out_l, n_out, in_l, x.numel(), len(shape) - 1 - ax)
            need_ws = max(need_ws, ws)
            esize = x.element_size()
            self.ops.append(dict(tag=tag, i=i, j=j, op=op, dtype=dt, in_l=in_l, out_l=out_l, n_in=x.numel(),
                                 n_out=n_out, axis=len(shape) - 1 - ax, ws=ws, np_axis=ax,
                                 bytes=(x.numel() + n_out) * esize, launches=2 if ws else 1))
            self.host_out.append(torch.empty(oshape, dtype=x.dtype).pin_memory() if device is not None
                                 else torch.empty(oshape, dtype=x.dtype))
            if device is not None:
                self.dev_out.append(torch.empty(oshape, dtype=x.dtype, device=device))
        if device is not None:
            self.workspace = torch.empty(max(need_ws, 16), dtype=torch.uint8, device=device)

    def units(self):
        return sum(op["bytes"] for op in self.ops)

    def run_op(self, op, stream_handle, dev_in=None, dev_out=None):
        src = (dev_in or self.dev_in)[op["i"]]
        dst = (dev_out or self.dev_out)[op["j"]]
        self.t4.reduce_raw(stream_handle, op["dtype"], op["op"], ctypes.c_void_p(dst.data_ptr()), op["out_l"],
                           op["n_out"], ctypes.c_void_p(src.data_ptr()), op["in_l"], op["n_in"], op["axis"], 32,
                           ctypes.c_void_p(self.workspace.data_ptr()), op["ws"])

    def cpu_op(self, op, threads, srcs, dsts):
        oracle = _oracle()
        host_src, host_dst = srcs[op["i"]], dsts[op["j"]]
        rc = oracle.lib().t4a_oracle_reduce_threaded(op["dtype"], op["op"], oracle.ptr(host_dst),
                                                     ctypes.byref(op["out_l"]), oracle.ptr(host_src),
                                                     ctypes.byref(op["in_l"]), op["axis"], 32, threads)
        assert rc == 0

    def host_arrays(self):
        srcs = [h.numpy() for h in self.host_in]
        outs = [h.numpy() for h in self.host_out]
        return srcs, outs


class GatherScatterWorkload(Workload):
    """XLA gather of 4,194,304 rows from an F32 table
    [1,048,576,128] with I64 indices uniform in [0, 1048576) (seeds 6, 7), and
    scatter_add of F64 updates [4,194,304,128] normal(0,1) (seed 8) into a
    [1,048,576,128] destination with Zipf(s=1.1) row indices (seed 9; inverse CDF over
    ranks 1..1048576, row = rank - 1).  Algorithmic bytes: gather = output + gathered
    rows + indices; scatter = updates + indices + destination read and write.  The
    destination is zeroed once; the caller's operand copy (copy_exact) is not part of
    the timed scatter op.  The CPU leg runs the oracle on the first 262,144 index rows
    of each op."""

    name = "config4-gather-scatter"
    dtype = "f32 (gather), f64 (scatter); i64 indices"
    ROWS, COLS, N, SAMPLE = 1 << 20, 128, 1 << 22, 1 << 18

    def __init__(self, device=None):
        import numpy as np
        import torch
        import t4a_b200 as t4
        from t4a_b200 import abi
        self.t4, self.abi = t4, abi
        self.device = device
        gdev = device if device is not None else gen_device()
        R, C, N = self.ROWS, self.COLS, self.N
        table = gen_normal(6, R * C, np.float32, gdev).reshape(R, C)
        gidx = self._uniform_rows(7, N, R, gdev)
        upd = gen_normal(8, N * C, np.float64, gdev).reshape(N, C)
        sidx = self._zipf_rows(9, N, R, 1.1, gdev)
        dest0 = torch.zeros((R, C), dtype=torch.float64)
        pin = device is not None
        self.host = {"table": table, "gidx": gidx, "upd": upd, "sidx": sidx, "dest": dest0,
                     "gout": torch.empty((N, C), dtype=torch.float32)}
        if pin:
            self.host = {k: v.pin_memory() for k, v in self.host.items()}
            self.dev = {k: v.to(device) for k, v in self.host.items()}
        self.gplan = abi.gather_plan([0], [0], [1], [C, 1], 1, 2)
        self.splan = abi.scatter_plan([0], [0], [1], 1, 2, 2)
        self.ws_bytes = t4.scatter_add_workspace_bytes(abi.F64, abi.I64, abi.numpy_layout([R, C]),
                                                       abi.layout([N, 1]), abi.numpy_layout([N, C]), self.splan)
        if pin:
            self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=device)
        # On N > 1 ranks the scatter has its exchange step: every rank adds its own
        # update batch into a full-size partial destination and one NCCL reduce-scatter
        # leaves it its 1/N of the destination rows (t4a_b200.dist); the gather needs no
        # collective (each rank gathers its own batch).
        self.sharded = pin and torch.distributed.is_available() and torch.distributed.is_initialized() \
            and torch.distributed.get_world_size() > 1
        if self.sharded:
            from t4a_b200 import dist as t4dist
            self.t4dist = t4dist
            world = torch.distributed.get_world_size()
            self.partial = t4dist.scatter_partial(self.dev["dest"])
            self.shard_out = torch.empty((R // world, C), dtype=torch.float64, device=device)
        self.ops = [
            dict(tag="gather-f32-4Mx128-of-1Mx128", kind="gather", i=0,
                 bytes=N * C * 4 * 2 + N * 8),
            dict(tag="scatter-add-f64-4Mx128-zipf-into-1Mx128", kind="scatter", i=1, launches=2,
                 bytes=N * C * 8 + N * 8 + 2 * R * C * 8),
        ]

    @staticmethod
    def _uniform_rows(seed, n, rows, gdev):
        import numpy as np
        import torch
        if gdev is None:
            z = _splitmix_bits(seed, 0, n)
            u = (z >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
            return torch.from_numpy((u * rows).astype(np.int64))
        z = _splitmix_bits_torch(seed, 0, n, gdev)
        u = _srl(z, 11).double() * (1.0 / (1 << 53))
        return (u * rows).to(torch.int64).cpu()

    @staticmethod
    def _zipf_rows(seed, n, rows, s, gdev):
        import numpy as np
        import torch
        w = np.arange(1, rows + 1, dtype=np.float64) ** -s
        cdf = np.cumsum(w)
        cdf /= cdf[-1]
        if gdev is None:
            z = _splitmix_bits(seed, 0, n)
            u = (z >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
            return torch.from_numpy(np.minimum(np.searchsorted(cdf, u, side="right"), rows - 1).astype(np.int64))
        z = _splitmix_bits_torch(seed, 0, n, gdev)
        u = _srl(z, 11).double() * (1.0 / (1 << 53))
        r = torch.searchsorted(torch.from_numpy(cdf).to(gdev), u, right=True)
        return torch.clamp(r, max=rows - 1).to(torch.int64).cpu()

    def units(self):
        return sum(op["bytes"] for op in self.ops)

    def run_op(self, op, stream_handle, dev_in=None, dev_out=None):
        t4, abi, d = self.t4, self.abi, self.dev
        R, C, N = self.ROWS, self.COLS, self.N
        vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        if op["kind"] == "gather":
            t4.gather_raw(stream_handle, abi.F32, abi.I64, vp(d["gout"]), abi.numpy_layout([N, C]), N * C,
                          vp(d["table"]), abi.numpy_layout([R, C]), R * C, vp(d["gidx"]), abi.layout([N, 1]), N,
                          self.gplan)
        elif self.sharded:
            self.t4dist.scatter_add_rows_sharded(self.partial, d["sidx"].view(N), d["upd"], workspace=self.ws,
                                                 out=self.shard_out)
        else:
            t4.scatter_add_raw(stream_handle, abi.F64, abi.I64, vp(d["dest"]), abi.numpy_layout([R, C]), R * C,
                               vp(d["sidx"]), abi.layout([N, 1]), N, vp(d["upd"]), abi.numpy_layout([N, C]), N * C,
                               self.splan, vp(self.ws), self.ws_bytes)

    def e2e_inputs(self, op):
        if op["kind"] == "gather":
            keys = ["table", "gidx"]
        else:
            keys = ["sidx", "upd"] if self.sharded else ["dest", "sidx", "upd"]
        return [(self.host[k], self.dev[k]) for k in keys]

    def e2e_outputs(self, op):
        if op["kind"] != "gather" and self.sharded:
            return [(self.shard_out, self.host["dest"][:self.shard_out.shape[0]])]
        k = "gout" if op["kind"] == "gather" else "dest"
        return [(self.dev[k], self.host[k])]

    def host_arrays(self):
        return self.host, None

    def cpu_units(self):
        return sum(op["bytes"] for op in self.ops) * self.SAMPLE // self.N

    def cpu_sample(self):
        return f"the first {self.SAMPLE} of {self.N} index rows of each {self.name} op"

    def cpu_op(self, op, threads, srcs, dsts):
        oracle = _oracle()
        abi = self.abi
        R, C, S = self.ROWS, self.COLS, self.SAMPLE
        h = srcs
        if op["kind"] == "gather":
            rc = oracle.lib().t4a_oracle_gather(abi.F32, abi.I64, oracle.ptr(h["gout"].numpy()),
                                                oracle.ptr(h["table"].numpy()), oracle.ptr(h["gidx"].numpy()),
                                                ctypes.byref(abi.numpy_layout([S, C])),
                                                ctypes.byref(abi.numpy_layout([R, C])),
                                                ctypes.byref(abi.layout([S, 1])), ctypes.byref(self.gplan), threads)
        else:
            rc = oracle.lib().t4a_oracle_scatter_add(abi.F64, abi.I64, oracle.ptr(h["dest"].numpy()),
                                                     oracle.ptr(h["sidx"].numpy()), oracle.ptr(h["upd"].numpy()),
                                                     ctypes.byref(abi.numpy_layout([R, C])),
                                                     ctypes.byref(abi.layout([S, 1])),
                                                     ctypes.byref(abi.numpy_layout([S, C])),
                                                     ctypes.byref(self.splan), threads)
        assert rc == 0



class RrqrWorkload(Workload):
    """tall-skinny F64 RRQR of A = U V^T + 1e-10 N, U [65536,64],
    V [256,64], N [65536,256] normal(0,1) (NumPy generators seeded 10, 11, 12): 256
    steps of column_norms -> select_pivot -> swap_columns -> reflector ->
    apply_reflector (t4a_rrqr, bit-identical to that loop of primitives).  Algorithmic
    bytes per factorization: sum over steps s of norms 8(m-s)(n-s) + apply
    16(m-s)(n-s-1) + swap 32m + reflector 16(m-s).  Each step restores A from a
    pristine device copy outside the timed events; in the end-to-end leg the timed
    host-to-device copy of A is the restore."""

    name = "config5-rrqr-65536x256-f64"
    dtype = "f64"
    e2e_restores = True
    M, N, RANK = 65536, 256, 64

    def __init__(self, device=None):
        import numpy as np
        import torch
        import t4a_b200 as t4
        from t4a_b200 import abi
        self.t4, self.abi = t4, abi
        self.device = device
        m, n, k = self.M, self.N, self.RANK
        u = np.random.default_rng(10).standard_normal((m, k))
        v = np.random.default_rng(11).standard_normal((n, k))
        noise = np.random.default_rng(12).standard_normal((m, n))
        a = np.asfortranarray(u @ v.T + 1e-10 * noise)
        self.a_host = torch.from_numpy(a.ravel(order="K").copy())  # column-major buffer
        self.steps = n
        self.ops = [dict(tag="rrqr-f64-65536x256-256steps", i=0, launches=2 * n + 1, bytes=self.algorithmic_bytes())]
        if device is not None:
            self.host_in = [self.a_host.pin_memory()]
            self.pristine = self.a_host.to(device)
            self.work = torch.empty_like(self.pristine)
            self.dev_in = [self.work]
            self.perm = torch.empty(n, dtype=torch.int64, device=device)
            self.coeff = torch.empty(n, dtype=torch.float64, device=device)
            self.pivots = torch.empty(n, dtype=torch.int64, device=device)
            self.status = torch.zeros(1, dtype=torch.int64, device=device)
            self.layout = abi.layout([m, n])
            self.ws = torch.empty(t4.rrqr_workspace_bytes(abi.F64, self.layout), dtype=torch.uint8, device=device)
            self.dev_out = [self.pivots]
            self.host_out = [torch.empty(n, dtype=torch.int64).pin_memory()]

    def algorithmic_bytes(self):
        m, n = self.M, self.N
        return sum(8 * (m - s) * (n - s) + 16 * (m - s) * (n - s - 1) + 32 * m + 16 * (m - s) for s in range(n))

    def units(self):
        return sum(op["bytes"] for op in self.ops)

    def prepare(self, op):
        """Untimed: restore A before a factorization."""
        self.work.copy_(self.pristine)

    def run_op(self, op, stream_handle, dev_in=None, dev_out=None):
        t4, abi = self.t4, self.abi
        vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        t4.check(t4.lib().t4a_rrqr(stream_handle, abi.F64, vp(self.work), ctypes.byref(self.layout),
                                   self.M * self.N, self.steps, vp(self.perm), vp(self.coeff), vp(self.pivots),
                                   vp(self.status), vp(self.ws), self.ws.numel()), "rrqr")

    def host_arrays(self):
        return [self.a_host.numpy()], [None]

    def measure_epilogue(self, stream, stream_handle, args):
        """The reference bench's Q formation after the factorization
        (examples/bench_kernels.rs:2560-2590) through t4a_rrqr_form_q: identity_shifted,
        then apply_reflector for step = n-1 .. 0 over all n columns of Q [m, n].  Timed
        with CUDA events on the launching stream after 3 untimed runs, `args.steps`
        runs, L2 not flushed (Q alone is 134 MB).  Algorithmic bytes: the identity's
        writes 8 m n, then per step s the reflector's rows 8 (m - s) and Q's rows read
        and written 16 n (m - s)."""
        import torch
        t4, abi = self.t4, self.abi
        m, n = self.M, self.N
        q = torch.empty((n, m), dtype=torch.float64, device=self.device).t()
        wl_, ql, cl = abi.layout([m, n]), abi.layout([m, n], [1, m]), abi.layout([n])
        vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

        qstatus = torch.zeros(1, dtype=torch.int64, device=self.device)

        def form_q():
            t4.check(t4.lib().t4a_rrqr_form_q(stream_handle, abi.F64, vp(self.work), ctypes.byref(wl_), m * n,
                                              vp(self.coeff), ctypes.byref(cl), n, vp(q), ctypes.byref(ql), m * n,
                                              vp(qstatus)),
                     "rrqr_form_q")
        for _ in range(3):
            form_q()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            form_q()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        if int(qstatus.item()) != 0:
            raise RuntimeError(f"Q formation status {int(qstatus.item())}: a bounded wait ran out")
        nbytes = 8 * m * n + sum(8 * (m - s) + 16 * n * (m - s) for s in range(n))
        return {"what": "Q formation (identity_shifted + 256 reflector passes over Q's columns), t4a_rrqr_form_q",
                "ms": round(ms, 3), "bytes": nbytes, "gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
                "launches": n + 1, "status": int(qstatus.item())}

    def cpu_sample(self):
        return f"one full {self.name} factorization"

    def cpu_op(self, op, threads, srcs, dsts):
        import numpy as np
        oracle = _oracle()
        work = srcs[0].copy()
        perm = np.zeros(self.N, np.int64)
        coeff = np.zeros(self.N)
        oracle.lib().t4a_oracle_rrqr_f64(oracle.ptr(work), self.M, self.N, self.steps, oracle.lptr(perm),
                                         oracle.ptr(coeff), 1e-8, 0.0, threads)


WORKLOADS = {"movement": MovementWorkload, "reduce": ReduceWorkload, "gather": GatherScatterWorkload,
             "rrqr": RrqrWorkload}


def torch_int64():
    import torch
    return torch.int64


def flush_l2(buf):
    """Evict the working set from L2 by reading a buffer larger than L2 (clean lines, so
    nothing is written back during the next timed op)."""
    buf.sum(dtype=torch_int64())


def run_ours(args, rank, world, local_rank):
    import torch
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    wl = WORKLOADS[args.op](device)
    if args.only:
        keep = set(args.only.split(","))
        wl.ops = [op for op in wl.ops if op["tag"] in keep]
    t4 = wl.t4
    stream = torch.cuda.current_stream()
    sh = ctypes.c_void_p(stream.cuda_stream)
    flush = torch.ones(256 * MIB, dtype=torch.uint8, device=device)
    dist = world > 1

    def barrier():
        if dist:
            torch.distributed.barrier()

    prepare = getattr(wl, "prepare", None)
    for _ in range(args.warmup):
        for op in wl.ops:
            if prepare:
                prepare(op)
            wl.run_op(op, sh)
        flush_l2(flush)
    torch.cuda.synchronize()

    # Timed region: K steps, CUDA events around every op on the launching stream.
    events = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in wl.ops]
              for _ in range(args.steps)]
    sampler = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    with sampler:
        # Hold the stream with a bounded sleep kernel while the timed steps are enqueued,
        # so each event pair brackets GPU work only, not the host's launch latency.
        torch.cuda._sleep(int(2e8))
        for k in range(args.steps):
            for j, op in enumerate(wl.ops):
                if prepare:
                    prepare(op)
                flush_l2(flush)
                events[k][j][0].record(stream)
                wl.run_op(op, sh)
                events[k][j][1].record(stream)
        torch.cuda.synchronize()
    barrier()
    wall = time.perf_counter() - wall0
    per_op_ms = [[events[k][j][0].elapsed_time(events[k][j][1]) for k in range(args.steps)] for j in range(len(wl.ops))]
    kernel_ms = sum(sum(x) for x in per_op_ms)
    step_ms = kernel_ms / args.steps
    if dist:
        t = torch.tensor([kernel_ms], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        kernel_ms = t.item()
        step_ms = kernel_ms / args.steps
    value = wl.units() * world * args.steps / (kernel_ms / 1e3) / 1e9

    # End to end through the public API: pinned host inputs -> device -> op -> host.
    e2e_ms = None
    h2d = sum(h.numel() * h.element_size() for op in wl.ops for h, _ in wl.e2e_inputs(op))
    d2h = sum(h.numel() * h.element_size() for op in wl.ops for _, h in wl.e2e_outputs(op))
    # Three streams, as a caller pipelines host data through the library: host->device
    # copies on s_in, the ops on the launching stream, device->host copies on s_out, so
    # one op's result copy overlaps the next op's input copy (PCIe is full duplex).  A
    # copy into a device input waits for the last op that read that buffer; an op waits
    # for its input copies and for the last copy out of its output buffers.
    s_in = torch.cuda.Stream(device=device)
    s_out = torch.cuda.Stream(device=device)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    read_done, copied_out = {}, {}  # device buffer -> event: last op that read it / last copy out of it
    for _ in range(args.steps):
        for op in wl.ops:
            ins, outs = wl.e2e_inputs(op), wl.e2e_outputs(op)
            with torch.cuda.stream(s_in):
                for h, d in ins:
                    if d.data_ptr() in read_done:
                        s_in.wait_event(read_done[d.data_ptr()])
                    d.copy_(h, non_blocking=True)
                arrived = torch.cuda.Event()
                arrived.record(s_in)
            stream.wait_event(arrived)
            for d, _ in outs:
                if d.data_ptr() in copied_out:
                    stream.wait_event(copied_out[d.data_ptr()])
            if prepare and not getattr(wl, "e2e_restores", False):
                prepare(op)
            wl.run_op(op, sh)
            done = torch.cuda.Event()
            done.record(stream)
            for _, d in ins:
                read_done[d.data_ptr()] = done
            s_out.wait_event(done)
            with torch.cuda.stream(s_out):
                for d, h in outs:
                    h.copy_(d, non_blocking=True)
                out_done = torch.cuda.Event()
                out_done.record(s_out)
            for d, _ in outs:
                copied_out[d.data_ptr()] = out_done
    tail_in, tail_out = torch.cuda.Event(), torch.cuda.Event()
    tail_in.record(s_in)
    tail_out.record(s_out)
    stream.wait_event(tail_in)
    stream.wait_event(tail_out)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = t.item()
    e2e_value = wl.units() * world * args.steps / (e2e_ms / 1e3) / 1e9
    # A workload may time a follow-on stage of the path separately (RRQR: the Q
    # formation that follows the factorization in the reference bench).
    epilogue = wl.measure_epilogue(stream, sh, args) if hasattr(wl, "measure_epilogue") else None

    # Roofline of the dominant kernel (longest total time).
    peak, peak_kind = read_peaks()
    totals = [sum(x) for x in per_op_ms]
    dom = max(range(len(wl.ops)), key=lambda j: totals[j])
    dom_op = wl.ops[dom]
    dom_ms = totals[dom] / args.steps
    achieved = dom_op["bytes"] / (dom_ms / 1e3) / 1e9
    traffic = profile_traffic(dom_op["tag"])
    ops_detail = {wl.ops[j]["tag"]: {"bytes": wl.ops[j]["bytes"], "us": round(1e3 * totals[j] / args.steps, 2),
                                     "gbs": round(wl.ops[j]["bytes"] / (totals[j] / args.steps / 1e3) / 1e9, 1),
                                     "frac_of_measured": round(wl.ops[j]["bytes"] / (totals[j] / args.steps / 1e3)
                                                               / 1e9 / peak, 3)}
                  for j in range(len(wl.ops))}

    line = {
        "metric": "achieved HBM GB/s (% of B200 peak) per op at 1/2/4/8 GPUs vs CPU baseline",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": wl.dtype,
        "data": "synthetic (seeded normal(0,1), SplitMix64 Box-Muller)",
        "config": {"workload": wl.name, "ops": [op["tag"] for op in wl.ops],
                   "bytes_per_step_per_gpu": wl.units(), "l2": "flushed before every op (256 MiB read, untimed)",
                   "parallelism": f"replicas x{world}" if world > 1 else "1 gpu",
                   "timing": "CUDA events per op on the launching stream, max over ranks"},
        "roofline": {"bound": "hbm", "kernel": dom_op["tag"], "achieved": round(achieved, 1), "peak": peak,
                     "peak_kind": f"{peak_kind} hbm_gbs", "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": traffic},
        "ops": ops_detail,
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms / args.steps, 3)},
        "gpu_launches": sum(op.get("launches", 1) for op in wl.ops) * args.steps,
        "clocks": sampler.summary(),
        "wall_s_timed_region": round(wall, 3),
    }
    if epilogue is not None:
        line["epilogue"] = epilogue
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl, args)
    return line


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(wl, args, repeats=1):
    """The oracle port over every host core on the same workload (one full step)."""
    import numpy as np
    threads = host_threads()
    srcs, dsts = wl.host_arrays()
    t0 = time.perf_counter()
    n = 0
    while True:
        for op in wl.ops:
            wl.cpu_op(op, threads, srcs, dsts)
        n += 1
        if time.perf_counter() - t0 > 2.0 or n >= repeats:
            break
    dt = time.perf_counter() - t0
    return {"value": round(wl.cpu_units() * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} step(s) of {wl.cpu_sample()} ({wl.cpu_units() / MIB:.0f} MiB algorithmic), {dt:.2f} s"}


def run_reference(args, rank, world):
    """CPU implementation of the path on the host cores (see module docstring)."""
    import torch
    if rank != 0:
        return None
    wl = WORKLOADS[args.op](None)
    threads = host_threads()
    srcs, dsts = wl.host_arrays()
    for _ in range(max(0, min(args.warmup, 1))):
        for op in wl.ops:
            wl.cpu_op(op, threads, srcs, dsts)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for op in wl.ops:
            wl.cpu_op(op, threads, srcs, dsts)
    dt = time.perf_counter() - t0
    value = wl.cpu_units() * args.steps / dt / 1e9
    return {
        "impl": "reference",
        "metric": "achieved HBM GB/s (% of B200 peak) per op at 1/2/4/8 GPUs vs CPU baseline",
        "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * dt / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded normal(0,1))",
        "config": {"workload": wl.name, "ops": [op["tag"] for op in wl.ops], "bytes_per_step": wl.units()},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps of {wl.cpu_sample()} on the host cores"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--op", default="movement", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", default=None, help="comma-separated op tags of the workload to run (profiling)")
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
    try:
        if world > 1:
            import datetime
            torch.cuda.set_device(local_rank)
            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        try:
            line = run_ours(args, rank, world, local_rank)
        finally:
            if world > 1:
                torch.distributed.destroy_process_group()
    finally:
        sys.stdout.flush()
        os.dup2(saved_stdout, 1)
        os.close(saved_stdout)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
