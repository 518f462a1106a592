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

`--op` selects another BASELINE config as the workload (reduce, gather, scatter,
rrqr) for the secondary lines; the driver's runs use the default.

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

def splitmix_normal(seed, count, dtype):
    """Seeded normal(0,1) values (Box-Muller over a counter-based SplitMix64 stream)."""
    import numpy as np
    with np.errstate(over="ignore"):
        k = np.arange(1, 2 * count + 1, dtype=np.uint64)
        z = np.uint64(seed) + k * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u = ((z >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / (1 << 53))
    u1, u2 = u[0::2], u[1::2]
    return (np.sqrt(-2.0 * np.log(u1)) * np.cos(2 * np.pi * u2)).astype(dtype)


class MovementWorkload:
    name = "config2-permutation-movement"
    dtype = "f32,c64"

    def __init__(self, device=None):
        import numpy as np
        import torch
        import t4a_b200 as t4
        from t4a_b200 import abi
        self.t4, self.abi = t4, abi
        self.device = device
        a = splitmix_normal(2, 64 ** 4, np.float32)
        re = splitmix_normal(3, 16 ** 6, np.float64)
        im = splitmix_normal(3 + 1000, 16 ** 6, np.float64)
        b = np.empty(16 ** 6, dtype=np.complex128)
        b.real, b.imag = re, im
        c = splitmix_normal(4, 64 ** 4, np.float32)
        pin = device is not None
        host = [torch.from_numpy(a), torch.from_numpy(b.view(np.float64)), torch.from_numpy(c)]
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

    def cpu_op(self, op, threads, host_src, host_dst):
        oracle = _oracle()
        rc = oracle.lib().t4a_oracle_strided_to_strided(op["dtype"], oracle.ptr(host_dst), oracle.ptr(host_src),
                                                        ctypes.byref(op["src_l"]), ctypes.byref(op["dst_l"]), threads)
        assert rc == 0

    def host_arrays(self):
        return [h.numpy() for h in self.host_in], [h.numpy() for h in self.host_out]



WORKLOADS = {"movement": MovementWorkload}


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

    for _ in range(args.warmup):
        for op in wl.ops:
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
    h2d = sum(wl.host_in[op["i"]].numel() * wl.host_in[op["i"]].element_size() for op in wl.ops)
    d2h = sum(wl.host_out[op["i"]].numel() * wl.host_out[op["i"]].element_size() for op in wl.ops)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        for op in wl.ops:
            i = op["i"]
            wl.dev_in[i].copy_(wl.host_in[i], non_blocking=True)
            wl.run_op(op, sh)
            wl.host_out[i].copy_(wl.dev_out[i], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = t.item()
    e2e_value = wl.units() * world * args.steps / (e2e_ms / 1e3) / 1e9

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
        "gpu_launches": len(wl.ops) * args.steps,
        "clocks": sampler.summary(),
        "wall_s_timed_region": round(wall, 3),
    }
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
            wl.cpu_op(op, threads, srcs[op["i"]], dsts[op["i"]])
        n += 1
        if time.perf_counter() - t0 > 2.0 or n >= repeats:
            break
    dt = time.perf_counter() - t0
    return {"value": round(wl.units() * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} full step(s) of {wl.name} ({wl.units() / MIB:.0f} MiB algorithmic), {dt:.2f} s"}


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
            wl.cpu_op(op, threads, srcs[op["i"]], dsts[op["i"]])
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for op in wl.ops:
            wl.cpu_op(op, threads, srcs[op["i"]], dsts[op["i"]])
    dt = time.perf_counter() - t0
    value = wl.units() * args.steps / dt / 1e9
    return {
        "impl": "reference",
        "metric": "achieved HBM GB/s (% of B200 peak) per op at 1/2/4/8 GPUs vs CPU baseline",
        "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * dt / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded normal(0,1))",
        "config": {"workload": wl.name, "ops": [op["tag"] for op in wl.ops], "bytes_per_step": wl.units()},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} full steps of {wl.name} on the host cores"},
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
    if world > 1:
        import datetime
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        line = run_ours(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
