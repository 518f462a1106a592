"""Build libt4a_b200.so and the kernel modules for sm_100a.

    python t4a-cuda-kernels_b200/build.py [--jobs N] [--force]

Objects go to <repo>/_build/; the library and the modules to
t4a-cuda-kernels_b200/t4a_b200/lib/.  The modules are one image per kernel family
(reduce, movement, gather_scatter, rrqr, linalg_aux), like the reference's per-file modules,
exporting the reference's `extern "C" __global__` symbols, each in three forms: .cubin
(sm_100a), .fatbin (sm_100a plus compute_100a PTX) and .ptx (compute_100a, for JIT).  A source is rebuilt when it, or any header
of csrc/ or include/, is newer than its object.
"""
import argparse
import concurrent.futures
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIBDIR = os.path.join(HERE, "t4a_b200", "lib")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = os.environ.get("NVCC", "nvcc")
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include")]
# Translation units that export the reference's __global__ symbols (the module).
MODULE_TUS = ["reduce_abi.cu", "movement_abi.cu", "gather_scatter_abi.cu", "rrqr_abi.cu", "linalg_aux_abi.cu"]


def headers(src=None):
    """Headers `src` includes, transitively (quoted includes only); all when src is None."""
    if src is None:
        return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
            glob.glob(os.path.join(ROOT, "include", "**", "*.h"), recursive=True)
    seen, todo = set(), [src]
    while todo:
        path = todo.pop()
        try:
            text = open(path).read()
        except OSError:
            continue
        for line in text.splitlines():
            line = line.strip()
            if line.startswith("#include \""):
                dep = os.path.normpath(os.path.join(os.path.dirname(path), line.split('"')[1]))
                if dep not in seen:
                    seen.add(dep)
                    todo.append(dep)
    return sorted(seen)


def stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
        raise SystemExit(f"build failed: {os.path.basename(cmd[-1])}")
    return proc


def compile_one(src, force):
    name = os.path.basename(src)
    obj = os.path.join(BUILD, name + ".o")
    if force or stale(obj, [src] + headers(src)):
        run([NVCC] + COMMON + ARCH + ["-c", src, "-o", obj])
    return obj


def module_one(src, force):
    """One kernel family as three module images with the same exported symbols:
    <family>.cubin (sm_100a SASS), <family>.fatbin (sm_100a SASS plus compute_100a PTX,
    which the driver JIT-compiles where the SASS does not run) and <family>.ptx
    (compute_100a PTX alone, for callers that load text and JIT it themselves)."""
    name = os.path.basename(src)
    stem = os.path.join(LIBDIR, name.replace("_abi.cu", ""))
    base = [NVCC, "-std=c++17", "-O3", "-lineinfo", "-I", os.path.join(ROOT, "include")]
    deps = [src] + headers(src)
    if force or stale(stem + ".cubin", deps):
        run(base + ["-cubin", "-gencode", "arch=compute_100a,code=sm_100a", src, "-o", stem + ".cubin"])
    if force or stale(stem + ".fatbin", deps):
        run(base + ["-fatbin", "-gencode", "arch=compute_100a,code=[sm_100a,compute_100a]", src, "-o",
                    stem + ".fatbin"])
    if force or stale(stem + ".ptx", deps):
        run(base + ["-ptx", "-arch=compute_100a", src, "-o", stem + ".ptx"])
    return stem + ".cubin"


# A test build of the kernels that stage data with bulk copies (RRQR, scatter_add), with
# every staged-data wait limited to zero rounds: the GPU tests drive it to check that a
# wait that runs out sets the status word and leaves nothing in flight.
WAITZERO_TUS = ["rrqr_fast.cu", "gather_scatter_fast.cu", "runtime.cu"]


def build_waitzero(force=False):
    out_dir = os.path.join(BUILD, "waitzero")
    os.makedirs(out_dir, exist_ok=True)
    objs = []
    for name in WAITZERO_TUS:
        src = os.path.join(CSRC, name)
        obj = os.path.join(out_dir, name + ".o")
        if force or stale(obj, [src] + headers(src)):
            run([NVCC] + COMMON + ARCH + ["-DT4A_STAGE_WAIT_LIMIT=0", "-c", src, "-o", obj])
        objs.append(obj)
    lib = os.path.join(LIBDIR, "libt4a_waitzero.so")
    if force or stale(lib, objs):
        run([NVCC, "-shared"] + ARCH + ["-o", lib] + objs + ["-lcudart"])
    return lib


def build(jobs=8, force=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    module_sources = [os.path.join(CSRC, n) for n in MODULE_TUS if os.path.exists(os.path.join(CSRC, n))]
    lib_sources = [s for s in sources if os.path.basename(s) not in MODULE_TUS]
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as pool:
        obj_futures = [pool.submit(compile_one, s, force) for s in lib_sources]
        cubin_futures = [pool.submit(module_one, s, force) for s in module_sources]
        objs = [f.result() for f in obj_futures]
        [f.result() for f in cubin_futures]
    lib = os.path.join(LIBDIR, "libt4a_b200.so")
    if force or stale(lib, objs):
        run([NVCC, "-shared"] + ARCH + ["-o", lib] + objs + ["-lcudart", "-ldl"])
    build_waitzero(force)
    return lib


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(args.jobs, args.force))


if __name__ == "__main__":
    main()
