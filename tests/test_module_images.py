"""The kernel modules in their three forms: <family>.cubin (sm_100a SASS),
<family>.fatbin (sm_100a SASS plus compute_100a PTX) and <family>.ptx (compute_100a PTX,
JIT-compiled by the driver on load).  The reference's callers load a module by name and
look its `extern "C" __global__` entries up by name (reference tests/gpu/mod.rs:105-113);
each form must export every entry its family's source declares.  On the GPU the golden
split reductions run through the PTX form and match the fixture bit for bit.

The driver JIT-compiles a whole PTX module on load: on a B200 that took about 140 s each
for reduce.ptx and movement.ptx (many template instances) and under 16 s for the other
three.  The two large ones are JIT-loaded only with T4A_JIT_LARGE=1."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "t4a-cuda-kernels_b200", "csrc")
LIBDIR = os.path.join(ROOT, "t4a-cuda-kernels_b200", "t4a_b200", "lib")
FAMILIES = ["reduce", "movement", "gather_scatter", "rrqr", "linalg_aux"]
FORMS = ["cubin", "fatbin", "ptx"]
JIT_LARGE = os.environ.get("T4A_JIT_LARGE") == "1"
LARGE = {"reduce", "movement"}


def exported(family):
    with open(os.path.join(CSRC, family + "_abi.cu")) as fh:
        src = fh.read()
    return sorted(set(re.findall(
        r'extern\s+"C"\s+__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s+)?(t4a_cuda_\w+)\s*\(', src)))


@pytest.mark.parametrize("family", FAMILIES)
def test_every_family_is_built_in_every_form(family):
    assert exported(family), family
    for form in FORMS:
        path = os.path.join(LIBDIR, f"{family}.{form}")
        assert os.path.isfile(path) and os.path.getsize(path) > 0, path


@pytest.mark.gpu
@pytest.mark.parametrize("form", ["fatbin", "ptx"])
@pytest.mark.parametrize("family", FAMILIES)
def test_module_form_exports_every_entry(cuda, family, form):
    from cuda_module import Module
    if form == "ptx" and family in LARGE and not JIT_LARGE:
        pytest.skip("JIT of this module takes minutes; set T4A_JIT_LARGE=1")
    module = Module(os.path.join(LIBDIR, f"{family}.{form}"))
    for name in exported(family):
        module.function(name)


@pytest.mark.gpu
def test_golden_split_reductions_through_the_ptx_module(cuda):
    if not JIT_LARGE:
        pytest.skip("JIT of reduce.ptx takes minutes; set T4A_JIT_LARGE=1")
    import reduce_inputs as ri
    from cuda_module import Module
    from reduce_cases import same_bits_or_nan
    from test_reduce_gpu import FIXTURE, run_case
    module = Module(os.path.join(LIBDIR, "reduce.ptx"))
    bad, exact = [], 0
    for case in ri.cases():
        key = "|".join([case[0], f"w{case[1]}", case[2], case[3], case[4]])
        _, _, _, finals, variant = FIXTURE[key]
        got, _, ftype = run_case("module", case, module)
        if got.hex() == finals:
            exact += 1
        elif not same_bits_or_nan(finals, got, ftype, variant):
            bad.append(key)
    assert not bad, bad[:5]
    assert exact > 0


@pytest.mark.gpu
def test_column_norms_through_the_ptx_module_match_the_cubin(cuda):
    """t4a_cuda_column_norms from rrqr.ptx (JIT) and from rrqr.cubin with the reference's
    geometry (one 32-lane block per column) and the same arguments: the same bits."""
    import ctypes
    import numpy as np
    import torch
    from cuda_module import Module
    from t4a_b200 import abi
    m, n = 3000, 37
    a = torch.from_numpy(np.random.default_rng(9).standard_normal((n, m))).cuda()  # column-major [m, n]
    wl, nl = abi.layout([m, n], [1, m]), abi.layout([n])
    outs = []
    for form in ("cubin", "ptx"):
        norms = torch.full((n,), -7.0, dtype=torch.float64, device="cuda")
        Module(os.path.join(LIBDIR, f"rrqr.{form}")).launch(
            "t4a_cuda_column_norms", (n,), (32,), 0,
            [ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(norms.data_ptr()), ctypes.c_int(abi.F64), wl, nl,
             ctypes.c_longlong(0)])
        torch.cuda.synchronize()
        outs.append(norms.cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint64), outs[1].view(np.uint64))
    want = np.linalg.norm(a.cpu().numpy(), axis=1)
    assert np.allclose(outs[0], want, rtol=1e-13)
