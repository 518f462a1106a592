"""The reduction entry that allocates nothing (t4a_reduce_noalloc), on a GPU.

It serves callers that cannot give the library a device workspace (no device
allocator available to them, or one they must not call on their path, since a
cudaMalloc can synchronize the device).  Its partials live in a fixed array of the
library's module.  Each case compares two calls in a row of the no-alloc entry with
the existing entry t4a_reduce (caller-provided workspace), bit for bit, which is this
suite's tolerance for reductions; a reduction whose partials exceed the array is
refused before anything runs.  This file is collected last so that a run stopping at
its first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

import t4a_b200 as t4
from t4a_b200 import abi

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20


def noalloc():
    fn = t4.lib().t4a_reduce_noalloc
    P, I, U, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint, ctypes.c_longlong
    LP = ctypes.POINTER(abi.Layout)
    fn.argtypes = [P, I, I, P, LP, LL, P, LP, LL, U, U]
    fn.restype = I
    return fn


CASES = [
    ((256, 1024, 64), 1, abi.SUM, np.float64),       # BASELINE config 1 (4 splits)
    ((256, 1024, 64), 1, abi.MAX, np.float64),
    ((512, 1024, 32), 0, abi.SUM_SQUARES, np.float32),
    ((96, 8192), 1, abi.SUM, np.complex128),
    ((3, 1_000_003), 1, abi.PROD, np.float32),
]


@pytest.mark.parametrize("shape,axis,op,np_dtype", CASES)
def test_noalloc_matches_workspace_entry_twice(cuda, shape, axis, op, np_dtype):
    import torch
    rng = np.random.default_rng(len(shape) * 1000 + axis)
    x = rng.uniform(0.5, 1.5, size=shape) if op == abi.PROD else rng.standard_normal(shape)
    if np.issubdtype(np_dtype, np.complexfloating):
        x = x + 1j * rng.standard_normal(shape)
    x = torch.from_numpy(np.ascontiguousarray(x.astype(np_dtype))).cuda()
    want = t4.reduce(x, axis, op)  # t4a_reduce with a torch-allocated workspace
    dtype = t4.torch_dtype_tag(x)
    in_l = t4.tensor_layout(x)
    oshape = list(shape)
    oshape[axis] = 1
    assert t4.reduce_workspace_bytes(dtype, op, abi.numpy_layout(oshape), int(np.prod(oshape)), in_l,
                                     x.numel(), len(shape) - 1 - axis) > 0, "case must need partials"
    fn = noalloc()
    for _ in range(2):
        got = torch.full(oshape, float("nan"), dtype=x.dtype, device=x.device)
        rc = fn(t4.stream_handle(), dtype, op, ctypes.c_void_p(got.data_ptr()), ctypes.byref(t4.tensor_layout(got)),
                got.numel(), ctypes.c_void_p(x.data_ptr()), ctypes.byref(in_l), x.numel(), len(shape) - 1 - axis, 32)
        assert rc == 0, t4.status_string(rc)
        torch.cuda.synchronize()
        a = want.cpu().numpy().view(np.uint8)
        b = got.cpu().numpy().view(np.uint8)
        assert np.array_equal(a, b)


def test_noalloc_refuses_partials_beyond_its_array(cuda):
    import torch
    # A broadcast F64 input (strides 0) of 16384 x 65536: 64 splits x 65536 outputs x 8 B
    # = 32 MiB of partials, over the 16 MiB array; refused before any launch.
    buf = torch.zeros(1, dtype=torch.float64, device="cuda")
    out = torch.zeros(65536, dtype=torch.float64, device="cuda")
    in_l = abi.layout([16384, 65536], [0, 0])
    out_l = abi.layout([1, 65536])
    rc = noalloc()(t4.stream_handle(), abi.F64, abi.SUM, ctypes.c_void_p(out.data_ptr()), ctypes.byref(out_l), 65536,
                   ctypes.c_void_p(buf.data_ptr()), ctypes.byref(in_l), 1, 0, 32)
    assert rc == 65  # T4A_ERR_WORKSPACE
