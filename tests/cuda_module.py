"""Launch `extern "C" __global__` kernels from a cubin by name through the CUDA
driver API, the way the reference's callers do (tests/gpu/mod.rs:105-113, :297-331).

Used by the GPU tests to run this library's exported symbols (its cubin modules)
and the reference's own kernels compiled from source (oracle/_ref/*.cubin).
"""
import ctypes

_CU = None


def cu():
    global _CU
    if _CU is None:
        _CU = ctypes.CDLL("libcuda.so.1")
        _CU.cuModuleLoadData.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]
        _CU.cuModuleGetFunction.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
        _CU.cuLaunchKernel.argtypes = [ctypes.c_void_p] + [ctypes.c_uint] * 6 + [ctypes.c_uint, ctypes.c_void_p,
                                                                                   ctypes.c_void_p, ctypes.c_void_p]
        _CU.cuFuncSetAttribute.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        _CU.cuModuleUnload.argtypes = [ctypes.c_void_p]
    return _CU


class Module:
    """A loaded cubin in the current (torch primary) context."""

    def __init__(self, path):
        import torch
        torch.cuda.init()
        torch.zeros(1, device="cuda")  # make the primary context current
        with open(path, "rb") as fh:
            self._image = fh.read()
        self.handle = ctypes.c_void_p()
        rc = cu().cuModuleLoadData(ctypes.byref(self.handle), self._image)
        if rc != 0:
            raise RuntimeError(f"cuModuleLoadData({path}) failed: {rc}")
        self._functions = {}

    def function(self, name):
        if name not in self._functions:
            fn = ctypes.c_void_p()
            rc = cu().cuModuleGetFunction(ctypes.byref(fn), self.handle, name.encode())
            if rc != 0:
                raise RuntimeError(f"cuModuleGetFunction({name}) failed: {rc}")
            self._functions[name] = fn
        return self._functions[name]

    def launch(self, name, grid, block, shared, args, stream=None):
        """`args`: ctypes objects in parameter order (by-value structs included)."""
        import torch
        fn = self.function(name)
        if shared > 48 * 1024:
            cu().cuFuncSetAttribute(fn, 8, shared)  # CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES
        params = (ctypes.c_void_p * len(args))(*[ctypes.cast(ctypes.pointer(a), ctypes.c_void_p) for a in args])
        s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        g = list(grid) + [1] * (3 - len(grid))
        b = list(block) + [1] * (3 - len(block))
        rc = cu().cuLaunchKernel(fn, g[0], g[1], g[2], b[0], b[1], b[2], shared, ctypes.c_void_p(s), params, None)
        if rc != 0:
            raise RuntimeError(f"cuLaunchKernel({name}) failed: {rc}")
