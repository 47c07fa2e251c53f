"""Minimal CUDA driver-API access through ctypes, used by the GPU tests to
load this package's module images FROM FILE and launch the drop-in kernels
with the reference hosts' own hard-coded geometry -- exactly what
gpu_workload.c / qwen_engine.c / gpt2_engine.c do with cuModuleLoadData,
cuModuleGetFunction and cuLaunchKernel (void** parameter arrays)."""
import ctypes

_cuda = None


def cuda():
    global _cuda
    if _cuda is None:
        _cuda = ctypes.CDLL("libcuda.so.1")
    return _cuda


def check(rc, what):
    if rc != 0:
        s = ctypes.c_char_p()
        cuda().cuGetErrorString(rc, ctypes.byref(s))
        raise RuntimeError(f"{what} failed: {rc} {s.value.decode() if s.value else ''}")


class Module:
    """A module image loaded into the current context (torch's primary one)."""

    def __init__(self, path):
        with open(path, "rb") as f:
            self._img = ctypes.create_string_buffer(f.read())
        self.mod = ctypes.c_void_p()
        check(cuda().cuModuleLoadData(ctypes.byref(self.mod), self._img), f"cuModuleLoadData({path})")
        self._fns = {}

    def has(self, name):
        f = ctypes.c_void_p()
        return cuda().cuModuleGetFunction(ctypes.byref(f), self.mod, name.encode()) == 0

    def fn(self, name):
        if name not in self._fns:
            f = ctypes.c_void_p()
            check(cuda().cuModuleGetFunction(ctypes.byref(f), self.mod, name.encode()), f"cuModuleGetFunction({name})")
            self._fns[name] = f
        return self._fns[name]

    def launch(self, name, grid, block, *args, smem=0, stream=None):
        """args: ints are passed as int32, floats as float32, tensors (or
        ('ptr', int)) as 64-bit device pointers."""
        vals = []
        for a in args:
            if hasattr(a, "data_ptr"):
                vals.append(ctypes.c_uint64(a.data_ptr()))
            elif isinstance(a, tuple) and a[0] == "ptr":
                vals.append(ctypes.c_uint64(a[1]))
            elif isinstance(a, float):
                vals.append(ctypes.c_float(a))
            elif isinstance(a, int):
                vals.append(ctypes.c_int(a))
            elif a is None:
                vals.append(ctypes.c_uint64(0))
            else:
                raise TypeError(type(a))
        arr = (ctypes.c_void_p * len(vals))(*[ctypes.cast(ctypes.pointer(v), ctypes.c_void_p) for v in vals])
        g = tuple(grid) + (1,) * (3 - len(grid))
        b = tuple(block) + (1,) * (3 - len(block))
        check(cuda().cuLaunchKernel(self.fn(name), ctypes.c_uint(g[0]), ctypes.c_uint(g[1]), ctypes.c_uint(g[2]),
                                    ctypes.c_uint(b[0]), ctypes.c_uint(b[1]), ctypes.c_uint(b[2]),
                                    ctypes.c_uint(smem), ctypes.c_void_p(stream), arr, None),
              f"cuLaunchKernel({name})")
