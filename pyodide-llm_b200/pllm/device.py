"""Device buffers over the C ABI's allocator and copies (include/pllm.h: pllm_alloc, pllm_h2d, pllm_d2h)."""
import ctypes

import numpy as np

from .lib import L, check

_ready = {}


def init(device=0):
    """Select the device (once per process and device)."""
    if device not in _ready:
        if L.pllm_init(device) != 0:
            check("pllm_init")
        _ready[device] = True


class Buffer:
    """nbytes of device memory; .ptr is the device address the kernels take."""

    def __init__(self, nbytes):
        self.nbytes = int(nbytes)
        self.ptr = L.pllm_alloc(max(self.nbytes, 1))
        if not self.ptr:
            check("pllm_alloc")
            raise MemoryError(f"pllm_alloc({nbytes}) failed")

    @classmethod
    def of(cls, array):
        a = np.ascontiguousarray(array)
        b = cls(a.nbytes)
        b.upload(a)
        return b

    def upload(self, array, offset=0):
        a = np.ascontiguousarray(array)
        assert offset + a.nbytes <= self.nbytes, "upload past the buffer"
        L.pllm_h2d(self.ptr + offset, a.ctypes.data, a.nbytes)
        check("pllm_h2d")
        return self

    def download(self, dtype, count=None, offset=0):
        dtype = np.dtype(dtype)
        count = (self.nbytes - offset) // dtype.itemsize if count is None else count
        out = np.empty(count, dtype)
        L.pllm_sync()
        L.pllm_d2h(out.ctypes.data, self.ptr + offset, out.nbytes)
        L.pllm_sync()
        check("pllm_d2h")
        return out

    def zero(self):
        L.pllm_memset(self.ptr, 0, self.nbytes)
        return self

    def free(self):
        if self.ptr:
            L.pllm_free(self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Pinned:
    """Pinned host memory viewed as a NumPy array (the end-to-end copies)."""

    def __init__(self, count, dtype):
        dtype = np.dtype(dtype)
        self.nbytes = count * dtype.itemsize
        self.ptr = L.pllm_alloc_host(max(self.nbytes, 1))
        if not self.ptr:
            check("pllm_alloc_host")
        self.array = np.ctypeslib.as_array(ctypes.cast(self.ptr, ctypes.POINTER(ctypes.c_byte * self.nbytes)).contents)
        self.array = np.frombuffer(self.array, dtype=dtype, count=count)

    def __del__(self):
        try:
            if self.ptr:
                L.pllm_free_host(self.ptr)
                self.ptr = 0
        except Exception:
            pass
