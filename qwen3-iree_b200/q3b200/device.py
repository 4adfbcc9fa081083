"""Device memory through the library's own plumbing (no PyTorch, no CUDA binding)."""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import call, lib


def device_count() -> int:
    n = ctypes.c_int(0)
    call("q3_device_count", ctypes.byref(n))
    return n.value


def set_device(d: int) -> None:
    call("q3_set_device", d)


def device_info(d: int = 0) -> dict:
    sms, ma, mi, mem = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
    call("q3_device_info", d, ctypes.byref(sms), ctypes.byref(ma), ctypes.byref(mi),
         ctypes.byref(mem))
    return {"sm_count": sms.value, "cc": (ma.value, mi.value), "total_mem": mem.value}


class DeviceArray:
    """A device allocation with a numpy dtype/shape view of its contents."""

    def __init__(self, shape, dtype, zero: bool = False):
        self.shape = tuple(int(s) for s in (shape if isinstance(shape, (tuple, list)) else (shape,)))
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        p = ctypes.c_void_p()
        call("q3_device_malloc", ctypes.byref(p), max(self.nbytes, 16))
        self.ptr = p.value
        if zero:
            self.zero()

    @classmethod
    def from_host(cls, a: np.ndarray, stream=None) -> "DeviceArray":
        a = np.ascontiguousarray(a)
        d = cls(a.shape, a.dtype)
        d.upload(a, stream)
        return d

    def upload(self, a: np.ndarray, stream=None) -> None:
        a = np.ascontiguousarray(a, dtype=self.dtype)
        assert a.nbytes == self.nbytes, (a.nbytes, self.nbytes)
        call("q3_memcpy_htod", self.ptr, a.ctypes.data, self.nbytes, stream)
        call("q3_stream_synchronize", stream)

    def download(self, stream=None) -> np.ndarray:
        out = np.empty(self.shape, dtype=self.dtype)
        call("q3_memcpy_dtoh", out.ctypes.data, self.ptr, self.nbytes, stream)
        call("q3_stream_synchronize", stream)
        return out

    def zero(self, stream=None) -> None:
        call("q3_memset", self.ptr, 0, self.nbytes, stream)
        call("q3_stream_synchronize", stream)

    def fill_bytes(self, value: int, stream=None) -> None:
        call("q3_memset", self.ptr, value, self.nbytes, stream)
        call("q3_stream_synchronize", stream)

    def at(self, byte_offset: int) -> int:
        return self.ptr + byte_offset

    def free(self) -> None:
        if self.ptr:
            lib().q3_device_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def synchronize(stream=None) -> None:
    call("q3_stream_synchronize", stream)


class Events:
    """CUDA-event timing on a stream (device time, not wall clock)."""

    def __init__(self):
        a, b = ctypes.c_void_p(), ctypes.c_void_p()
        call("q3_event_create", ctypes.byref(a))
        call("q3_event_create", ctypes.byref(b))
        self.start, self.end = a.value, b.value

    def record_start(self, stream=None):
        call("q3_event_record", self.start, stream)

    def record_end(self, stream=None):
        call("q3_event_record", self.end, stream)

    def elapsed_ms(self) -> float:
        call("q3_event_synchronize", self.end)
        ms = ctypes.c_float()
        call("q3_event_elapsed_ms", self.start, self.end, ctypes.byref(ms))
        return ms.value

    def __del__(self):
        try:
            lib().q3_event_destroy(self.start)
            lib().q3_event_destroy(self.end)
        except Exception:
            pass
