"""Device runtime over libmathplus_cuda.so: device handle, memory, copies, streams, events.

The C library owns the device allocator, streams and events; this module only keeps handles
and turns status codes into exceptions. No torch, no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import threading

import numpy as np

from . import _ffi as F


class DeviceBuffer:
    """A block of device memory from the library's caching allocator, reference-counted: views
    and pending work retain it; it returns to the allocator when the last holder releases it
    (or on garbage collection)."""

    __slots__ = ("device", "ptr", "nbytes", "refs", "__weakref__")

    def __init__(self, device: "Device", nbytes: int):
        self.device = device
        self.nbytes = int(nbytes)
        self.refs = 1
        p = C.c_void_p()
        F.call("mpc_alloc", device.handle, max(self.nbytes, 1), C.byref(p))
        self.ptr = p.value

    def retain(self) -> "DeviceBuffer":
        self.refs += 1
        return self

    def release(self) -> None:
        self.refs -= 1
        if self.refs <= 0:
            self.free()

    def free(self) -> None:
        if self.ptr is not None and self.device.handle is not None:
            F.load().mpc_free(self.device.handle, C.c_void_p(self.ptr))
        self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Device:
    """One CUDA device (``mpc_device_create``); one per ordinal and process is the intended use."""

    _lock = threading.Lock()
    _open: dict[int, "Device"] = {}

    def __init__(self, ordinal: int = 0, library_path: str | None = None):
        F.load(library_path)
        h = C.c_void_p()
        F.call("mpc_device_create", ordinal, 0, C.byref(h))
        self.handle = h.value
        self.ordinal = ordinal
        info = F.DeviceInfo()
        F.call("mpc_device_info", self.handle, C.byref(info))
        self.info = {
            "name": info.name.decode(), "ordinal": info.ordinal, "cc": (info.cc_major, info.cc_minor),
            "sm_count": info.sm_count, "total_bytes": info.total_bytes,
            "runtime_version": info.runtime_version, "driver_version": info.driver_version,
        }
        s = C.c_void_p()
        F.call("mpc_device_stream", self.handle, C.byref(s))
        self.stream = s.value

    @classmethod
    def shared(cls, ordinal: int = 0, library_path: str | None = None) -> "Device":
        """The process-wide device for an ordinal (one runtime per device, like bridge.ts:8-12)."""
        with cls._lock:
            d = cls._open.get(ordinal)
            if d is None or d.handle is None:
                d = cls(ordinal, library_path)
                cls._open[ordinal] = d
            return d

    # ---- memory and copies -------------------------------------------------------------
    def alloc(self, nbytes: int) -> DeviceBuffer:
        return DeviceBuffer(self, nbytes)

    def upload(self, arr: np.ndarray, stream=None) -> DeviceBuffer:
        a = np.ascontiguousarray(arr)
        buf = DeviceBuffer(self, a.nbytes)
        if a.nbytes:
            F.call("mpc_memcpy_h2d_async", self.handle, C.c_void_p(buf.ptr), a.ctypes.data_as(C.c_void_p),
                   a.nbytes, C.c_void_p(stream))
            self.stream_sync(stream)  # the host array may be released after return
        return buf

    def copy_h2d(self, dst_ptr: int, arr: np.ndarray, stream=None) -> None:
        a = np.ascontiguousarray(arr)
        F.call("mpc_memcpy_h2d_async", self.handle, C.c_void_p(dst_ptr), a.ctypes.data_as(C.c_void_p), a.nbytes,
               C.c_void_p(stream))

    def download(self, ptr: int, nbytes: int, dtype, shape, stream=None) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        assert out.nbytes == nbytes
        if nbytes:
            F.call("mpc_memcpy_d2h_async", self.handle, out.ctypes.data_as(C.c_void_p), C.c_void_p(ptr), nbytes,
                   C.c_void_p(stream))
            self.stream_sync(stream)
        return out

    def copy_d2h_into(self, out: np.ndarray, ptr: int, stream=None) -> None:
        F.call("mpc_memcpy_d2h_async", self.handle, out.ctypes.data_as(C.c_void_p), C.c_void_p(ptr), out.nbytes,
               C.c_void_p(stream))

    def memset(self, ptr: int, value: int, nbytes: int, stream=None) -> None:
        F.call("mpc_memset_async", self.handle, C.c_void_p(ptr), value, nbytes, C.c_void_p(stream))

    def host_alloc(self, nbytes: int) -> int:
        p = C.c_void_p()
        F.call("mpc_host_alloc", self.handle, nbytes, C.byref(p))
        return p.value

    def host_free(self, ptr: int) -> None:
        F.call("mpc_host_free", self.handle, C.c_void_p(ptr))

    def pinned_array(self, shape, dtype) -> tuple[np.ndarray, int]:
        """A numpy array over pinned host memory (release with host_free(ptr))."""
        dt = np.dtype(dtype)
        n = int(np.prod(shape)) * dt.itemsize
        ptr = self.host_alloc(max(n, 1))
        buf = (C.c_uint8 * max(n, 1)).from_address(ptr)
        return np.frombuffer(buf, dtype=dt, count=int(np.prod(shape))).reshape(shape), ptr

    # ---- sync, streams, events ------------------------------------------------------------
    def sync(self) -> None:
        F.call("mpc_sync", self.handle)

    def stream_sync(self, stream=None) -> None:
        F.call("mpc_stream_sync", self.handle, C.c_void_p(stream))

    def event(self) -> int:
        e = C.c_void_p()
        F.call("mpc_event_create", self.handle, C.byref(e))
        return e.value

    def record(self, event: int, stream=None) -> None:
        F.call("mpc_event_record", self.handle, C.c_void_p(event), C.c_void_p(stream))

    def wait_event(self, stream, event: int) -> None:
        """Orders later work on ``stream`` after ``event``'s last recording."""
        F.call("mpc_stream_wait_event", self.handle, C.c_void_p(stream), C.c_void_p(event))

    def new_stream(self) -> int:
        s = C.c_void_p()
        F.call("mpc_stream_create", self.handle, C.byref(s))
        return s.value

    def destroy_stream(self, stream: int) -> None:
        F.call("mpc_stream_destroy", self.handle, C.c_void_p(stream))

    def elapsed_ms(self, start: int, stop: int) -> float:
        ms = C.c_float()
        F.call("mpc_event_elapsed_ms", self.handle, C.c_void_p(start), C.c_void_p(stop), C.byref(ms))
        return ms.value

    def destroy_event(self, e: int) -> None:
        F.call("mpc_event_destroy", self.handle, C.c_void_p(e))

    def launch_count(self) -> int:
        n = C.c_uint64()
        F.call("mpc_launch_count", self.handle, C.byref(n))
        return n.value

    def alloc_stats(self) -> tuple[int, int]:
        a, b = C.c_size_t(), C.c_size_t()
        F.call("mpc_alloc_stats", self.handle, C.byref(a), C.byref(b))
        return a.value, b.value

    def status(self) -> int:
        return F.load().mpc_device_status(self.handle)

    def destroy(self) -> None:
        if self.handle is not None:
            F.load().mpc_device_destroy(self.handle)
            self.handle = None
            with Device._lock:
                if Device._open.get(self.ordinal) is self:
                    del Device._open[self.ordinal]

    # ---- raw kernel entry points (pointers in, pointers out) ------------------------------
    def gemm(self, desc: F.GemmDesc, a: int, b: int, c: int, bias: int | None = None, stream=None) -> None:
        F.call("mpc_gemm", self.handle, C.byref(desc), C.c_void_p(a), C.c_void_p(b), C.c_void_p(c),
               C.c_void_p(bias), C.c_void_p(stream))

    def sdpa(self, desc: F.SdpaDesc, q: int, k: int, v: int, mask: int | None, o: int, lse: int | None = None,
             stream=None) -> None:
        F.call("mpc_sdpa", self.handle, C.byref(desc), C.c_void_p(q), C.c_void_p(k), C.c_void_p(v),
               C.c_void_p(mask), C.c_void_p(o), C.c_void_p(lse), C.c_void_p(stream))


def device_count() -> int:
    n = C.c_int()
    F.call("mpc_device_count", C.byref(n))
    return n.value


def gemm_desc(m: int, n: int, k: int, dtype_in: int, dtype_out: int, b_layout: int = F.B_KN, epilogue: int = 0,
              alpha: float = 1.0, batch_shape=(), a_batch_strides=(), b_batch_strides=()) -> F.GemmDesc:
    d = F.GemmDesc()
    d.m, d.n, d.k = m, n, k
    d.dtype_in, d.dtype_out, d.b_layout, d.epilogue, d.alpha = dtype_in, dtype_out, b_layout, epilogue, alpha
    d.batch_rank = len(batch_shape)
    for i, s in enumerate(batch_shape):
        d.batch_shape[i] = s
        d.a_batch_stride[i] = a_batch_strides[i]
        d.b_batch_stride[i] = b_batch_strides[i]
    return d


def sdpa_desc(b, h, hk, lq, lk, d, dv, dtype, causal=False, scale=None, mask_kind=F.MASK_NONE,
              mask_strides=(0, 0, 0, 0)) -> F.SdpaDesc:
    x = F.SdpaDesc()
    x.b, x.h, x.hk, x.lq, x.lk, x.d, x.dv = b, h, hk, lq, lk, d, dv
    x.dtype, x.causal = dtype, 1 if causal else 0
    x.scale = (1.0 / d ** 0.5) if scale is None else scale
    x.mask_kind = mask_kind
    for i in range(4):
        x.mask_strides[i] = mask_strides[i]
    return x
