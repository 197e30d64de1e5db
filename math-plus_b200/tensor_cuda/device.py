"""``createCudaDevice()`` / ``CudaDevice`` / ``DeviceArray``: the chainable device-array API.

A Python twin of tensor-cpu's ``ArrayDevice`` / ``DeviceArray`` (packages/tensor-cpu/src/device-array.ts:65-540)
with the CUDA device facade shaped like ``createWebGpuDevice`` (packages/tensor-webgpu/src/facade.ts:52-199),
for the ops on the GEMM / attention path. The reference's rules hold:

* no implicit transfers: data enters through ``fromTensor`` / ``fromHost`` and leaves through
  ``toTensor`` / ``toHost``, both async; validation errors raise before any coroutine is awaited;
* no implicit dtype promotion: binary ops need matching dtypes, ``cast`` is the only way across;
* lazy inside, eager-observable: values appear at ``eval()`` / ``toTensor()`` / ``toHost()``;
* arrays belong to one device; ``dispose`` is idempotent; ``scope`` frees what it does not return.
"""
from __future__ import annotations

import numpy as np

from . import _ffi as F
from .backend import FLOAT, CudaBackend, CudaTensor, HostTensor, host
from .runtime import Device

_LABEL = "tensor-cuda"


def _dtype_of(arr: np.ndarray) -> str:
    if arr.dtype == np.float32:
        return "f32"
    if arr.dtype == np.float16:
        return "f16"
    if arr.dtype == np.int32:
        return "i32"
    if arr.dtype == np.bool_:
        return "bool"
    raise TypeError(f"{_LABEL} fromTensor: unsupported dtype {arr.dtype}; cast to float32 / float16 / int32 / "
                    "bool explicitly first (bf16 uploads go through fromHost with uint16 bits)")


class ArrayDevice:
    """A device: a backend plus the bookkeeping the chainable arrays need."""

    def __init__(self, backend: CudaBackend):
        self.backend = backend
        self.name = backend.name
        self._scopes: list[set] = []

    def supports(self, dtype: str) -> bool:
        return self.backend.supports(dtype)

    # ---- transfers ---------------------------------------------------------------------------
    def fromTensor(self, t: np.ndarray):
        """Explicit, async upload of a C-contiguous host array (one copy). Non-contiguous input or
        an unsupported dtype raises here, before the coroutine runs (host.ts:58-97)."""
        if not isinstance(t, np.ndarray):
            raise TypeError(f"{_LABEL} fromTensor: expected a numpy array, got {type(t).__name__}")
        if not t.flags.c_contiguous:
            raise ValueError(f"{_LABEL} fromTensor: the tensor must be C-contiguous (call .copy() first)")
        return self.fromHost(host(_dtype_of(t), t.shape, t))

    def fromHost(self, h: HostTensor):
        """Explicit, async upload of a HostTensor. An unsupported dtype raises here."""
        self._check_dtype(h.dtype, "fromHost")

        async def go():
            return self.wrap(await self.backend.fromHost(h))

        return go()

    def wrap(self, h: CudaTensor) -> "DeviceArray":
        a = DeviceArray(self, h)
        if self._scopes:
            self._scopes[-1].add(a)
        return a

    # ---- graph control & lifetime --------------------------------------------------------------
    def eval(self, *arrays: "DeviceArray") -> None:
        hs = [self._own(a, "eval") for a in arrays]
        self.backend.flush(*hs)

    def scope(self, fn):
        created: set = set()
        self._scopes.append(created)
        holder = {}

        def inner():
            holder["r"] = fn()
            # the backend scope keeps the handles of the arrays returned (directly or one level deep)
            return [a._h for a in _arrays_of(holder["r"]) if a._h is not None]

        try:
            self.backend.scope(inner)
            result = holder["r"]
        except BaseException:
            self._scopes.pop()
            for a in created:
                a._mark_disposed()
            raise
        self._scopes.pop()
        kept = set(_arrays_of(result))
        for a in created:
            if a not in kept:
                a._mark_disposed()
        if self._scopes:
            for a in kept:
                if a in created:
                    self._scopes[-1].add(a)
        return result

    def destroy(self) -> None:
        self.backend.destroy()

    def _own(self, x, op: str) -> CudaTensor:
        if not isinstance(x, DeviceArray):
            raise TypeError(f"{_LABEL} {op}: expected a DeviceArray, got {type(x).__name__} — upload explicitly "
                            "with device.fromTensor() (no implicit transfers)")
        if x.device is not self:
            raise ValueError(f"{_LABEL} {op}: array belongs to a different device (no implicit transfers)")
        return x._handle(op)

    def _check_dtype(self, dtype: str, op: str) -> None:
        if not self.backend.supports(dtype):
            raise TypeError(f"{_LABEL} {op}: this {self.name} device does not support {dtype}; cast to a supported "
                            "dtype (e.g. \"f32\") explicitly first")


def _arrays_of(v):
    if isinstance(v, DeviceArray):
        return [v]
    if isinstance(v, (list, tuple)):
        return [x for x in v if isinstance(x, DeviceArray)]
    if isinstance(v, dict):
        return [x for x in v.values() if isinstance(x, DeviceArray)]
    return []


class DeviceArray:
    """A chainable array on an ArrayDevice; every op returns a new array of the same device."""

    def __init__(self, device: ArrayDevice, h: CudaTensor):
        self.device = device
        self._h = h

    # ---- properties ----------------------------------------------------------------------------
    @property
    def shape(self) -> tuple:
        return self._handle("shape").shape

    @property
    def dtype(self) -> str:
        return self._handle("dtype").dtype

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @property
    def size(self) -> int:
        return self._handle("size").size

    @property
    def disposed(self) -> bool:
        return self._h is None or self._h.disposed

    @property
    def handle(self) -> CudaTensor:
        """The backend handle, for ``device.backend.*`` ops this API does not wrap."""
        return self._handle("handle")

    def _handle(self, op: str) -> CudaTensor:
        if self._h is None or self._h.disposed:
            raise RuntimeError(f"{_LABEL} {op}: array used after dispose")
        return self._h

    def _mark_disposed(self) -> None:
        if self._h is not None:
            self._h._release()
        self._h = None

    # ---- transfers & lifetime ------------------------------------------------------------------
    async def toHost(self) -> HostTensor:
        return await self.device.backend.read(self._handle("toHost"))

    async def toTensor(self) -> np.ndarray:
        """Explicit download as a numpy array (bf16 widened exactly to float32: numpy has no bf16)."""
        h = await self.toHost()
        data = h.data
        if h.dtype == "bf16":
            data = (data.astype(np.uint32) << 16).view(np.float32)
        elif h.dtype == "bool":
            data = data.astype(np.bool_)
        return data.reshape(h.shape)

    def eval(self) -> "DeviceArray":
        self.device.eval(self)
        return self

    def dispose(self) -> None:
        if self._h is not None:
            self.device.backend.dispose(self._h)
        self._h = None

    # ---- ops --------------------------------------------------------------------------------
    def _wrap(self, h: CudaTensor) -> "DeviceArray":
        return self.device.wrap(h)

    def _float(self, op: str) -> CudaTensor:
        x = self._handle(op)
        if x.dtype not in FLOAT:
            raise TypeError(f"{_LABEL} {op}: needs a float array, got {x.dtype}")
        return x

    def add(self, other: "DeviceArray") -> "DeviceArray":
        x = self._float("add")
        y = self.device._own(other, "add")
        if x.dtype != y.dtype:
            raise TypeError(f"{_LABEL} add: dtype mismatch {x.dtype} vs {y.dtype} (no implicit promotion; cast() first)")
        return self._wrap(self.device.backend.add(x, y))

    def gelu(self) -> "DeviceArray":
        return self._wrap(self.device.backend.gelu(self._float("gelu")))

    def softmax(self, axis: int = -1) -> "DeviceArray":
        return self._wrap(self.device.backend.softmax(self._float("softmax"), axis))

    def matmul(self, other: "DeviceArray") -> "DeviceArray":
        x = self._float("matmul")
        y = self.device._own(other, "matmul")
        if x.dtype != y.dtype:
            raise TypeError(f"{_LABEL} matmul: dtype mismatch {x.dtype} vs {y.dtype} (no implicit promotion; cast() first)")
        return self._wrap(self.device.backend.matmul(x, y))

    def layerNorm(self, weight: "DeviceArray | None" = None, bias: "DeviceArray | None" = None,
                  eps: float = 1e-5) -> "DeviceArray":
        x = self._float("layerNorm")
        w = self.device._own(weight, "layerNorm") if weight is not None else None
        b = self.device._own(bias, "layerNorm") if bias is not None else None
        return self._wrap(self.device.backend.layerNorm(x, w, b, eps))

    def cast(self, dtype: str) -> "DeviceArray":
        self.device._check_dtype(dtype, "cast")
        return self._wrap(self.device.backend.cast(self._handle("cast"), dtype))

    def reshape(self, shape) -> "DeviceArray":
        return self._wrap(self.device.backend.reshape(self._handle("reshape"), shape))

    def transpose(self, axes=None) -> "DeviceArray":
        """Permute axes (default: reverse them), like numpy.transpose."""
        return self._wrap(self.device.backend.transpose(self._handle("transpose"), axes))


class CudaDevice(ArrayDevice):
    """The CUDA device facade (the shape of WebGpuDevice, packages/tensor-webgpu/src/facade.ts:93-199)."""

    def __init__(self, device: Device):
        super().__init__(CudaBackend(device))
        self.device = device
        self.info = dict(device.info)

    async def toTensor(self, a: DeviceArray) -> np.ndarray:
        return await a.toTensor()

    async def toHost(self, a: DeviceArray) -> HostTensor:
        return await a.toHost()

    def dispose(self, a: DeviceArray) -> None:
        a.dispose()

    def sync(self) -> None:
        """Waits for all queued work (facade.ts:175); raises MpcError on a kernel-side error."""
        self.device.sync()

    # synchronous conveniences for Python callers
    def from_numpy(self, arr: np.ndarray, dtype: str | None = None) -> DeviceArray:
        """Upload now (no coroutine): ``dtype="bf16"`` rounds float input to bfloat16 (or takes
        uint16 bits as they are)."""
        if dtype is None:
            h = host(_dtype_of(np.ascontiguousarray(arr)), np.shape(arr), np.ascontiguousarray(arr))
        else:
            h = host(dtype, np.shape(arr), arr)
        self._check_dtype(h.dtype, "fromHost")
        return self.wrap(self.backend.from_host_sync(h))

    def to_numpy(self, a: DeviceArray) -> np.ndarray:
        h = self.backend.read_sync(self._own(a, "toHost"))
        data = h.data
        if h.dtype == "bf16":
            data = (data.astype(np.uint32) << 16).view(np.float32)
        return data.reshape(h.shape)


def cuda_unavailable_reason(ordinal: int = 0) -> str | None:
    """Why ``createCudaDevice()`` would fail here, or None (webGpuUnavailableReason, facade.ts:67-73)."""
    try:
        F.load()
    except OSError as e:
        return str(e)
    try:
        import ctypes as C
        n = C.c_int()
        F.call("mpc_device_count", C.byref(n))
        if n.value <= ordinal:
            return f"no CUDA device {ordinal} (found {n.value})"
    except F.MpcError as e:
        return str(e)
    return None


def create_cuda_device(ordinal: int = 0, library_path: str | None = None) -> CudaDevice:
    """The device for ``ordinal`` (one backend per device, bridge.ts:8-12). Raises MpcError without
    a B200 — there is no CPU fallback."""
    return CudaDevice(Device.shared(ordinal, library_path))


async def createCudaDevice(opts: dict | None = None) -> CudaDevice:
    opts = opts or {}
    return create_cuda_device(opts.get("ordinal", 0), opts.get("libraryPath"))
