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

    def where(self, cond: "DeviceArray", a: "DeviceArray", b: "DeviceArray") -> "DeviceArray":
        """cond ? a : b, elementwise with broadcasting (device-array.ts:154-162)."""
        c = self._own(cond, "where")
        x, y = self._own(a, "where"), self._own(b, "where")
        if c.dtype != "bool":
            raise TypeError(f"{_LABEL} where: the condition must be bool, got {c.dtype}")
        if x.dtype != y.dtype:
            raise TypeError(f"{_LABEL} where: dtype mismatch {x.dtype} vs {y.dtype} (no implicit promotion; cast() first)")
        return self.wrap(self.backend.where(c, x, y))

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

    def _check(self, op: str, kind: str) -> CudaTensor:
        """What an op accepts: any dtype, numeric (not bool), float only, or bool only
        (device-array.ts:486-494)."""
        x = self._handle(op)
        dt = x.dtype
        if kind == "numeric" and dt == "bool":
            raise TypeError(f"{_LABEL} {op}: not defined for bool; cast() first")
        if kind == "float" and dt not in FLOAT:
            raise TypeError(f"{_LABEL} {op}: needs a float dtype, got {dt}; cast(\"f32\") first (no implicit promotion)")
        if kind == "bool" and dt != "bool":
            raise TypeError(f"{_LABEL} {op}: needs bool operands, got {dt}; cast(\"bool\") first (no implicit truthiness)")
        return x

    def _unary(self, op: str, kind: str, f) -> "DeviceArray":
        return self._wrap(f(self.device.backend, self._check(op, kind)))

    def _binary(self, op: str, other, kind: str, f) -> "DeviceArray":
        """A binary op; a number operand becomes an on-device constant of this array's dtype
        (device-array.ts:503-516)."""
        x = self._check(op, kind)
        be = self.device.backend
        if isinstance(other, (int, float)) and not isinstance(other, bool):
            if kind == "bool":
                raise TypeError(f"{_LABEL} {op}: needs a DeviceArray operand")
            y = be.from_host_sync(host(x.dtype, (1,), [other]))
            try:
                return self._wrap(f(be, x, y))
            finally:
                be.dispose(y)
        y = self.device._own(other, op)
        if x.dtype != y.dtype:
            raise TypeError(f"{_LABEL} {op}: dtype mismatch {x.dtype} vs {y.dtype} (no implicit promotion; cast() first)")
        return self._wrap(f(be, x, y))

    def _reduce(self, op: str, kind: str, axis, keepDims: bool, f) -> "DeviceArray":
        """One axis, or every element (through a flat view) when ``axis`` is None (:519-539)."""
        x = self._check(op, kind)
        be = self.device.backend
        nd = len(x.shape)
        if axis is not None:
            if not -nd <= axis < nd:
                raise ValueError(f"{_LABEL} {op}: axis {axis} out of range for ndim {nd}")
            return self._wrap(f(be, x, axis % nd, keepDims))
        flat = be.reshape(x, (x.size,))
        try:
            r = f(be, flat, 0, False)
        finally:
            be.dispose(flat)
        if keepDims:
            kept = be.reshape(r, (1,) * nd)
            be.dispose(r)
            r = kept
        return self._wrap(r)

    # element-wise arithmetic (NumPy broadcasting, matching dtypes)
    def add(self, other) -> "DeviceArray":
        return self._binary("add", other, "numeric", lambda b, x, y: b.add(x, y))

    def sub(self, other) -> "DeviceArray":
        return self._binary("sub", other, "numeric", lambda b, x, y: b.sub(x, y))

    def mul(self, other) -> "DeviceArray":
        return self._binary("mul", other, "numeric", lambda b, x, y: b.mul(x, y))

    def div(self, other) -> "DeviceArray":
        return self._binary("div", other, "numeric", lambda b, x, y: b.div(x, y))

    def maximum(self, other) -> "DeviceArray":
        return self._binary("maximum", other, "numeric", lambda b, x, y: b.maximum(x, y))

    def minimum(self, other) -> "DeviceArray":
        """Composed as -maximum(-a, -b), as the reference does (device-array.ts:304-307)."""
        def f(b, x, y):
            nx, ny = b.neg(x), b.neg(y)
            m = b.maximum(nx, ny)
            r = b.neg(m)
            for t in (nx, ny, m):
                b.dispose(t)
            return r
        return self._binary("minimum", other, "numeric", f)

    def pow(self, other) -> "DeviceArray":
        return self._binary("pow", other, "float", lambda b, x, y: b.pow(x, y))

    # unary math
    def neg(self):
        return self._unary("neg", "numeric", lambda b, x: b.neg(x))

    def abs(self):
        return self._unary("abs", "numeric", lambda b, x: b.abs(x))

    def exp(self):
        return self._unary("exp", "float", lambda b, x: b.exp(x))

    def log(self):
        return self._unary("log", "float", lambda b, x: b.log(x))

    def sqrt(self):
        return self._unary("sqrt", "float", lambda b, x: b.sqrt(x))

    def rsqrt(self):
        return self._unary("rsqrt", "float", lambda b, x: b.rsqrt(x))

    def tanh(self):
        return self._unary("tanh", "float", lambda b, x: b.tanh(x))

    def sigmoid(self):
        return self._unary("sigmoid", "float", lambda b, x: b.sigmoid(x))

    def erf(self):
        return self._unary("erf", "float", lambda b, x: b.erf(x))

    def relu(self):
        return self._unary("relu", "numeric", lambda b, x: b.relu(x))

    # comparisons & logic (bool results)
    def equal(self, other):
        return self._binary("equal", other, "any", lambda b, x, y: b.equal(x, y))

    def notEqual(self, other):
        return self._binary("notEqual", other, "any", lambda b, x, y: b.notEqual(x, y))

    def less(self, other):
        return self._binary("less", other, "any", lambda b, x, y: b.less(x, y))

    def lessEqual(self, other):
        return self._binary("lessEqual", other, "any", lambda b, x, y: b.lessEqual(x, y))

    def greater(self, other):
        return self._binary("greater", other, "any", lambda b, x, y: b.greater(x, y))

    def greaterEqual(self, other):
        return self._binary("greaterEqual", other, "any", lambda b, x, y: b.greaterEqual(x, y))

    def logicalAnd(self, other):
        return self._binary("logicalAnd", other, "bool", lambda b, x, y: b.logicalAnd(x, y))

    def logicalOr(self, other):
        return self._binary("logicalOr", other, "bool", lambda b, x, y: b.logicalOr(x, y))

    def logicalNot(self):
        return self._unary("logicalNot", "bool", lambda b, x: b.logicalNot(x))

    # reductions & scans
    def sum(self, axis=None, keepDims: bool = False):
        return self._reduce("sum", "numeric", axis, keepDims, lambda b, x, a, k: b.sum(x, a, k))

    def mean(self, axis=None, keepDims: bool = False):
        return self._reduce("mean", "float", axis, keepDims, lambda b, x, a, k: b.mean(x, a, k))

    def max(self, axis=None, keepDims: bool = False):
        return self._reduce("max", "numeric", axis, keepDims, lambda b, x, a, k: b.max(x, a, k))

    def min(self, axis=None, keepDims: bool = False):
        return self._reduce("min", "numeric", axis, keepDims, lambda b, x, a, k: b.min(x, a, k))

    def argmax(self, axis=None, keepDims: bool = False):
        return self._reduce("argmax", "numeric", axis, keepDims, lambda b, x, a, k: b.argmax(x, a, k))

    def argmin(self, axis=None, keepDims: bool = False):
        return self._reduce("argmin", "numeric", axis, keepDims, lambda b, x, a, k: b.argmin(x, a, k))

    def cumsum(self, axis=None):
        """Inclusive prefix sum along ``axis``; with no axis, over the flattened array."""
        x = self._check("cumsum", "numeric")
        be = self.device.backend
        if axis is not None:
            return self._wrap(be.cumsum(x, axis))
        flat = be.reshape(x, (x.size,))
        try:
            return self._wrap(be.cumsum(flat, 0))
        finally:
            be.dispose(flat)

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

    # ---- fusion (tensor-compile IR -> one CUDA kernel; facade.ts:126-164) -----------------------
    def fuse(self, expr, inputs, precision: str = "f64"):
        """Evaluates a traced element-wise expression (an IRNode dict or a ``Traced``) over
        ``inputs`` in ONE kernel launch with no intermediate buffers. Inputs are float arrays (or
        raw backend tensors) that broadcast against each other like NumPy's; the result is a new
        f32 array of the broadcast shape (a raw tensor when the first input is one). The
        expression is evaluated in f64 and rounded once (the CPU backend's evaluator), or with
        ``precision="f32"`` in f32 throughout (the WebGPU backend's WGSL kernels)."""
        from .fusion import fuse
        if not inputs:
            raise ValueError(f"{_LABEL} fuse: needs at least one input")
        arrays = isinstance(inputs[0], DeviceArray)
        raw = [self._own(x, "fuse") if isinstance(x, DeviceArray) else x for x in inputs]
        out = fuse(self.backend, expr, raw, precision)
        return self.wrap(out) if arrays else out

    def compile(self, num_inputs: int, fn, precision: str = "f64"):
        """Traces ``fn`` once over symbolic inputs and returns a function that runs it fused on this
        device: ``f = dev.compile(2, lambda x, y: x.mul(y).add(1).gelu()); z = f(a, b)``."""
        from .fusion import Traced
        node = fn(*[Traced.input(i) for i in range(num_inputs)]).node

        def run(*inputs):
            if len(inputs) != num_inputs:
                raise ValueError(f"{_LABEL} compile: expects {num_inputs} input(s), got {len(inputs)}")
            return self.fuse(node, list(inputs), precision)

        return run

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
