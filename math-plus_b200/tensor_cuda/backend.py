"""``CudaBackend``: the ``@johnhenry/tensor-backend`` ``Backend`` contract over libmathplus_cuda.so.

Mirrors the method set of tensor-cpu's ``CpuBackendImpl`` (packages/tensor-cpu/src/index.ts:200-861):
transfers (``fromHost`` / ``read``, async), lifetime (``dispose``, ``scope``, ``flush``,
``destroy``), ``reshape``, ``transpose``, ``slice``, ``split``, ``concat``, ``cast``, the element-wise
ops (``add``, ``sub``, ``mul``, ``div``, ``maximum``, ``pow``, ``where``, ``scale``, ``exp``, ``log``,
``relu``, ``gelu``, ``sqrt``, ``rsqrt``, ``tanh``, ``sigmoid``, ``erf``, ``neg``, ``abs``),
comparisons and logical ops, reductions (``sum``, ``mean``, ``max``, ``min``, ``argmax``,
``argmin``, ``cumsum``, ``softmax``), and the contractions ``matmul``, ``linear``, ``sdpa``,
``layerNorm``, ``embedding``.

Lazy inside, eager-observable (RFC 0001 §12 Q1, as the MLX and WebGPU backends): ``matmul`` and
``linear`` return a handle whose GEMM has not run yet; an ``add`` of a bias row, a ``gelu`` and
then an ``add`` of a same-shape array (a residual) applied to that handle fold into the GEMM's
epilogue, so ``x.matmul(w).add(b).gelu()`` and ``h.add(x.matmul(w))`` are one kernel each. Anything that reads the handle (another op, ``read``, ``flush``) runs it. Shape and dtype
errors are raised at the call site.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, replace

import numpy as np

from . import _ffi as F
from . import plan as P
from .runtime import Device, DeviceBuffer, gemm_desc, sdpa_desc

FLOAT = ("f32", "f16", "bf16")
STORAGE = {"f32": np.float32, "f16": np.float16, "bf16": np.uint16, "i32": np.int32, "bool": np.uint8}


@dataclass
class HostTensor:
    """tensor-backend's ``HostTensor``: dtype, shape and flat data (bf16 as raw uint16 bits)."""
    dtype: str
    shape: tuple
    data: np.ndarray


def host(dtype: str, shape, data) -> HostTensor:
    """tensor-backend's ``host()`` helper: values are converted to the dtype's storage."""
    shape = tuple(int(s) for s in shape)
    if dtype == "bf16":
        arr = np.asarray(data)
        if arr.dtype != np.uint16:
            x = np.ascontiguousarray(arr, np.float32).view(np.uint32).astype(np.uint64)
            arr = ((x + 0x7FFF + ((x >> 16) & 1)) >> 16).astype(np.uint16)
    elif dtype == "bool":
        arr = (np.asarray(data) != 0).astype(np.uint8)
    else:
        arr = np.asarray(data, dtype=STORAGE[dtype])
    return HostTensor(dtype, shape, np.ascontiguousarray(arr).reshape(-1))


class _Slice:
    """A byte range of a DeviceBuffer, used as a buffer: views at an offset (``split``) share and
    keep alive the block they point into."""

    __slots__ = ("base", "offset")

    def __init__(self, base, offset: int):
        self.base, self.offset = base, int(offset)

    @property
    def ptr(self) -> int:
        return self.base.ptr + self.offset

    def retain(self) -> "_Slice":
        self.base.retain()
        return self

    def release(self) -> None:
        self.base.release()


class _Borrowed:
    """Device memory owned elsewhere, used as a buffer (retain / release do nothing)."""

    __slots__ = ("ptr",)

    def __init__(self, ptr: int):
        self.ptr = int(ptr)

    def retain(self) -> "_Borrowed":
        return self

    def release(self) -> None:
        pass


@dataclass
class _PendingGemm:
    """A GEMM not yet run. It holds references to its operands' buffers, so disposing the operand
    arrays does not free memory the GEMM will still read."""
    a: DeviceBuffer
    b: DeviceBuffer
    dtype_in: str
    b_layout: int
    m: int
    n: int
    k: int
    batch_shape: tuple
    a_strides: tuple
    b_strides: tuple
    bias: DeviceBuffer | None = None
    bias_dtype: str = "f32"
    epilogue: int = 0
    resid: DeviceBuffer | None = None  # added last (MPC_EPI_RESIDUAL), in the output dtype

    def retain(self) -> "_PendingGemm":
        for b in (self.a, self.b, self.bias, self.resid):
            if b is not None:
                b.retain()
        return self

    def release(self) -> None:
        for b in (self.a, self.b, self.bias, self.resid):
            if b is not None:
                b.release()


class CudaTensor:
    """A backend handle: shape, dtype and device memory (or a GEMM that has not run yet)."""

    def __init__(self, backend: "CudaBackend", shape, dtype: str, buf: DeviceBuffer | None = None,
                 pending: _PendingGemm | None = None):
        self.backend = backend
        self.shape = tuple(int(s) for s in shape)
        self.dtype = dtype
        self._buf = buf
        self._pending = pending
        self.disposed = False

    @property
    def size(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    @property
    def nbytes(self) -> int:
        return self.size * F.DTYPE_BYTES[F.DTYPE_CODES[self.dtype]]

    @property
    def ptr(self) -> int:
        """Device address; runs a pending GEMM first."""
        if self.disposed:
            raise RuntimeError("tensor-cuda: tensor used after dispose")
        if self._pending is not None:
            self.backend._run_gemm(self)
        return self._buf.ptr

    def _release(self) -> None:
        if self.disposed:
            return
        if self._buf is not None:
            self._buf.release()
        if self._pending is not None:
            self._pending.release()
        self._buf = None
        self._pending = None
        self.disposed = True


class CudaBackend:
    """The device backend (one per device ordinal, like bridge.ts:8-12 for WebGPU)."""

    name = "cuda"

    def __init__(self, device: Device):
        self.device = device
        self._scopes: list[set] = []

    # ---- bookkeeping -----------------------------------------------------------------------
    def supports(self, dtype: str) -> bool:
        return dtype in ("f32", "f16", "bf16", "i32", "bool")

    def _make(self, shape, dtype, buf=None, pending=None) -> CudaTensor:
        t = CudaTensor(self, shape, dtype, buf, pending)
        if self._scopes:
            self._scopes[-1].add(t)
        return t

    def _alloc(self, shape, dtype) -> CudaTensor:
        n = 1
        for s in shape:
            n *= int(s)
        return self._make(shape, dtype, self.device.alloc(n * F.DTYPE_BYTES[F.DTYPE_CODES[dtype]]))

    @staticmethod
    def _check_live(*ts):
        for t in ts:
            if t is not None and t.disposed:
                raise RuntimeError("tensor-cuda: tensor used after dispose")

    # ---- transfers / lifetime ----------------------------------------------------------------
    async def fromHost(self, h: HostTensor) -> CudaTensor:
        return self.from_host_sync(h)

    def from_host_sync(self, h: HostTensor) -> CudaTensor:
        if not self.supports(h.dtype):
            raise TypeError(f"tensor-cuda: fromHost: unsupported dtype {h.dtype}")
        n = 1
        for s in h.shape:
            n *= int(s)
        data = np.ascontiguousarray(h.data).reshape(-1)
        if data.size != n:
            raise ValueError(f"tensor-cuda: fromHost {data.size} values for shape [{','.join(map(str, h.shape))}]")
        if h.dtype == "bool":
            data = (data != 0).astype(np.uint8)
        else:
            data = data.astype(STORAGE[h.dtype], copy=False)
        t = self._alloc(h.shape, h.dtype)
        if n:
            self.device.copy_h2d(t._buf.ptr, data)
            self.device.stream_sync()  # the host buffer may change after the call returns
        return t

    async def read(self, t: CudaTensor) -> HostTensor:
        return self.read_sync(t)

    def read_sync(self, t: CudaTensor) -> HostTensor:
        self._check_live(t)
        ptr = t.ptr
        out = np.empty(t.size, dtype=STORAGE[t.dtype])
        if t.size:
            self.device.copy_d2h_into(out, ptr)
            self.device.stream_sync()
        return HostTensor(t.dtype, t.shape, out)

    def dispose(self, t: CudaTensor) -> None:
        t._release()

    def external(self, ptr: int, shape, dtype: str) -> CudaTensor:
        """A handle over device memory this backend does not own (another allocator's tensor);
        the caller keeps that memory alive while the handle is in use."""
        if dtype not in STORAGE:
            raise TypeError(f"tensor-cuda: external: unsupported dtype {dtype}")
        return self._make(shape, dtype, _Borrowed(ptr))

    def scope(self, fn):
        created: set = set()
        self._scopes.append(created)
        try:
            result = fn()
        except BaseException:
            self._scopes.pop()
            for t in created:
                t._release()
            raise
        self._scopes.pop()
        keep = set()

        def visit(v):
            if isinstance(v, CudaTensor):
                keep.add(v)

        if isinstance(result, CudaTensor):
            keep.add(result)
        elif isinstance(result, (list, tuple)):
            for v in result:
                visit(v)
        elif isinstance(result, dict):
            for v in result.values():
                visit(v)
        parent = self._scopes[-1] if self._scopes else None
        for t in created:
            if t in keep:
                if parent is not None:
                    parent.add(t)
            else:
                t._release()
        return result

    def flush(self, *ts) -> None:
        for t in ts:
            _ = t.ptr
        self.device.stream_sync()

    def destroy(self) -> None:
        for s in self._scopes:
            for t in s:
                t._release()
        self._scopes.clear()

    # ---- shape / dtype -----------------------------------------------------------------------
    def reshape(self, x: CudaTensor, shape) -> CudaTensor:
        self._check_live(x)
        shape = list(shape)
        if shape.count(-1) > 1:
            raise ValueError("tensor-cuda: reshape allows one -1")
        if -1 in shape:
            known = 1
            for s in shape:
                if s != -1:
                    known *= s
            if known == 0 or x.size % known:
                raise ValueError(f"tensor-cuda: reshape [{','.join(map(str, x.shape))}] to {shape}")
            shape[shape.index(-1)] = x.size // known
        n = 1
        for s in shape:
            n *= s
        if n != x.size:
            raise ValueError(f"tensor-cuda: reshape [{','.join(map(str, x.shape))}] to {shape}")
        _ = x.ptr
        return self._make(shape, x.dtype, x._buf.retain())  # a view sharing the buffer

    def split(self, x: CudaTensor, sections: int, axis: int = 0) -> list:
        """Equal parts along ``axis`` (Backend.split). Along the leading axis (or one behind
        leading 1s) the parts are views sharing x's memory; other axes are not supported here."""
        self._check_live(x)
        nd = len(x.shape)
        ax = axis % nd
        if any(d != 1 for d in x.shape[:ax]):
            raise NotImplementedError("tensor-cuda: split: only along the leading non-unit axis")
        if sections <= 0 or x.shape[ax] % sections:
            raise ValueError(f"tensor-cuda: split: {x.shape[ax]} is not divisible into {sections} parts")
        _ = x.ptr
        part = x.shape[ax] // sections
        shape = x.shape[:ax] + (part,) + x.shape[ax + 1:]
        step = x.nbytes // sections
        base, off = (x._buf.base, x._buf.offset) if isinstance(x._buf, _Slice) else (x._buf, 0)
        return [self._make(shape, x.dtype, _Slice(base, off + i * step).retain()) for i in range(sections)]

    def transpose(self, x: CudaTensor, perm=None) -> CudaTensor:
        """Axis permutation (default: reversed), like numpy.transpose (device-array.ts:457-471)."""
        self._check_live(x)
        nd = len(x.shape)
        perm = list(range(nd - 1, -1, -1)) if perm is None else [p % nd if nd else p for p in perm]
        if sorted(perm) != list(range(nd)):
            raise ValueError(f"tensor-cuda: transpose: {perm} is not a permutation")
        if nd <= 1 or perm == list(range(nd)):
            return self.reshape(x, x.shape)
        out = self._alloc(tuple(x.shape[p] for p in perm), x.dtype)
        shape = (C.c_int64 * nd)(*x.shape)
        pm = (C.c_int32 * nd)(*perm)
        F.call("mpc_transpose", self.device.handle, C.c_void_p(x.ptr), C.c_void_p(out._buf.ptr),
               F.DTYPE_BYTES[F.DTYPE_CODES[x.dtype]], nd, shape, pm, None)
        return out

    def cast(self, x: CudaTensor, dtype: str) -> CudaTensor:
        self._check_live(x)
        if dtype == x.dtype:
            return self.reshape(x, x.shape)
        if x.dtype not in FLOAT or dtype not in FLOAT:
            raise NotImplementedError(f"tensor-cuda: cast {x.dtype} -> {dtype} (float <-> float only)")
        out = self._alloc(x.shape, dtype)
        F.call("mpc_cast", self.device.handle, C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype], C.c_void_p(out._buf.ptr),
               F.DTYPE_CODES[dtype], x.size, None)
        return out

    # ---- element-wise ------------------------------------------------------------------------
    def add(self, x: CudaTensor, y: CudaTensor) -> CudaTensor:
        self._check_live(x, y)
        if x.dtype != y.dtype:
            raise TypeError(f"tensor-cuda: add: dtype mismatch {x.dtype} vs {y.dtype} (no implicit promotion)")
        if x.dtype not in FLOAT or P.broadcast_shapes(x.shape, y.shape) not in (tuple(x.shape), tuple(y.shape)):
            return self._binary(x, y, "add")  # integer data, or both operands broadcast
        if x.size < y.size:  # add is commutative: keep the larger operand first
            x, y = y, x
        pg = x._pending
        done = F.EPI_BIAS | F.EPI_GELU | F.EPI_RESIDUAL
        bias_like = pg is not None and not (pg.epilogue & done) and y.size == pg.n and \
            all(s == 1 for s in y.shape[:-1]) and y.shape[-1] == pg.n and len(y.shape) <= len(x.shape)
        if bias_like:  # fold the bias row into the pending GEMM's epilogue
            _ = y.ptr
            folded = replace(pg, bias=y._buf, bias_dtype=y.dtype, epilogue=pg.epilogue | F.EPI_BIAS).retain()
            return self._make(x.shape, x.dtype, pending=folded)
        if x is not y and x.shape == y.shape:
            # a residual add: fold the other operand into a pending GEMM's epilogue (added last)
            for a, r in ((x, y), (y, x)):
                pa = a._pending
                if pa is not None and not (pa.epilogue & F.EPI_RESIDUAL):
                    _ = r.ptr
                    folded = replace(pa, resid=r._buf, epilogue=pa.epilogue | F.EPI_RESIDUAL).retain()
                    return self._make(a.shape, a.dtype, pending=folded)
        try:
            n_x, n_y = P.add_plan(x.shape, y.shape)
        except NotImplementedError:  # not a repeated trailing block: the general broadcast kernel
            return self._binary(x, y, "add")
        out = self._alloc(x.shape, x.dtype)
        F.call("mpc_add", self.device.handle, C.c_void_p(x.ptr), C.c_void_p(y.ptr), C.c_void_p(out._buf.ptr),
               F.DTYPE_CODES[x.dtype], n_x, n_y, None)
        return out

    def gelu(self, x: CudaTensor) -> CudaTensor:
        self._check_live(x)
        if x.dtype not in FLOAT:
            raise TypeError(f"tensor-cuda: gelu: float dtypes only, got {x.dtype}")
        pg = x._pending
        if pg is not None and not (pg.epilogue & (F.EPI_GELU | F.EPI_RESIDUAL)):  # fold into the pending GEMM
            return self._make(x.shape, x.dtype, pending=replace(pg, epilogue=pg.epilogue | F.EPI_GELU).retain())
        out = self._alloc(x.shape, x.dtype)
        F.call("mpc_gelu", self.device.handle, C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype], C.c_void_p(out._buf.ptr),
               F.DTYPE_CODES[x.dtype], x.size, None)
        return out

    def softmax(self, x: CudaTensor, axis: int = -1) -> CudaTensor:
        """Stable softmax along ``axis`` (softmaxAxis, kernels.ts:219-247); f32 result for f32 input,
        the input's dtype otherwise."""
        self._check_live(x)
        if x.dtype not in FLOAT:
            raise TypeError(f"tensor-cuda: softmax: float dtypes only, got {x.dtype}")
        nd = len(x.shape)
        if not -nd <= axis < nd:
            raise ValueError(f"tensor-cuda: softmax: axis {axis} out of range")
        ax = axis % nd
        outer = int(np.prod(x.shape[:ax])) if ax else 1
        inner = int(np.prod(x.shape[ax + 1:])) if ax + 1 < nd else 1
        out = self._alloc(x.shape, "f32")
        F.call("mpc_softmax", self.device.handle, C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype], C.c_void_p(out._buf.ptr),
               outer, x.shape[ax], inner, None)
        if x.dtype != "f32":
            res = self.cast(out, x.dtype)
            out._release()
            return res
        return out

    # ---- the rest of the element-wise / comparison / reduction / copy ops -----------------------
    # (CpuBackendImpl, packages/tensor-cpu/src/index.ts:318-735): evaluated in f64 on the device
    # with one rounding on store; same-dtype operands (no implicit promotion), broadcasting as
    # tensor-core's broadcastShapes.
    def _unary(self, x: CudaTensor, name: str, out_dtype: str | None = None, alpha: float = 0.0) -> CudaTensor:
        self._check_live(x)
        out = self._alloc(x.shape, out_dtype or x.dtype)
        F.call("mpc_unary", self.device.handle, F.UNARY_OPS[name], C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype],
               C.c_void_p(out._buf.ptr), F.DTYPE_CODES[out.dtype], x.size, C.c_float(alpha), None)
        return out

    def _float_out(self, x: CudaTensor) -> str:
        return x.dtype if x.dtype in FLOAT else "f32"

    def exp(self, x):
        return self._unary(x, "exp", self._float_out(x))

    def log(self, x):
        return self._unary(x, "log", self._float_out(x))

    def sqrt(self, x):
        return self._unary(x, "sqrt", self._float_out(x))

    def rsqrt(self, x):
        return self._unary(x, "rsqrt", self._float_out(x))

    def tanh(self, x):
        return self._unary(x, "tanh", self._float_out(x))

    def sigmoid(self, x):
        return self._unary(x, "sigmoid", self._float_out(x))

    def erf(self, x):
        return self._unary(x, "erf", self._float_out(x))

    def relu(self, x):
        return self._unary(x, "relu")

    def neg(self, x):
        return self._unary(x, "neg")

    def abs(self, x):
        return self._unary(x, "abs")

    def scale(self, x, s: float):
        return self._unary(x, "scale", self._float_out(x), float(s))

    def logicalNot(self, x):
        return self._unary(x, "logicalNot", "bool")

    @staticmethod
    def _strides_arr(strides):
        return (C.c_int64 * max(1, len(strides)))(*strides)

    def _binary(self, a: CudaTensor, b: CudaTensor, name: str, out_dtype: str | None = None) -> CudaTensor:
        self._check_live(a, b)
        if a.dtype != b.dtype:
            raise TypeError(f"tensor-cuda: {name}: dtype mismatch {a.dtype} vs {b.dtype} (no implicit promotion)")
        shape = P.broadcast_shapes(a.shape, b.shape)
        if len(shape) > 6:
            raise NotImplementedError(f"tensor-cuda: {name}: more than 6 axes")
        dt = out_dtype or ("i32" if a.dtype == "bool" else a.dtype)
        out = self._alloc(shape, dt)
        F.call("mpc_binary", self.device.handle, F.BINARY_OPS[name], C.c_void_p(a.ptr), C.c_void_p(b.ptr),
               F.DTYPE_CODES[a.dtype], C.c_void_p(out._buf.ptr), F.DTYPE_CODES[dt], len(shape),
               self._strides_arr(shape), self._strides_arr(P.aligned_strides(a.shape, shape)),
               self._strides_arr(P.aligned_strides(b.shape, shape)), None)
        return out

    def sub(self, a, b):
        return self._binary(a, b, "sub")

    def mul(self, a, b):
        return self._binary(a, b, "mul")

    def div(self, a, b):
        return self._binary(a, b, "div")

    def maximum(self, a, b):
        return self._binary(a, b, "maximum")

    def pow(self, a, b):
        if a.dtype not in FLOAT:
            raise TypeError(f"tensor-cuda: pow: float dtypes only, got {a.dtype}")
        return self._binary(a, b, "pow")

    def equal(self, a, b):
        return self._binary(a, b, "equal", "bool")

    def notEqual(self, a, b):
        return self._binary(a, b, "notEqual", "bool")

    def less(self, a, b):
        return self._binary(a, b, "less", "bool")

    def lessEqual(self, a, b):
        return self._binary(a, b, "lessEqual", "bool")

    def greater(self, a, b):
        return self._binary(a, b, "greater", "bool")

    def greaterEqual(self, a, b):
        return self._binary(a, b, "greaterEqual", "bool")

    def logicalAnd(self, a, b):
        return self._binary(a, b, "logicalAnd", "bool")

    def logicalOr(self, a, b):
        return self._binary(a, b, "logicalOr", "bool")

    def where(self, cond: CudaTensor, a: CudaTensor, b: CudaTensor) -> CudaTensor:
        """cond ? a : b with broadcasting (index.ts:511-545); cond is bool."""
        self._check_live(cond, a, b)
        if cond.dtype != "bool":
            raise TypeError(f"tensor-cuda: where: the condition is bool, got {cond.dtype}")
        if a.dtype != b.dtype:
            raise TypeError(f"tensor-cuda: where: dtype mismatch {a.dtype} vs {b.dtype} (no implicit promotion)")
        shape = P.broadcast_shapes(P.broadcast_shapes(cond.shape, a.shape), b.shape)
        out = self._alloc(shape, a.dtype)
        F.call("mpc_where", self.device.handle, C.c_void_p(cond.ptr), C.c_void_p(a.ptr), C.c_void_p(b.ptr),
               F.DTYPE_CODES[a.dtype], C.c_void_p(out._buf.ptr), len(shape), self._strides_arr(shape),
               self._strides_arr(P.aligned_strides(cond.shape, shape)),
               self._strides_arr(P.aligned_strides(a.shape, shape)),
               self._strides_arr(P.aligned_strides(b.shape, shape)), None)
        return out

    @staticmethod
    def _around(shape, axis: int):
        nd = len(shape)
        if not -nd <= axis < nd:
            raise ValueError(f"tensor-cuda: axis {axis} out of range for rank {nd}")
        a = axis % nd
        outer = int(np.prod(shape[:a])) if a else 1
        inner = int(np.prod(shape[a + 1:])) if a + 1 < nd else 1
        return a, outer, int(shape[a]), inner

    def _reduce(self, x: CudaTensor, axis: int, keepDims: bool, name: str, dt: str) -> CudaTensor:
        self._check_live(x)
        a, outer, dim, inner = self._around(x.shape, axis)
        if dim == 0 and name not in ("sum", "mean"):
            raise ValueError(f"tensor-cuda: {name} over an empty axis")
        shape = tuple(x.shape[:a]) + ((1,) if keepDims else ()) + tuple(x.shape[a + 1:])
        out = self._alloc(shape, dt)
        F.call("mpc_reduce", self.device.handle, F.REDUCE_OPS[name], C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype],
               C.c_void_p(out._buf.ptr), F.DTYPE_CODES[dt], outer, dim, inner, None)
        return out

    def sum(self, x, axis: int, keepDims: bool = False):
        return self._reduce(x, axis, keepDims, "sum", "i32" if x.dtype in ("bool", "i32") else x.dtype)

    def mean(self, x, axis: int, keepDims: bool = False):
        return self._reduce(x, axis, keepDims, "mean", self._float_out(x))

    def max(self, x, axis: int, keepDims: bool = False):
        return self._reduce(x, axis, keepDims, "max", x.dtype)

    def min(self, x, axis: int, keepDims: bool = False):
        return self._reduce(x, axis, keepDims, "min", x.dtype)

    def argmax(self, x, axis: int, keepDims: bool = False):
        return self._reduce(x, axis, keepDims, "argmax", "i32")

    def argmin(self, x, axis: int, keepDims: bool = False):
        return self._reduce(x, axis, keepDims, "argmin", "i32")

    def cumsum(self, x: CudaTensor, axis: int) -> CudaTensor:
        self._check_live(x)
        _, outer, dim, inner = self._around(x.shape, axis)
        dt = "i32" if x.dtype in ("bool", "i32") else x.dtype
        out = self._alloc(x.shape, dt)
        F.call("mpc_cumsum", self.device.handle, C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype], C.c_void_p(out._buf.ptr),
               F.DTYPE_CODES[dt], outer, dim, inner, None)
        return out

    def slice(self, x: CudaTensor, begin, end) -> CudaTensor:
        """x[begin:end] per axis, negative indices from the end, clamped (index.ts:333-352)."""
        self._check_live(x)
        nd = len(x.shape)
        in_st = [int(np.prod(x.shape[i + 1:])) for i in range(nd)]  # row-major strides
        shape, base = [], 0
        for i, d in enumerate(x.shape):
            lo = begin[i] if i < len(begin) else 0
            hi = end[i] if i < len(end) else d
            lo += d if lo < 0 else 0
            hi += d if hi < 0 else 0
            lo = min(max(lo, 0), d)
            hi = min(max(hi, lo), d)
            base += lo * in_st[i]
            shape.append(hi - lo)
        out = self._alloc(shape, x.dtype)
        eb = F.DTYPE_BYTES[F.DTYPE_CODES[x.dtype]]
        out_st = [int(np.prod(shape[i + 1:])) for i in range(nd)]
        F.call("mpc_strided_copy", self.device.handle, C.c_void_p(x.ptr + base * eb), self._strides_arr(in_st),
               C.c_void_p(out._buf.ptr), self._strides_arr(out_st), eb, nd, self._strides_arr(shape), None)
        return out

    def concat(self, xs, axis: int) -> CudaTensor:
        """Join along ``axis`` (index.ts:368-404); every input has the same dtype."""
        if not xs:
            raise ValueError("tensor-cuda: concat of nothing")
        self._check_live(*xs)
        first = xs[0]
        nd = len(first.shape)
        a = axis % nd
        for t in xs:
            if t.dtype != first.dtype:
                raise TypeError(f"tensor-cuda: concat: dtype mismatch {first.dtype} vs {t.dtype} (no implicit promotion)")
            if len(t.shape) != nd or any(t.shape[i] != first.shape[i] for i in range(nd) if i != a):
                raise ValueError(f"tensor-cuda: concat: shapes {[list(t.shape) for t in xs]} along axis {axis}")
        shape = list(first.shape)
        shape[a] = sum(t.shape[a] for t in xs)
        out = self._alloc(shape, first.dtype)
        eb = F.DTYPE_BYTES[F.DTYPE_CODES[first.dtype]]
        out_st = [int(np.prod(shape[i + 1:])) for i in range(nd)]
        off = 0
        for t in xs:
            if t.size:
                in_st = [int(np.prod(t.shape[i + 1:])) for i in range(nd)]
                F.call("mpc_strided_copy", self.device.handle, C.c_void_p(t.ptr), self._strides_arr(in_st),
                       C.c_void_p(out._buf.ptr + off * out_st[a] * eb), self._strides_arr(out_st), eb, nd,
                       self._strides_arr(t.shape), None)
            off += t.shape[a]
        return out

    # ---- contractions --------------------------------------------------------------------------
    def matmul(self, a: CudaTensor, b: CudaTensor, out_dtype: str | None = None) -> CudaTensor:
        """[..., m, k] @ [..., k, n] with broadcast batch axes (Tensor.matmul); the result keeps the
        operands' dtype unless ``out_dtype`` asks otherwise (f32 accumulation either way)."""
        self._check_live(a, b)
        if a.dtype != b.dtype:
            raise TypeError(f"tensor-cuda: matmul: dtype mismatch {a.dtype} vs {b.dtype} (no implicit promotion; cast() first)")
        if a.dtype not in FLOAT:
            raise NotImplementedError("tensor-cuda: matmul: float dtypes only")
        pl = P.matmul_plan(a.shape, b.shape)
        _, _ = a.ptr, b.ptr
        pg = _PendingGemm(a._buf, b._buf, a.dtype, F.B_KN, pl.m, pl.n, pl.k, pl.batch_shape, pl.a_batch_strides,
                          pl.b_batch_strides).retain()
        return self._make(pl.out_shape, out_dtype or a.dtype, pending=pg)

    def linear(self, x: CudaTensor, w: CudaTensor, bias: CudaTensor | None = None, activation: str | None = None,
               out_dtype: str | None = None) -> CudaTensor:
        """x · wᵀ (+ bias) with w [out, in] (linearNT); ``activation="gelu"`` fuses the exact GELU."""
        self._check_live(x, w, bias)
        rows, n_in, n_out, out_shape = P.linear_plan(x.shape, w.shape, bias.shape if bias is not None else None)
        if x.dtype != w.dtype:
            raise TypeError(f"tensor-cuda: linear: dtype mismatch {x.dtype} vs {w.dtype}")
        epi = F.EPI_BIAS if bias is not None else 0
        if activation == "gelu":
            epi |= F.EPI_GELU
        elif activation is not None:
            raise ValueError(f"tensor-cuda: linear: unknown activation {activation}")
        _, _ = x.ptr, w.ptr
        if bias is not None:
            _ = bias.ptr
        pg = _PendingGemm(x._buf, w._buf, x.dtype, F.B_NK, rows, n_out, n_in, (), (), (),
                          bias._buf if bias is not None else None, bias.dtype if bias is not None else "f32",
                          epi).retain()
        return self._make(out_shape, out_dtype or x.dtype, pending=pg)

    def _run_gemm(self, t: CudaTensor) -> None:
        pg = t._pending
        bias_ptr = None
        tmp = None
        if pg.bias is not None:
            bias_ptr = pg.bias.ptr
            if pg.bias_dtype != "f32":  # the epilogue reads an f32 bias row
                tmp = self.device.alloc(pg.n * 4)
                F.call("mpc_cast", self.device.handle, C.c_void_p(bias_ptr), F.DTYPE_CODES[pg.bias_dtype],
                       C.c_void_p(tmp.ptr), F.F32, pg.n, None)
                bias_ptr = tmp.ptr
        out = self.device.alloc(t.nbytes)
        desc = gemm_desc(pg.m, pg.n, pg.k, F.DTYPE_CODES[pg.dtype_in], F.DTYPE_CODES[t.dtype], pg.b_layout,
                         pg.epilogue, 1.0, pg.batch_shape, pg.a_strides, pg.b_strides)
        if pg.resid is not None:
            F.call("mpc_gemm_residual", self.device.handle, C.byref(desc), C.c_void_p(pg.a.ptr),
                   C.c_void_p(pg.b.ptr), C.c_void_p(out.ptr), C.c_void_p(bias_ptr) if bias_ptr else None,
                   C.c_void_p(pg.resid.ptr), None)
        else:
            self.device.gemm(desc, pg.a.ptr, pg.b.ptr, out.ptr, bias_ptr)
        if tmp is not None:
            tmp.release()
        pg.release()
        t._buf = out
        t._pending = None

    def sdpa(self, q: CudaTensor, k: CudaTensor, v: CudaTensor, mask: CudaTensor | None, scale: float,
             causal: bool = False, lse: bool = False):
        """softmax(scale·QKᵀ + mask)·V (attention, nn-kernels.ts:179-239). ``causal=True`` is the
        lower-triangular bool mask without materialising it; ``lse=True`` also returns the f32
        log-sum-exp per row."""
        self._check_live(q, k, v, mask)
        if not (q.dtype == k.dtype == v.dtype) or q.dtype not in FLOAT:
            raise TypeError("tensor-cuda: sdpa: q, k, v must share a float dtype")
        pl = P.sdpa_plan(q.shape, k.shape, v.shape, mask.shape if mask is not None else None)
        kind = F.MASK_NONE
        if mask is not None:
            kind = F.MASK_BOOL if mask.dtype == "bool" else F.MASK_ADD
            if kind == F.MASK_ADD and mask.dtype != "f32":
                raise TypeError("tensor-cuda: sdpa: additive masks are f32")
        out = self._alloc((pl.b, pl.h, pl.lq, pl.dv), q.dtype)
        lse_t = self._alloc((pl.b, pl.h, pl.lq), "f32") if lse else None
        desc = sdpa_desc(pl.b, pl.h, pl.hk, pl.lq, pl.lk, pl.d, pl.dv, F.DTYPE_CODES[q.dtype], causal, scale, kind,
                         pl.mask_strides)
        self.device.sdpa(desc, q.ptr, k.ptr, v.ptr, mask.ptr if mask is not None else None, out._buf.ptr,
                         lse_t._buf.ptr if lse_t is not None else None)
        return (out, lse_t) if lse else out

    def sdpa_packed(self, qkv: CudaTensor, n_head: int, scale: float, causal: bool = False) -> CudaTensor:
        """Self-attention over a packed projection, as ``MultiheadAttention`` does it
        (packages/tensor-autograd/src/transformer.ts:223-241): ``qkv`` [B, L, 3·H·Dh] laid out
        [B, L, 3, H, Dh] (the in-projection's output) -> [B, L, H·Dh] with heads merged, read and
        written in place by one kernel (no head split / merge copies)."""
        self._check_live(qkv)
        if len(qkv.shape) != 3 or qkv.shape[2] % (3 * n_head):
            raise ValueError(f"tensor-cuda: sdpa_packed: qkv [{','.join(map(str, qkv.shape))}] for {n_head} heads")
        if qkv.dtype not in FLOAT:
            raise TypeError("tensor-cuda: sdpa_packed: float dtypes only")
        B, L, three_e = qkv.shape
        E = three_e // 3
        Dh = E // n_head
        out = self._alloc((B, L, E), qkv.dtype)
        base = qkv.ptr
        eb = F.DTYPE_BYTES[F.DTYPE_CODES[qkv.dtype]]
        lay = F.SdpaLayout()
        for name in ("q", "k", "v"):
            getattr(lay, name)[:] = [L * three_e, Dh, three_e]
        lay.o[:] = [L * E, Dh, E]
        desc = sdpa_desc(B, n_head, n_head, L, L, Dh, Dh, F.DTYPE_CODES[qkv.dtype], causal, scale)
        F.call("mpc_sdpa_strided", self.device.handle, C.byref(desc), C.c_void_p(base), C.c_void_p(base + E * eb),
               C.c_void_p(base + 2 * E * eb), None, C.c_void_p(out._buf.ptr), None, C.byref(lay), None)
        return out

    def layerNorm(self, x: CudaTensor, weight: CudaTensor | None, bias: CudaTensor | None, eps: float = 1e-5):
        self._check_live(x, weight, bias)
        d = x.shape[-1]
        ws = []
        for t in (weight, bias):
            if t is not None and t.dtype != "f32":
                t = self.cast(t, "f32")
            ws.append(t)
        out = self._alloc(x.shape, x.dtype)
        F.call("mpc_layer_norm", self.device.handle, C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype],
               C.c_void_p(ws[0].ptr if ws[0] is not None else None), C.c_void_p(ws[1].ptr if ws[1] is not None else None),
               C.c_float(eps), C.c_void_p(out._buf.ptr), F.DTYPE_CODES[x.dtype], x.size // d if d else 0, d, None)
        return out

    def embedding(self, table: CudaTensor, ids: CudaTensor) -> CudaTensor:
        self._check_live(table, ids)
        if len(table.shape) != 2:
            raise ValueError("tensor-cuda: embedding table must be [V, D]")
        if ids.dtype != "i32":
            raise TypeError("tensor-cuda: embedding ids are i32")
        V, D = table.shape
        out = self._alloc(ids.shape + (D,), table.dtype)
        bad = C.c_int64(-1)
        rc = F.load().mpc_embedding(self.device.handle, C.c_void_p(table.ptr), F.DTYPE_CODES[table.dtype],
                                    C.c_void_p(ids.ptr), C.c_void_p(out._buf.ptr), ids.size, V, D, C.byref(bad), None)
        if rc == F.ERR_INVALID and bad.value >= 0:
            raise IndexError(f"tensor-cuda: embedding: id at position {bad.value} out of range [0, {V})")
        F.check(rc, "mpc_embedding")
        return out

    # ---- sort, row gather, rotary embedding, GEGLU, masked mean pool ----------------------------
    # (CpuBackendImpl, packages/tensor-cpu/src/index.ts:724-861): f64 arithmetic with one rounding;
    # results keep the input's dtype where the CPU backend returns f32 (f32 inputs give its bits).
    def sort(self, x: CudaTensor, axis: int = -1) -> CudaTensor:
        """Ascending along ``axis``: numeric order, -0 before +0, NaN last (sortAxis)."""
        self._check_live(x)
        _, outer, dim, inner = self._around(x.shape, axis)
        out = self._alloc(x.shape, x.dtype)
        F.call("mpc_sort", self.device.handle, C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype], C.c_void_p(out._buf.ptr),
               outer, dim, inner, None)
        return out

    def gatherRows(self, x: CudaTensor, idx: CudaTensor) -> CudaTensor:
        """x [B, L, D], idx i32 [B, M] -> [B, M, D]: out[b, m] = x[b, idx[b, m]], a negative index
        counting from the end (index.ts:793-810)."""
        self._check_live(x, idx)
        if len(x.shape) != 3 or len(idx.shape) != 2 or idx.shape[0] != x.shape[0]:
            raise ValueError(f"tensor-cuda: gatherRows [{','.join(map(str, x.shape))}] idx "
                             f"[{','.join(map(str, idx.shape))}]")
        if idx.dtype != "i32":
            raise TypeError("tensor-cuda: gatherRows idx is i32")
        B, L, D = x.shape
        M = idx.shape[1]
        out = self._alloc((B, M, D), x.dtype)
        bad = C.c_int64(-1)
        rc = F.load().mpc_gather_rows(self.device.handle, C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype],
                                      C.c_void_p(idx.ptr), C.c_void_p(out._buf.ptr), B, L, M, D, C.byref(bad), None)
        if rc == F.ERR_INVALID and bad.value >= 0:
            raw = self.read_sync(self.slice(self.reshape(idx, (B * M,)), [bad.value], [bad.value + 1])).data[0]
            out._release()
            raise IndexError(f"tensor-cuda: gatherRows index {int(raw)} out of range for length {L}")
        F.check(rc, "mpc_gather_rows")
        return out

    def rope(self, x: CudaTensor, base: float = 10000.0) -> CudaTensor:
        """Split-half rotary embedding of x [B, H, L, Dh], positions 0..L-1 (ropeHalf)."""
        self._check_live(x)
        if len(x.shape) != 4:
            raise ValueError(f"tensor-cuda: rope expects [B, H, L, Dh], got [{','.join(map(str, x.shape))}]")
        B, H, L, Dh = x.shape
        if Dh % 2:
            raise ValueError(f"tensor-cuda: rope needs an even head dim, got {Dh}")
        if x.dtype not in FLOAT:
            raise TypeError(f"tensor-cuda: rope: float dtypes only, got {x.dtype}")
        out = self._alloc(x.shape, x.dtype)
        F.call("mpc_rope", self.device.handle, C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype], C.c_void_p(out._buf.ptr),
               B * H, L, Dh, C.c_double(base), None)
        return out

    def geglu(self, x: CudaTensor) -> CudaTensor:
        """[..., 2D] -> [..., D]: GELU(first half) * second half (gegluRows)."""
        self._check_live(x)
        d2 = x.shape[-1] if x.shape else 0
        if not x.shape or d2 % 2:
            raise ValueError(f"tensor-cuda: geglu needs an even last axis, got {d2}")
        if x.dtype not in FLOAT:
            raise TypeError(f"tensor-cuda: geglu: float dtypes only, got {x.dtype}")
        D = d2 // 2
        rows = x.size // d2 if d2 else 0
        out = self._alloc(tuple(x.shape[:-1]) + (D,), x.dtype)
        F.call("mpc_geglu", self.device.handle, C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype], C.c_void_p(out._buf.ptr),
               rows, D, None)
        return out

    def meanPool(self, x: CudaTensor, mask: CudaTensor) -> CudaTensor:
        """x [B, L, D], mask [B, L] (nonzero = keep) -> [B, D] (maskedMeanPool)."""
        self._check_live(x, mask)
        if len(x.shape) != 3 or len(mask.shape) != 2 or tuple(mask.shape) != tuple(x.shape[:2]):
            raise ValueError(f"tensor-cuda: meanPool x [{','.join(map(str, x.shape))}] mask "
                             f"[{','.join(map(str, mask.shape))}]")
        if x.dtype not in FLOAT:
            raise TypeError(f"tensor-cuda: meanPool: float dtypes only, got {x.dtype}")
        B, L, D = x.shape
        out = self._alloc((B, D), x.dtype)
        F.call("mpc_mean_pool", self.device.handle, C.c_void_p(x.ptr), F.DTYPE_CODES[x.dtype], C.c_void_p(mask.ptr),
               F.DTYPE_CODES[mask.dtype], C.c_void_p(out._buf.ptr), B, L, D, None)
        return out
