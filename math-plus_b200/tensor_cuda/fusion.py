"""Element-wise fusion on the device: the tensor-compile IR (``Traced`` / ``IRNode``,
packages/tensor-compile/src/ir.ts) compiled into ONE CUDA kernel per expression, the counterpart of
``WebGpuDevice.fuse`` / ``compile`` (packages/tensor-webgpu/src/facade.ts:137-164).

``IRNode`` is the reference's JSON shape (``{"kind": "input", "index": 0}``, ``{"kind": "unary",
"op": "exp", "arg": ...}``, ...), so an expression serialised by the reference loads as is.
``lower`` turns it into the C ABI's instruction DAG (shared subtrees become one instruction), and
``FusedKernel`` compiles that once per device and input dtypes (NVRTC, sm_100a) and runs it with
NumPy broadcasting over the inputs. Every node evaluates in f64 with the reference's formulas;
the result is f32, like ``CompiledFn.forward`` on f32 inputs.
"""
from __future__ import annotations

import ctypes as C
import threading

import numpy as np

from . import _ffi as F

UNARY_OPS = ("neg", "relu", "sigmoid", "gelu", "gelu_tanh", "exp", "log", "sqrt", "sin", "cos", "tan", "asin",
             "acos", "atan", "sinh", "cosh", "tanh", "cot", "sec", "csc", "asinh", "acosh", "atanh", "coth", "sech",
             "csch", "acot", "asec", "acsc", "acoth", "asech", "acsch", "abs", "log10", "log2", "cbrt", "floor",
             "ceil", "round", "sign", "trunc", "expm1", "log1p", "erf")
BINARY_OPS = ("add", "sub", "mul", "div", "pow", "atan2", "hypot", "min", "max")
CMP_OPS = ("lt", "le", "gt", "ge", "eq", "ne")

IR_INPUT, IR_CONST, IR_SELECT = 1, 2, 3
UNARY_CODES = {op: 16 + i for i, op in enumerate(UNARY_OPS)}
BINARY_CODES = {op: 64 + i for i, op in enumerate(BINARY_OPS)}
CMP_CODES = {op: 80 + i for i, op in enumerate(CMP_OPS)}
MAX_INPUTS = 16


class Traced:
    """The IR builder of tensor-compile (ir.ts:386-596): methods build a node tree, nothing runs."""

    __slots__ = ("node",)

    def __init__(self, node: dict):
        self.node = node

    @staticmethod
    def input(index: int) -> "Traced":
        return Traced({"kind": "input", "index": int(index)})

    def _unary(self, op: str) -> "Traced":
        return Traced({"kind": "unary", "op": op, "arg": self.node})

    def _binary(self, op: str, other) -> "Traced":
        return Traced({"kind": "binary", "op": op, "left": self.node, "right": _to_node(other)})

    def cmp(self, op: str, other) -> "Traced":
        if op not in CMP_OPS:
            raise ValueError(f"unknown comparison {op!r}")
        return Traced({"kind": "cmp", "op": op, "left": self.node, "right": _to_node(other)})

    def select(self, then, else_value) -> "Traced":
        """``self`` is the condition: nonzero takes ``then``, zero ``else_value``."""
        return Traced({"kind": "select", "cond": self.node, "then": _to_node(then), "else": _to_node(else_value)})

    def gelu(self, approximate: str = "none") -> "Traced":
        if approximate not in ("none", "tanh"):
            raise ValueError(f'gelu: approximate must be "none" or "tanh", got {approximate!r}')
        return self._unary("gelu_tanh" if approximate == "tanh" else "gelu")

    def lt(self, other):
        return self.cmp("lt", other)

    def le(self, other):
        return self.cmp("le", other)

    def gt(self, other):
        return self.cmp("gt", other)

    def ge(self, other):
        return self.cmp("ge", other)

    def eq(self, other):
        return self.cmp("eq", other)

    def ne(self, other):
        return self.cmp("ne", other)


def _make_unary(op):
    return lambda self: self._unary(op)


def _make_binary(op):
    return lambda self, other: self._binary(op, other)


for _op in UNARY_OPS:
    if _op not in ("gelu", "gelu_tanh"):
        setattr(Traced, _op, _make_unary(_op))
for _op in BINARY_OPS:
    setattr(Traced, _op, _make_binary(_op))


def _to_node(x) -> dict:
    if isinstance(x, Traced):
        return x.node
    if isinstance(x, dict):
        return x
    return {"kind": "const", "value": float(x)}


def lower(node, n_inputs: int):
    """IRNode -> (instructions int32 [K, 4], constants f64 [C]) in the C ABI's form. Identical
    subtrees (the same node object, or equal structure) become one instruction."""
    node = node.node if isinstance(node, Traced) else node
    code, consts, memo, const_idx = [], [], {}, {}

    def emit(key, ins):
        if key not in memo:
            memo[key] = len(code)
            code.append(ins)
        return memo[key]

    def visit(n) -> int:
        kind = n.get("kind") if isinstance(n, dict) else None
        if kind == "input":
            i = int(n["index"])
            if not 0 <= i < n_inputs:
                raise ValueError(f"IR references input {i}, but numInputs is {n_inputs}")
            return emit(("input", i), (IR_INPUT, i, 0, 0))
        if kind == "const":
            v = float(n["value"])
            bits = np.float64(v).view(np.uint64).item()
            if bits not in const_idx:
                const_idx[bits] = len(consts)
                consts.append(v)
            return emit(("const", bits), (IR_CONST, const_idx[bits], 0, 0))
        if kind == "unary":
            if n["op"] not in UNARY_CODES:
                raise ValueError(f"unknown unary op {n['op']!r}")
            a = visit(n["arg"])
            return emit(("u", n["op"], a), (UNARY_CODES[n["op"]], a, 0, 0))
        if kind in ("binary", "cmp"):
            table = BINARY_CODES if kind == "binary" else CMP_CODES
            if n["op"] not in table:
                raise ValueError(f"unknown {kind} op {n['op']!r}")
            a, b = visit(n["left"]), visit(n["right"])
            return emit((kind, n["op"], a, b), (table[n["op"]], a, b, 0))
        if kind == "select":
            c, t, e = visit(n["cond"]), visit(n["then"]), visit(n["else"])
            return emit(("select", c, t, e), (IR_SELECT, c, t, e))
        raise ValueError(f"not an IR node: {n!r}")

    visit(node)
    return np.array(code, np.int32).reshape(-1, 4), np.array(consts, np.float64)


PRECISIONS = {"f64": 0, "f32": F.FUSED_F32}


def _flags(precision: str) -> int:
    """MPC_FUSED_* flags of an evaluation precision: "f64" (the JavaScript numbers of the CPU
    backend's evaluator, the default) or "f32" (the WebGPU backend's WGSL arithmetic)."""
    try:
        return PRECISIONS[precision]
    except KeyError:
        raise ValueError(f"fusion: precision must be 'f64' or 'f32', got {precision!r}") from None


def lowered_source(node, n_inputs: int, dtypes=None, check_compile: bool = False, precision: str = "f64") -> str:
    """The CUDA source the expression compiles to (no device needed); ``check_compile`` also runs
    NVRTC on it."""
    flags = _flags(precision)
    code, consts = lower(node, n_inputs)
    dts = (C.c_int32 * n_inputs)(*[F.DTYPE_CODES[d] for d in (dtypes or ["f32"] * n_inputs)])
    n = C.c_size_t(0)
    args = (code.ctypes.data_as(C.POINTER(C.c_int32)), len(code),
            consts.ctypes.data_as(C.POINTER(C.c_double)) if len(consts) else None, len(consts), n_inputs, dts)
    F.call("mpc_fused_lower", *args, flags, 0, None, 0, C.byref(n))
    buf = C.create_string_buffer(n.value + 1)
    F.call("mpc_fused_lower", *args, flags, 1 if check_compile else 0, buf, n.value + 1, C.byref(n))
    return buf.value.decode()


def broadcast_strides(shape, out_shape):
    """Element strides of a contiguous array of ``shape`` read at ``out_shape`` (0 on broadcast
    axes; NumPy's trailing alignment)."""
    st, acc = [0] * len(out_shape), 1
    off = len(out_shape) - len(shape)
    for k in range(len(shape) - 1, -1, -1):
        st[off + k] = 0 if shape[k] == 1 and out_shape[off + k] != 1 else acc
        acc *= shape[k]
    return st


class FusedKernel:
    """One compiled expression for one device, one tuple of input dtypes and one precision."""

    def __init__(self, device, code: np.ndarray, consts: np.ndarray, dtypes, precision: str = "f64"):
        self.device = device
        self.n_inputs = len(dtypes)
        dts = (C.c_int32 * self.n_inputs)(*[F.DTYPE_CODES[d] for d in dtypes])
        h = C.c_void_p()
        F.call("mpc_fused_create_ex", device.handle, code.ctypes.data_as(C.POINTER(C.c_int32)), len(code),
               consts.ctypes.data_as(C.POINTER(C.c_double)) if len(consts) else None, len(consts), self.n_inputs,
               dts, _flags(precision), C.byref(h))
        self.handle = h

    def run(self, ptrs, shapes, out_shape, out_ptr, stream=None) -> None:
        rank = len(out_shape)
        st = []
        for s in shapes:
            st += broadcast_strides(s, out_shape)
        F.call("mpc_fused_run", self.handle, (C.c_void_p * self.n_inputs)(*ptrs), rank,
               (C.c_int64 * max(rank, 1))(*out_shape), (C.c_int64 * max(len(st), 1))(*st), C.c_void_p(out_ptr),
               C.c_void_p(stream))

    def close(self) -> None:
        if self.handle:
            F.load().mpc_fused_destroy(self.handle)
            self.handle = None


_cache: dict = {}
_lock = threading.Lock()


def kernel_for(device, node, dtypes, precision: str = "f64") -> FusedKernel:
    """The compiled kernel of ``node`` for ``device``, these input dtypes and this precision
    (compiled once)."""
    _flags(precision)
    code, consts = lower(node, len(dtypes))
    key = (id(device), code.tobytes(), consts.tobytes(), tuple(dtypes), precision)
    with _lock:
        k = _cache.get(key)
        if k is None:
            k = _cache[key] = FusedKernel(device, code, consts, dtypes, precision)
    return k


def fuse(backend, expr, inputs, precision: str = "f64"):
    """Backend-level fusion: ``expr`` over backend tensors ``inputs`` (float dtypes), broadcast
    against each other; a new f32 tensor of the broadcast shape. ``precision`` "f64" evaluates as
    the CPU backend's evaluator does, "f32" as the WebGPU backend's WGSL kernels do."""
    node = expr.node if isinstance(expr, Traced) else expr
    if not inputs:
        raise ValueError("fuse: needs at least one input")
    if len(inputs) > MAX_INPUTS:
        raise ValueError(f"fuse: at most {MAX_INPUTS} inputs, got {len(inputs)}")
    backend._check_live(*inputs)
    for t in inputs:
        if t.dtype not in ("f32", "f16", "bf16"):
            raise TypeError(f"fuse: float inputs only, got {t.dtype}")
    try:
        out_shape = tuple(np.broadcast_shapes(*[tuple(t.shape) for t in inputs]))
    except ValueError as e:
        raise ValueError(f"fuse: shapes {[list(t.shape) for t in inputs]} do not broadcast") from e
    if len(out_shape) > 6:
        raise ValueError(f"fuse: rank {len(out_shape)} (at most 6)")
    k = kernel_for(backend.device, node, [t.dtype for t in inputs], precision)
    out = backend._alloc(out_shape, "f32")
    if out.size:
        k.run([t.ptr for t in inputs], [tuple(t.shape) for t in inputs], out_shape, out._buf.ptr)
    return out
