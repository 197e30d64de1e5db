"""ctypes front end of the CPU oracle (oracle/mp_oracle.c) — TEST INFRASTRUCTURE ONLY.

Imported by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg,
as the checker. The CUDA product path (math-plus_b200/) never imports it.

Each function names the reference function it restates (paths inside the
math-plus repository); the arithmetic lives in mp_oracle.c.
"""
from __future__ import annotations

import ctypes as C
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
            os.path.join(_HERE, "mp_oracle.c")
        ):
            build()
        L = C.CDLL(_LIB_PATH)
        f64, f32p, u64 = C.c_double, C.POINTER(C.c_float), C.c_uint64
        vp, sz, i64p = C.c_void_p, C.c_size_t, C.POINTER(C.c_int64)
        L.mp_rng_init.argtypes = [vp, u64, u64]
        L.mp_rng_next_u32.argtypes = [vp]
        L.mp_rng_next_u32.restype = C.c_uint32
        L.mp_rng_next_float.argtypes = [vp]
        L.mp_rng_next_float.restype = f64
        L.mp_rng_next_below.argtypes = [vp, C.c_uint32]
        L.mp_rng_next_below.restype = C.c_uint32
        L.mp_normal_sample.argtypes = [vp, f64, f64]
        L.mp_normal_sample.restype = f64
        L.mp_fill_uniform_f32.argtypes = [u64, sz, f64, f64, vp]
        L.mp_fill_normal_f32.argtypes = [u64, sz, f64, f64, vp]
        L.mp_fill_normal_half.argtypes = [u64, sz, f64, f64, C.c_int, vp]
        L.mp_fill_below_i32.argtypes = [u64, sz, C.c_uint32, vp]
        L.mp_encode_half.argtypes = [C.c_int, f64]
        L.mp_encode_half.restype = C.c_uint16
        L.mp_decode_half.argtypes = [C.c_int, C.c_uint16]
        L.mp_decode_half.restype = f64
        L.mp_lcg_gemm.argtypes = [sz, C.c_uint32, vp]
        L.mp_lcg_seeded.argtypes = [sz, C.c_uint32, f64, f64, vp]
        for n in ("mp_erf", "mp_erfc", "mp_gelu_erf"):
            getattr(L, n).argtypes = [f64]
            getattr(L, n).restype = f64
        L.mp_gemm_nt.argtypes = [vp, vp, vp, sz, sz, C.c_int, C.c_int, C.c_int]
        L.mp_gemm_nt_par.argtypes = [vp, vp, vp, sz, sz, C.c_int, C.c_int, C.c_int, C.c_int]
        L.mp_softmax_axis_f32.argtypes = [vp, C.c_int, C.c_int, C.c_int, vp]
        L.mp_matmul_f32.argtypes = [vp, i64p, C.c_int, vp, i64p, C.c_int, vp, C.c_int]
        L.mp_matmul_f32.restype = C.c_int
        L.mp_linear_f32.argtypes = [vp, C.c_int, C.c_int, vp, C.c_int, vp, vp, C.c_int]
        L.mp_attention_f32.argtypes = [vp, vp, vp] + [C.c_int] * 7 + [f64, vp, C.c_int, i64p, vp, C.c_int]
        L.mp_layer_norm_f32.argtypes = [vp, C.c_int, C.c_int, vp, vp, f64, vp]
        L.mp_gelu_f32.argtypes = [vp, sz, vp]
        L.mp_take_rows_f32.argtypes = [vp, C.c_int, C.c_int, vp, sz, vp]
        L.mp_take_rows_f32.restype = C.c_long
        L.mp_rope_half_f32.argtypes = [vp, C.c_int, C.c_int, C.c_int, f64, vp]
        L.mp_geglu_rows_f32.argtypes = [vp, C.c_int, C.c_int, vp]
        L.mp_masked_mean_pool_f32.argtypes = [vp, C.c_int, C.c_int, C.c_int, vp, vp]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def default_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


# ---- seeded inputs (packages/tensor-core/src/random.ts) ---------------------------------

class Rng:
    """PCG32 XSH-RR, ``new Rng(seed, sequence)`` (random.ts:17-66)."""

    def __init__(self, seed: int = 0, sequence: int = 1):
        self._st = (C.c_uint64 * 2)()
        lib().mp_rng_init(C.byref(self._st), seed & (2**64 - 1), sequence & (2**64 - 1))

    def next_uint32(self) -> int:
        return lib().mp_rng_next_u32(C.byref(self._st))

    def next_float(self) -> float:
        return lib().mp_rng_next_float(C.byref(self._st))

    def next_below(self, bound: int) -> int:
        return lib().mp_rng_next_below(C.byref(self._st), bound)

    def normal(self, mean: float = 0.0, std: float = 1.0) -> float:
        return lib().mp_normal_sample(C.byref(self._st), mean, std)


def uniform_f32(n: int, seed: int, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    """``random.uniform([n], {rng: seed(seed), min: lo, max: hi})`` in f32 storage."""
    out = np.empty(n, np.float32)
    lib().mp_fill_uniform_f32(seed, n, lo, hi, _ptr(out))
    return out


def normal_f32(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().mp_fill_normal_f32(seed, n, mean, std, _ptr(out))
    return out


def normal_half_bits(n: int, seed: int, mean: float, std: float, bf16: bool) -> np.ndarray:
    """``random.normal`` into f16/bf16 storage: Box-Muller then encodeHalf (RNE), as uint16 bits."""
    out = np.empty(n, np.uint16)
    lib().mp_fill_normal_half(seed, n, mean, std, 1 if bf16 else 0, _ptr(out))
    return out


def randint_i32(n: int, seed: int, bound: int) -> np.ndarray:
    out = np.empty(n, np.int32)
    lib().mp_fill_below_i32(seed, n, bound, _ptr(out))
    return out


def encode_half(x: float, bf16: bool) -> int:
    return lib().mp_encode_half(1 if bf16 else 0, float(x))


def decode_half(bits: int, bf16: bool) -> float:
    return lib().mp_decode_half(1 if bf16 else 0, bits)


def half_bits_to_f32(bits: np.ndarray, bf16: bool) -> np.ndarray:
    """Exact widening of f16/bf16 bit patterns (tensor-cpu's fromHost, packages/tensor-cpu/src/index.ts:226-229)."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    if bf16:
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


def lcg_gemm(n: int, seed: int) -> np.ndarray:
    """packages/tensor-webgpu/test/gemm.test.ts:85-93."""
    out = np.empty(n, np.float32)
    lib().mp_lcg_gemm(n, seed & 0xFFFFFFFF, _ptr(out))
    return out


def lcg_seeded(n: int, seed: int, lo: float = -2.0, hi: float = 2.0) -> np.ndarray:
    """packages/tensor-cpu/test/helpers.ts:115-124 (f64 values)."""
    out = np.empty(n, np.float64)
    lib().mp_lcg_seeded(n, seed & 0xFFFFFFFF, lo, hi, _ptr(out))
    return out


# ---- special functions (packages/special/src/index.ts) ----------------------------------

def erf(x: float) -> float:
    return lib().mp_erf(float(x))


def erfc(x: float) -> float:
    return lib().mp_erfc(float(x))


def gelu_erf(x: float) -> float:
    return lib().mp_gelu_erf(float(x))


# ---- ops (tensor-cpu Backend glue over tensor-core kernels) ---------------------------

def matmul(a, b, threads: int = 1) -> np.ndarray:
    """``CpuBackendImpl.matmul`` -> ``Tensor.matmul`` (tensor-cpu/src/index.ts:755-762)."""
    a, b = _f32(a), _f32(b)
    if a.ndim < 2 or b.ndim < 2:
        raise ValueError("matmul needs rank >= 2")
    batch = np.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    out = np.empty(batch + (a.shape[-2], b.shape[-1]), np.float32)
    sa = (C.c_int64 * a.ndim)(*a.shape)
    sb = (C.c_int64 * b.ndim)(*b.shape)
    rc = lib().mp_matmul_f32(_ptr(a), sa, a.ndim, _ptr(b), sb, b.ndim, _ptr(out), threads)
    if rc != 0:
        raise ValueError(f"matmul shapes {a.shape} @ {b.shape} (code {rc})")
    return out


def linear(x, w, bias=None, threads: int = 1) -> np.ndarray:
    """``CpuBackendImpl.linear`` -> ``linearNT`` (tensor-cpu/src/index.ts:764-774)."""
    x, w = _f32(x), _f32(w)
    n, k = w.shape
    rows = x.size // k if k else int(np.prod(x.shape[:-1]))
    out = np.empty(x.shape[:-1] + (n,), np.float32)
    bias_keep = _f32(bias) if bias is not None else None
    lib().mp_linear_f32(_ptr(x), rows, k, _ptr(w), n, _ptr(bias_keep) if bias_keep is not None else None,
                        _ptr(out), threads)
    return out


def sdpa(q, k, v, mask=None, scale: float | None = None, threads: int = 1) -> np.ndarray:
    """``CpuBackendImpl.sdpa`` -> ``attention`` (tensor-cpu/src/index.ts:821-840)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, H, Lq, Dh = q.shape
    Hk, Lk, Dv = k.shape[1], k.shape[2], v.shape[3]
    if H % Hk:
        raise ValueError("H must be a multiple of Hk")
    if scale is None:
        scale = 1.0 / np.sqrt(Dh)
    out = np.empty((B, H, Lq, Dv), np.float32)
    strides = (C.c_int64 * 4)(0, 0, 0, 0)
    kind, mptr, keep = 0, None, None
    if mask is not None:
        m = np.asarray(mask)
        shape = (1,) * (4 - m.ndim) + m.shape
        target = (B, H, Lq, Lk)
        if np.broadcast_shapes(shape, target) != target:
            raise ValueError(f"mask {m.shape} does not broadcast to {target}")
        if m.dtype == np.bool_ or m.dtype == np.uint8:
            keep = np.ascontiguousarray(m != 0, dtype=np.uint8).reshape(shape)
            kind = 1
        else:
            keep = _f32(m).reshape(shape)
            kind = 2
        st, acc = [0] * 4, 1
        for d in range(3, -1, -1):
            st[d] = 0 if shape[d] == 1 else acc
            acc *= shape[d]
        strides = (C.c_int64 * 4)(*st)
        mptr = _ptr(keep)
    lib().mp_attention_f32(_ptr(q), _ptr(k), _ptr(v), B, H, Hk, Lq, Lk, Dh, Dv, float(scale), mptr, kind,
                           strides, _ptr(out), threads)
    return out


def softmax(x, axis: int = -1) -> np.ndarray:
    """``CpuBackendImpl.softmax`` -> ``softmaxAxis`` (tensor-cpu/src/index.ts:716-722)."""
    x = _f32(x)
    axis = axis % x.ndim
    outer = int(np.prod(x.shape[:axis]))
    dim = x.shape[axis]
    inner = int(np.prod(x.shape[axis + 1:]))
    out = np.empty_like(x)
    if dim > 0:
        lib().mp_softmax_axis_f32(_ptr(x), outer, dim, inner, _ptr(out))
    return out


def gelu(x) -> np.ndarray:
    """``CpuBackendImpl.gelu`` -> ``unaryFlat(UN_GELU)`` (nn-kernels.ts:47)."""
    x = _f32(x)
    out = np.empty_like(x)
    lib().mp_gelu_f32(_ptr(x), x.size, _ptr(out))
    return out


def add_f32(x, y) -> np.ndarray:
    """Broadcasting f32 add with one f32 rounding (binaryFlat OP_ADD, kernels.ts:43-55)."""
    return (_f32(x).astype(np.float64) + _f32(y).astype(np.float64)).astype(np.float32)


def layer_norm(x, w=None, b=None, eps: float = 1e-5) -> np.ndarray:
    """``CpuBackendImpl.layerNorm`` -> ``layerNormRows`` (tensor-cpu/src/index.ts:776-782)."""
    x = _f32(x)
    D = x.shape[-1]
    out = np.empty_like(x)
    wk = _f32(w) if w is not None else None
    bk = _f32(b) if b is not None else None
    lib().mp_layer_norm_f32(_ptr(x), x.size // D if D else 0, D, _ptr(wk) if wk is not None else None,
                            _ptr(bk) if bk is not None else None, eps, _ptr(out))
    return out


def embedding(table, ids) -> np.ndarray:
    """``CpuBackendImpl.embedding`` -> ``takeRows`` (tensor-cpu/src/index.ts:784-791)."""
    table = _f32(table)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    V, D = table.shape
    out = np.empty(ids.shape + (D,), np.float32)
    bad = lib().mp_take_rows_f32(_ptr(table), D, V, _ptr(ids), ids.size, _ptr(out))
    if bad >= 0:
        raise IndexError(f"takeRows: row index {int(ids.reshape(-1)[bad])} out of range [0, {V})")
    return out


def sort_axis(x, axis: int = -1) -> np.ndarray:
    """``CpuBackendImpl.sort`` -> ``sortAxis`` (tensor-cpu/src/index.ts:724-734, kernels.ts:601-617):
    each lane sorted by the typed-array order (numeric ascending, -0 before +0, NaN last)."""
    x = np.asarray(x)
    if x.dtype.kind == "f":
        f = x.astype(np.float32)
        bits = f.view(np.uint32)
        key = np.where(bits & 0x80000000, ~bits, bits | 0x80000000).astype(np.uint32)
        key = np.where(np.isnan(f), np.uint32(0xFFFFFFFF), key)
        order = np.argsort(key, axis=axis, kind="stable")
        return np.take_along_axis(x, order, axis=axis)
    return np.sort(x, axis=axis, kind="stable")


def gather_rows(x, idx) -> np.ndarray:
    """``CpuBackendImpl.gatherRows`` (tensor-cpu/src/index.ts:793-810): x [B, L, D], idx [B, M]
    (negative counts from the end) -> [B, M, D] via takeRows."""
    x = np.asarray(x)
    idx = np.asarray(idx, np.int64)
    B, L, D = x.shape
    r = np.where(idx < 0, idx + L, idx)
    bad = np.argwhere((r < 0) | (r >= L))
    if bad.size:
        b, m = bad[0]
        raise IndexError(f"gatherRows index {int(idx[b, m])} out of range for length {L}")
    return x[np.arange(B)[:, None], r]


def rope(x, base: float) -> np.ndarray:
    """``CpuBackendImpl.rope`` -> ``ropeHalf`` (tensor-cpu/src/index.ts:812-819, nn-kernels.ts:138-160)."""
    x = _f32(x)
    B, H, L, Dh = x.shape
    out = np.empty_like(x)
    lib().mp_rope_half_f32(_ptr(x), B * H, L, Dh, float(base), _ptr(out))
    return out


def geglu(x) -> np.ndarray:
    """``CpuBackendImpl.geglu`` -> ``gegluRows`` (tensor-cpu/src/index.ts:842-850, nn-kernels.ts:245-250)."""
    x = _f32(x)
    D = x.shape[-1] // 2
    out = np.empty(x.shape[:-1] + (D,), np.float32)
    lib().mp_geglu_rows_f32(_ptr(x), x.size // (2 * D) if D else 0, D, _ptr(out))
    return out


def mean_pool(x, mask) -> np.ndarray:
    """``CpuBackendImpl.meanPool`` -> ``maskedMeanPool`` (tensor-cpu/src/index.ts:852-860,
    nn-kernels.ts:256-271)."""
    x = _f32(x)
    B, L, D = x.shape
    m = _f32(np.asarray(mask, np.float64))
    out = np.empty((B, D), np.float32)
    lib().mp_masked_mean_pool_f32(_ptr(x), B, L, D, _ptr(m), _ptr(out))
    return out


# ---- tensor-compile's evaluator (packages/tensor-compile/src/ir.ts) ----------------------

def _js_round(x: float) -> float:
    """Math.round: nearest integer, ties toward +Infinity, -0 for x in [-0.5, -0]."""
    if x != x or math.isinf(x):
        return x
    f = math.floor(x)
    r = f + 1.0 if x - f >= 0.5 else float(f)
    return math.copysign(0.0, x) if r == 0 else r


def _js_sign(x: float) -> float:
    return 1.0 if x > 0 else (-1.0 if x < 0 else x)


def _js_pow(a: float, b: float) -> float:
    """Math.pow: NaN for a NaN exponent and for (+-1) ** (+-Infinity)."""
    if b != b or (abs(a) == 1.0 and math.isinf(b)):
        return math.nan
    try:
        return math.pow(a, b)
    except ZeroDivisionError:  # 0 ** negative
        return math.copysign(math.inf, a) if (b % 2 == 1) else math.inf
    except (OverflowError, ValueError):
        return float(np.power(np.float64(a), np.float64(b)))


def _safe(fn):
    """A libm function with IEEE results where Python's math raises (domain -> NaN, overflow -> inf)."""
    def g(x):
        try:
            return fn(x)
        except ValueError:
            return math.nan
        except OverflowError:
            return math.inf
    return g


def _div(a, b):
    with np.errstate(all="ignore"):
        return np.divide(a, b)


_UNARY_F64 = {
    "neg": lambda x: -x,
    "relu": lambda x: np.where(x > 0, x, 0.0),
    "sigmoid": lambda x: _div(1.0, 1.0 + _map(math.exp, -x)),
    "gelu": lambda x: _map(lambda v: lib().mp_gelu_erf(v), x),
    "gelu_tanh": lambda x: 0.5 * x * (1.0 + _map(math.tanh, 0.7978845608028654 * (x + 0.044715 * x * x * x))),
    "exp": lambda x: _map(math.exp, x), "log": lambda x: _map(math.log, x), "sqrt": lambda x: _map(math.sqrt, x),
    "sin": lambda x: _map(math.sin, x), "cos": lambda x: _map(math.cos, x), "tan": lambda x: _map(math.tan, x),
    "asin": lambda x: _map(math.asin, x), "acos": lambda x: _map(math.acos, x), "atan": lambda x: _map(math.atan, x),
    "sinh": lambda x: _map(math.sinh, x), "cosh": lambda x: _map(math.cosh, x), "tanh": lambda x: _map(math.tanh, x),
    "cot": lambda x: _div(1.0, _map(math.tan, x)), "sec": lambda x: _div(1.0, _map(math.cos, x)),
    "csc": lambda x: _div(1.0, _map(math.sin, x)),
    "asinh": lambda x: _map(math.asinh, x), "acosh": lambda x: _map(math.acosh, x),
    "atanh": lambda x: _map(math.atanh, x),
    "coth": lambda x: _div(1.0, _map(math.tanh, x)), "sech": lambda x: _div(1.0, _map(math.cosh, x)),
    "csch": lambda x: _div(1.0, _map(math.sinh, x)),
    "acot": lambda x: _map(math.atan, _div(1.0, x)), "asec": lambda x: _map(math.acos, _div(1.0, x)),
    "acsc": lambda x: _map(math.asin, _div(1.0, x)),
    "acoth": lambda x: 0.5 * _map(math.log, _div(x + 1.0, x - 1.0)),
    "asech": lambda x: _map(math.acosh, _div(1.0, x)), "acsch": lambda x: _map(math.asinh, _div(1.0, x)),
    "abs": np.abs, "log10": lambda x: _map(math.log10, x), "log2": lambda x: _map(math.log2, x),
    "cbrt": lambda x: _map(math.cbrt, x), "floor": np.floor, "ceil": np.ceil, "round": lambda x: _map(_js_round, x),
    "sign": lambda x: _map(_js_sign, x), "trunc": np.trunc, "expm1": lambda x: _map(math.expm1, x),
    "log1p": lambda x: _map(math.log1p, x), "erf": lambda x: _map(lambda v: lib().mp_erf(v), x),
}


def _map(fn, x):
    f = np.frompyfunc(_safe(fn), 1, 1)
    return np.asarray(f(np.asarray(x, np.float64)), np.float64)


_BINARY_F64 = {
    "add": np.add, "sub": np.subtract, "mul": np.multiply, "div": _div,
    "pow": lambda a, b: np.asarray(np.frompyfunc(_js_pow, 2, 1)(a, b), np.float64),
    "atan2": lambda a, b: np.asarray(np.frompyfunc(math.atan2, 2, 1)(a, b), np.float64),
    "hypot": lambda a, b: np.asarray(np.frompyfunc(math.hypot, 2, 1)(a, b), np.float64),
    "min": lambda a, b: np.where(a <= b, a, b), "max": lambda a, b: np.where(a >= b, a, b),
}
_CMP_F64 = {"lt": np.less, "le": np.less_equal, "gt": np.greater, "ge": np.greater_equal, "eq": np.equal,
            "ne": np.not_equal}


def eval_ir(node: dict, inputs, precision: str = "f64") -> np.ndarray:
    """``CompiledFn.forward`` (packages/tensor-compile/src/index.ts) over ``evalValue``
    (ir.ts:339-383): every node in f64 on the broadcast inputs with the value formulas of
    ``unaryValueAndDeriv`` (ir.ts:96-215) and JavaScript's Math semantics; the result rounded once to
    f32. Transcendentals come from the C library here and from V8's in the reference: they agree to
    the last place of f64 or within it.

    ``precision="f32"`` models an f32 evaluation (the WebGPU backend's WGSL kernels,
    packages/tensor-webgpu/src/fusion-wgsl.ts, compute every node in f32): each node's value is
    rounded to f32 before its consumers see it. For +, -, *, / and sqrt of f32 operands that is
    IEEE f32 arithmetic exactly; for the other functions it is the correctly rounded f32 value."""
    if precision not in ("f64", "f32"):
        raise ValueError(f"precision must be 'f64' or 'f32', got {precision!r}")
    xs = [np.asarray(x, np.float64) for x in inputs]
    shape = np.broadcast_shapes(*[x.shape for x in xs])
    xs = [np.broadcast_to(x, shape) for x in xs]
    if precision == "f32":
        xs = [x.astype(np.float32).astype(np.float64) for x in xs]

    def ev(n):
        v = ev_node(n)
        return v.astype(np.float32).astype(np.float64) if precision == "f32" else v

    def ev_node(n):
        k = n["kind"]
        if k == "input":
            return xs[n["index"]]
        if k == "const":
            return np.full(shape, float(n["value"]))
        if k == "unary":
            with np.errstate(all="ignore"):
                return np.asarray(_UNARY_F64[n["op"]](ev(n["arg"])), np.float64)
        if k == "binary":
            with np.errstate(all="ignore"):
                return np.asarray(_BINARY_F64[n["op"]](ev(n["left"]), ev(n["right"])), np.float64)
        if k == "cmp":
            return np.where(_CMP_F64[n["op"]](ev(n["left"]), ev(n["right"])), 1.0, 0.0)
        if k == "select":
            c = ev(n["cond"])
            return np.where(c != 0, ev(n["then"]), ev(n["else"]))
        raise ValueError(n)

    with np.errstate(all="ignore"):
        return np.asarray(ev(node), np.float64).astype(np.float32)


def round_bf16(x) -> np.ndarray:
    """What a bf16 store keeps of an f32 value (round to nearest even), back in f32."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    bits = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint32) << 16
    return bits.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def gpt2_forward(w: dict, ids, n_layer: int, n_head: int, eps: float = 1e-5, store=round_bf16,
                 threads: int = 1, residual_in_epilogue: bool = False, stop_after: int | None = None) -> np.ndarray:
    """A GPT-2-shaped forward composed from the reference's CPU ops: token + position
    ``takeRows``, then per layer the pre-norm block of ``TransformerEncoderLayer.forward``
    (packages/tensor-autograd/src/transformer.ts:320-333, normFirst) with ``MultiheadAttention``'s
    packed in-projection and head split / merge (transformer.ts:223-241) under a causal mask,
    exact GELU, and a final LayerNorm and tied LM head (``linearNT`` with the token table).
    ``w`` holds f32 arrays under GPT-2's parameter names; ``store`` is applied to every op's
    output (the device stores bf16). ``residual_in_epilogue``: the two residual adds take the
    projection's f32 result before it is stored (the device adds the residual inside the GEMM's
    epilogue and stores once). ``stop_after``: return the residual stream [B, L, D] after that many
    blocks instead of the logits. Returns logits [B, L, vocab]."""
    ids = np.ascontiguousarray(ids, np.int32)
    B, L = ids.shape
    D = w["wte"].shape[1]
    Dh = D // n_head
    causal = np.tril(np.ones((L, L), np.bool_)).reshape(1, 1, L, L)
    proj_store = (lambda t: t) if residual_in_epilogue else store
    x = store(add_f32(embedding(w["wte"], ids), embedding(w["wpe"], np.arange(L, dtype=np.int32))))
    x = x.reshape(B * L, D)
    for i in range(n_layer if stop_after is None else stop_after):
        p = f"h.{i}."
        h = store(layer_norm(x, w[p + "ln_1.weight"], w[p + "ln_1.bias"], eps))
        qkv = store(linear(h, w[p + "attn.in_proj_weight"], w[p + "attn.in_proj_bias"], threads=threads))
        q, k, v = (np.ascontiguousarray(t) for t in np.transpose(qkv.reshape(B, L, 3, n_head, Dh), (2, 0, 3, 1, 4)))
        a = store(sdpa(q, k, v, causal, 1.0 / np.sqrt(Dh), threads=threads))
        merged = np.ascontiguousarray(np.transpose(a, (0, 2, 1, 3))).reshape(B * L, D)
        o = proj_store(linear(merged, w[p + "attn.out_proj.weight"], w[p + "attn.out_proj.bias"], threads=threads))
        x1 = store(add_f32(x, o))
        h2 = store(layer_norm(x1, w[p + "ln_2.weight"], w[p + "ln_2.bias"], eps))
        f = store(gelu(linear(h2, w[p + "mlp.fc.weight"], w[p + "mlp.fc.bias"], threads=threads)))
        g = proj_store(linear(f, w[p + "mlp.proj.weight"], w[p + "mlp.proj.bias"], threads=threads))
        x = store(add_f32(x1, g))
    if stop_after is not None:
        return x.reshape(B, L, D)
    h = store(layer_norm(x, w["ln_f.weight"], w["ln_f.bias"], eps))
    return store(linear(h, w["wte"], threads=threads)).reshape(B, L, -1)


def gemm_nt_f64(a: np.ndarray, b_nt: np.ndarray, threads: int = 1) -> np.ndarray:
    """Raw ``gemmNT`` over packed f64 panels (kernels.ts:299-362): a [M,K], b_nt [N,K]."""
    a = np.ascontiguousarray(a, np.float64)
    b_nt = np.ascontiguousarray(b_nt, np.float64)
    M, K = a.shape
    N = b_nt.shape[0]
    out = np.empty((M, N), np.float64)
    lib().mp_gemm_nt_par(_ptr(a), _ptr(b_nt), _ptr(out), 0, N, M, N, K, threads)
    return out
