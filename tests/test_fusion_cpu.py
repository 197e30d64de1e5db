"""Element-wise fusion on the CPU: the IR builder, the lowering to the C ABI's instruction DAG and
to CUDA source (checked like the reference's WGSL lowering tests,
packages/tensor-webgpu/test/fusion-wgsl.test.ts:29-125), NVRTC compiling every op for sm_100a
(no device needed), and the oracle's evaluator against the reference's documented values."""
import json
import math

import numpy as np
import pytest

import oracle as O
from tensor_cuda import _ffi as F
from tensor_cuda.fusion import BINARY_OPS, CMP_OPS, UNARY_OPS, Traced, lower, lowered_source


def unary(op):
    return {"kind": "unary", "op": op, "arg": {"kind": "input", "index": 0}}


@pytest.mark.parametrize("op", UNARY_OPS)
def test_every_unary_op_lowers_and_reads_its_input(op):
    src = lowered_source(unary(op), 1)
    assert src.startswith("typedef double real;")
    assert "const real t0 = x0;" in src
    assert "const real t1 = " in src and "t0" in src.split("const real t1 = ")[1].split(";")[0]


@pytest.mark.parametrize("op", BINARY_OPS + CMP_OPS)
def test_every_binary_and_cmp_op_lowers_with_both_inputs(op):
    t = Traced.input(0).cmp(op, Traced.input(1)) if op in CMP_OPS else getattr(Traced.input(0), op)(Traced.input(1))
    line = lowered_source(t, 2).split("const real t2 = ")[1].split(";")[0]
    assert "t0" in line and "t1" in line
    if op in CMP_OPS:
        assert "? 1.0 : 0.0" in line


def test_select_compares_the_condition_against_zero():
    line = lowered_source(Traced.input(0).select(Traced.input(1), 2.5), 2).split("const real t3 = ")[1].split(";")[0]
    assert line == "(t0 != 0.0 ? t1 : t2)"


def test_every_op_compiles_for_sm100a_with_nvrtc():
    """One expression using every UnaryOp, BinaryOp, CmpOp and select, over f32 / f16 / bf16 inputs."""
    x, y, z = Traced.input(0), Traced.input(1), Traced.input(2)
    acc = None
    for op in UNARY_OPS:
        n = x.gelu("tanh" if op == "gelu_tanh" else "none") if op.startswith("gelu") else getattr(x, op)()
        acc = n if acc is None else acc.add(n)
    for op in BINARY_OPS:
        acc = acc.add(getattr(y, op)(z))
    for op in CMP_OPS:
        acc = acc.add(y.cmp(op, z))
    acc = acc.gt(0).select(acc, x.mul(-1.25))
    src = lowered_source(acc, 3, ["f32", "f16", "bf16"], check_compile=True)
    assert "ld_f16(p.in[1]" in src and "ld_bf16(p.in[2]" in src


def test_constants_are_exact_bit_patterns_and_shared_subtrees_lower_once():
    x = Traced.input(0)
    s = x.mul(x).add(0.1)
    e = s.add(s).sub(float("nan")).max(float("-inf"))
    code, consts = lower(e, 1)
    # input, mul, 0.1, add, add (s + s), nan, sub, -inf, max
    assert len(code) == 9
    assert consts[0] == 0.1 and np.isnan(consts[1]) and consts[2] == -np.inf
    src = lowered_source(e, 1)
    assert "__longlong_as_double(0x3fb999999999999aLL)" in src          # 0.1
    assert "__longlong_as_double(0xfff0000000000000LL)" in src          # -Infinity
    assert "(t6 >= t7 ? t6 : t7)" in src                               # max as l >= r ? l : r


def test_reference_json_nodes_and_input_range():
    node = json.loads('{"kind":"binary","op":"mul","left":{"kind":"input","index":0},'
                      '"right":{"kind":"unary","op":"relu","arg":{"kind":"input","index":1}}}')
    code, _ = lower(node, 2)
    assert code.tolist() == [[1, 0, 0, 0], [1, 1, 0, 0], [16 + UNARY_OPS.index("relu"), 1, 0, 0], [66, 0, 2, 0]]
    with pytest.raises(ValueError, match="IR references input 2, but numInputs is 2"):
        lower(Traced.input(2).neg(), 2)
    with pytest.raises(ValueError, match="unknown unary op"):
        lower({"kind": "unary", "op": "gamma", "arg": {"kind": "input", "index": 0}}, 1)


def test_the_library_validates_programs():
    """A forward reference or an unknown op is refused by the C ABI itself."""
    import ctypes as C
    code = np.array([[1, 0, 0, 0], [64, 0, 2, 0]], np.int32)  # operand 2 is not earlier
    dts = (C.c_int32 * 1)(F.F32)
    n = C.c_size_t(0)
    rc = F.load().mpc_fused_lower(code.ctypes.data_as(C.POINTER(C.c_int32)), 2, None, 0, 1, dts, 0, 0, None, 0,
                                  C.byref(n))
    assert rc == F.ERR_INVALID and "operands" in F.last_error()
    code = np.array([[1, 0, 0, 0], [99, 0, 0, 0]], np.int32)
    rc = F.load().mpc_fused_lower(code.ctypes.data_as(C.POINTER(C.c_int32)), 2, None, 0, 1, dts, 0, 0, None, 0,
                                  C.byref(n))
    assert rc == F.ERR_INVALID and "unknown op" in F.last_error()
    code = np.array([[1, 0, 0, 0]], np.int32)
    rc = F.load().mpc_fused_lower(code.ctypes.data_as(C.POINTER(C.c_int32)), 1, None, 0, 1, dts, 6, 0, None, 0,
                                  C.byref(n))
    assert rc == F.ERR_INVALID and "flags" in F.last_error()


# ---- the oracle's evaluator (evalValue, ir.ts:339-383) ------------------------------------------

def test_oracle_js_semantics():
    x = Traced.input(0)
    v = np.array([-2.5, -0.5, -0.2, 0.49999999999999994, 0.5, 2.5, 2.3, np.nan, -0.0])
    got = O.eval_ir(x.round().node, [v])
    want = np.array([-2, -0.0, -0.0, 0, 1, 3, 2, np.nan, -0.0], np.float32)  # Math.round
    assert np.array_equal(np.signbit(got), np.signbit(want)) and np.allclose(got, want, equal_nan=True)
    # ir-extended.test.ts:74-85: floor / ceil / round / sign / trunc at 2.3 equal Math.*(2.3)
    for op, ref in (("floor", 2.0), ("ceil", 3.0), ("round", 2.0), ("sign", 1.0), ("trunc", 2.0)):
        assert O.eval_ir(getattr(x, op)().node, [np.array([2.3])])[0] == ref
    # Math.pow: NaN exponent and (+-1) ** (+-Infinity) are NaN; 0 ** -2 is Infinity
    p = O.eval_ir(x.pow(Traced.input(1)).node, [np.array([1.0, -1.0, 0.0, 2.0]), np.array([np.nan, np.inf, -2.0, 0.5])])
    assert np.isnan(p[0]) and np.isnan(p[1]) and p[2] == np.inf and p[3] == np.float32(math.sqrt(2))
    # min / max as l <= r ? l : r; relu(NaN) = 0; select takes `then` for a NaN condition
    a, b = np.array([np.nan, 1.0, 2.0]), np.array([0.0, np.nan, 2.0])
    assert np.array_equal(O.eval_ir(x.min(Traced.input(1)).node, [a, b]), np.array([0.0, np.nan, 2.0], np.float32),
                          equal_nan=True)
    assert O.eval_ir(x.relu().node, [np.array([np.nan])])[0] == 0.0
    assert O.eval_ir(x.select(1.0, 2.0).node, [np.array([np.nan, 0.0])]).tolist() == [1.0, 2.0]
    # CompiledFn's NumPy broadcasting of the inputs (tensor-compile/src/index.ts, #broadcastInputs)
    out = O.eval_ir(x.add(Traced.input(1)).node, [np.ones((2, 3)), np.arange(3.0)])
    assert out.shape == (2, 3) and out.tolist() == [[1, 2, 3], [1, 2, 3]]


def test_oracle_matches_closed_forms():
    xs = np.linspace(-0.79, 0.79, 101)
    x = Traced.input(0)
    for op, f in (("exp", np.exp), ("sin", np.sin), ("atanh", np.arctanh), ("expm1", np.expm1), ("cbrt", np.cbrt),
                  ("sigmoid", lambda v: 1 / (1 + np.exp(-v))), ("acoth", lambda v: 0.5 * np.log((v + 1) / (v - 1)))):
        got = O.eval_ir(getattr(x, op)().node, [xs])
        with np.errstate(all="ignore"):
            want = f(xs).astype(np.float32)
        assert np.allclose(got, want, rtol=2e-7, atol=0, equal_nan=True), op
    from scipy.special import erf
    g = O.eval_ir(x.gelu().node, [xs])
    assert np.allclose(g, (0.5 * xs * (1 + erf(xs / np.sqrt(2)))).astype(np.float32), rtol=2e-7, atol=1e-12)


# ---- f32 evaluation (the WebGPU backend's precision, fusion-wgsl.ts) ----------------------------

def test_f32_lowering_uses_float_math_and_compiles_every_op():
    x, y, z = Traced.input(0), Traced.input(1), Traced.input(2)
    acc = None
    for op in UNARY_OPS:
        n = x.gelu("tanh" if op == "gelu_tanh" else "none") if op.startswith("gelu") else getattr(x, op)()
        acc = n if acc is None else acc.add(n)
    for op in BINARY_OPS:
        acc = acc.add(getattr(y, op)(z))
    for op in CMP_OPS:
        acc = acc.add(y.cmp(op, z))
    acc = acc.gt(0).select(acc, x.mul(-1.25))
    src = lowered_source(acc, 3, ["f32", "f16", "bf16"], check_compile=True, precision="f32")
    body = src[src.index("mpc_eval("):src.index("return t")]
    assert src.startswith("typedef float real;")
    for f in ("expf(", "asinf(", "sinf(", "normcdff(", "fabsf(", "atan2f(", "hypotf(", "log1pf(", "erff("):
        assert f in body, f
    assert "asin(" not in body.replace("asinf(", "") and "exp(" not in body.replace("expf(", "")
    assert "(float)__longlong_as_double(0xbff4000000000000LL)" in body            # -1.25 rounded to f32
    assert "? 1.0f : 0.0f" in body and "!= 0.0f ?" in body
    # the default stays f64
    assert lowered_source(x.exp(), 1).startswith("typedef double real;")


def test_precision_is_validated():
    with pytest.raises(ValueError, match="precision"):
        lowered_source(Traced.input(0).exp(), 1, precision="f16")
    with pytest.raises(ValueError, match="precision"):
        O.eval_ir(Traced.input(0).exp().node, [np.ones(2)], precision="bf16")


def test_oracle_f32_rounds_every_node():
    """(x + 1e-8) - x: f64 keeps the 1e-8, f32 arithmetic loses it for |x| >= 1."""
    x = Traced.input(0)
    e = x.add(1e-8).sub(x)
    v = np.array([1.0, 3.0, -2.0, 1e-9], np.float32)
    f64 = O.eval_ir(e.node, [v])
    f32 = O.eval_ir(e.node, [v], precision="f32")
    assert np.allclose(f64[:3], 1e-8, rtol=1e-6)
    assert f32[:3].tolist() == [0.0, 0.0, 0.0]
    v32 = v.astype(np.float32)
    assert f32[3] == (v32[3] + np.float32(1e-8)) - v32[3]


def test_oracle_f32_mode_is_ieee_f32_arithmetic():
    """The oracle's f32 evaluation (every node rounded to f32) equals NumPy's float32 arithmetic
    step by step for +, -, *, / and sqrt, which is what the device's f32 mode is held to bit for
    bit; transcendental nodes are the correctly rounded f32 of the f64 value."""
    rng = np.random.default_rng(31)
    a, b, c = (rng.standard_normal(20000).astype(np.float32) * 3 for _ in range(3))
    x, y, z = Traced.input(0), Traced.input(1), Traced.input(2)
    e = x.add(y).mul(z).sub(x).div(y.add(3.5)).max(x.mul(0.1)).add(z.mul(z).mul(1.0 / 3.0)).abs().sqrt()
    got = O.eval_ir(e.node, [a, b, c], precision="f32")
    f = np.float32
    with np.errstate(all="ignore"):
        t = ((a + b) * c - a) / (b + f(3.5))
        t = np.where(t >= a * f(0.1), t, a * f(0.1))
        want = np.sqrt(np.abs(t + (c * c) * f(1.0 / 3.0)))
    assert want.dtype == np.float32
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    ex = O.eval_ir(x.exp().node, [a], precision="f32")
    assert np.array_equal(ex, np.exp(a.astype(np.float64)).astype(np.float32))
