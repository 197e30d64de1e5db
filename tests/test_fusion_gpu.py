"""Element-wise fusion on the B200 against the oracle's restatement of tensor-compile's evaluator
(evalValue, packages/tensor-compile/src/ir.ts:339-383): the reference's cross-check cases
(packages/tensor-webgpu/test/fusion.test.ts:91-190: single unary ops, binary ops, a fused chain,
select, comparisons) on the same LCG inputs, JavaScript's special-value semantics, broadcasting,
half-precision inputs and a size past L2.

Both sides evaluate in f64 and round once to f32, so arithmetic, comparisons, selections and the
rounding ops agree bit for bit; where CUDA's f64 library and the C library differ in the last f64
place (transcendentals), the f32 results may differ by one unit in the last place."""
import numpy as np
import pytest

import oracle as O
from tensor_cuda.fusion import BINARY_OPS, CMP_OPS, Traced

pytestmark = pytest.mark.gpu

EXACT_UNARY = {"neg", "relu", "abs", "floor", "ceil", "round", "sign", "trunc", "sqrt"}


@pytest.fixture(scope="module")
def dev():
    from tensor_cuda.device import create_cuda_device
    return create_cuda_device(0)


def random_data(size, seed, scale=1.0):
    """fusion.test.ts:24-31."""
    s = seed & 0xFFFFFFFF
    out = np.empty(size, np.float64)
    for i in range(size):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = ((s / 0xFFFFFFFF) * 2 - 1) * scale
    return out.astype(np.float32)


def run(dev, node, *arrays, dtypes=None):
    ins = [dev.from_numpy(a, d) for a, d in zip(arrays, dtypes or [None] * len(arrays))]
    out = dev.fuse(node, ins)
    assert out.dtype == "f32"
    return dev.to_numpy(out)


def ulps(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    both_nan = np.isnan(a) & np.isnan(b)
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)  # monotone integer line through -0 / +0
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    d = np.abs(ia - ib)
    d[both_nan] = 0
    d[np.isnan(a) ^ np.isnan(b)] = 1 << 40
    return d


def same_bits(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a)
    return np.array_equal(nan, np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


UNARY_CASES = [  # fusion.test.ts:92-130: the op and its input domain
    ("neg", "x"), ("relu", "x"), ("sigmoid", "x"), ("gelu", "x"), ("gelu_tanh", "x"), ("exp", "x"), ("log", "pos"),
    ("sqrt", "pos"), ("sin", "x"), ("cos", "x"), ("tan", "x"), ("asin", "x"), ("acos", "x"), ("atan", "x"),
    ("sinh", "x"), ("cosh", "x"), ("tanh", "x"), ("abs", "x"), ("log2", "pos"), ("log10", "pos"), ("cbrt", "x"),
    ("floor", "x"), ("ceil", "x"), ("round", "x"), ("sign", "x"), ("trunc", "x"), ("expm1", "x"), ("log1p", "pos"),
    ("erf", "x"), ("asinh", "x"), ("acosh", "pos1"), ("atanh", "x"),
    # the reciprocal and inverse forms the reference's cross-check leaves to its CPU tests
    ("cot", "x"), ("sec", "x"), ("csc", "x"), ("coth", "x"), ("sech", "x"), ("csch", "x"), ("acot", "x"),
    ("asec", "big"), ("acsc", "big"), ("acoth", "big"), ("asech", "unit"), ("acsch", "x"),
]


@pytest.mark.parametrize("op,domain", UNARY_CASES)
def test_unary_ops(dev, op, domain):
    x = random_data(4096, 1, 0.8)
    data = {"x": x, "pos": np.abs(random_data(4096, 2, 0.8)) + 0.1, "pos1": np.abs(random_data(4096, 2, 0.8)) + 1.1,
            "big": np.abs(x) + 1.2, "unit": np.abs(x) * 0.9 + 0.05}[domain]
    node = {"kind": "unary", "op": op, "arg": {"kind": "input", "index": 0}}
    got, want = run(dev, node, data), O.eval_ir(node, [data])
    if op in EXACT_UNARY:
        assert same_bits(got, want), op
    else:
        assert ulps(got, want).max() <= 1, op
    # the reference's own cross-check bound (fusion.test.ts:78-85)
    assert np.all(np.abs(got - want) <= 1e-2 * np.maximum(1, np.abs(want)))


@pytest.mark.parametrize("op", BINARY_OPS)
def test_binary_ops(dev, op):
    a = random_data(4096, 3, 3)
    b = random_data(4096, 4, 3)
    b[b == 0] = 0.5
    if op == "pow":
        a, b = np.abs(random_data(4096, 5, 2)) + 0.1, random_data(4096, 6, 2)
    node = getattr(Traced.input(0), op)(Traced.input(1)).node
    got, want = run(dev, node, a, b), O.eval_ir(node, [a, b])
    if op in ("add", "sub", "mul", "div", "min", "max"):
        assert same_bits(got, want), op
    else:
        assert ulps(got, want).max() <= 1, op


def test_fused_chain_select_and_cmp(dev):
    a, b, c = random_data(256, 7, 2), random_data(256, 8, 2), random_data(256, 9, 2)
    chain = Traced.input(0).add(Traced.input(1)).mul(Traced.input(2)).sigmoid().relu()
    assert ulps(run(dev, chain, a, b, c), O.eval_ir(chain.node, [a, b, c])).max() <= 1
    cond, t, e = random_data(64, 10, 1), random_data(64, 11, 5), random_data(64, 12, 5)
    sel = Traced.input(0).select(Traced.input(1), Traced.input(2))
    assert same_bits(run(dev, sel, cond, t, e), O.eval_ir(sel.node, [cond, t, e]))
    # the untaken branch's domain error never shows (piecewise sqrt)
    pw = Traced.input(0).ge(0).select(Traced.input(0).sqrt(), Traced.input(0).neg())
    x = random_data(64, 13, 3)
    assert same_bits(run(dev, pw, x), np.where(x >= 0, np.sqrt(x.astype(np.float64)), -x).astype(np.float32))
    a, b = random_data(64, 13, 3), random_data(64, 14, 3)
    b[::7] = a[::7]  # some equal pairs
    for op in CMP_OPS:
        node = Traced.input(0).cmp(op, Traced.input(1)).node
        assert same_bits(run(dev, node, a, b), O.eval_ir(node, [a, b])), op


def test_javascript_special_values(dev):
    """Math.round / Math.sign / Math.pow / min / max / relu on NaN, infinities and signed zeros."""
    v = np.array([-2.5, -0.5, -0.2, 0.5, 2.5, np.nan, -0.0, 0.0, np.inf, -np.inf, 1.0, -1.0], np.float32)
    w = np.array([np.nan, np.inf, -np.inf, -2.0, 0.5, 1.0, -1.0, np.nan, 0.0, 3.0, np.inf, np.inf], np.float32)
    x, y = Traced.input(0), Traced.input(1)
    for t in (x.round(), x.sign(), x.relu(), x.abs(), x.floor(), x.trunc(), x.neg(), x.pow(y), x.min(y), x.max(y),
              x.hypot(y), x.atan2(y), x.eq(y), x.ne(y), x.select(y, x), x.div(y), x.sqrt()):
        got, want = run(dev, t, v, w), O.eval_ir(t.node, [v, w])
        assert same_bits(got, want), t.node


@pytest.mark.parametrize("shapes", [[(64, 300), (300,)], [(64, 300), (64, 1)], [(5, 1, 7), (1, 4, 1), (7,)],
                                    [(2, 3, 4, 5, 6, 7), (1, 3, 1, 5, 1, 7)], [(1000,), ()]])
def test_broadcasting(dev, shapes):
    rng = np.random.default_rng(len(shapes))
    arrays = [rng.standard_normal(s).astype(np.float32) for s in shapes]
    expr = Traced.input(0)
    for i in range(1, len(shapes)):
        expr = expr.mul(Traced.input(i)).add(0.5)
    expr = expr.tanh().add(Traced.input(0))
    got = run(dev, expr, *arrays)
    want = O.eval_ir(expr.node, arrays)
    assert got.shape == np.broadcast_shapes(*shapes)
    assert ulps(got, want).max() <= 1


def test_half_inputs_and_raw_tensors(dev):
    from _helpers import to_device_dtype
    x = random_data(5000, 15, 4)
    y = random_data(5000, 16, 4)
    (hx, vx), (hy, vy) = to_device_dtype(x, "bf16"), to_device_dtype(y, "f16")
    expr = Traced.input(0).mul(Traced.input(1)).gelu()
    got = run(dev, expr, hx, hy, dtypes=["bf16", "f16"])
    assert ulps(got, O.eval_ir(expr.node, [vx, vy])).max() <= 1
    # raw backend tensors in, a raw tensor out
    a = dev.from_numpy(x).handle
    out = dev.fuse(expr, [a, a])
    from tensor_cuda.backend import CudaTensor
    assert isinstance(out, CudaTensor) and tuple(out.shape) == (5000,)


def test_compile_and_errors(dev):
    f = dev.compile(2, lambda x, y: x.mul(y).add(1).gelu())
    a, b = random_data(1000, 17, 2), random_data(1000, 18, 2)
    got = dev.to_numpy(f(dev.from_numpy(a), dev.from_numpy(b)))
    assert ulps(got, O.eval_ir(Traced.input(0).mul(Traced.input(1)).add(1).gelu().node, [a, b])).max() <= 1
    with pytest.raises(ValueError, match="expects 2 input"):
        f(dev.from_numpy(a))
    with pytest.raises(ValueError, match="do not broadcast"):
        dev.fuse(Traced.input(0).add(Traced.input(1)), [dev.from_numpy(np.ones((3, 4), np.float32)),
                                                        dev.from_numpy(np.ones(5, np.float32))])
    with pytest.raises(TypeError, match="float inputs"):
        dev.fuse(Traced.input(0).neg(), [dev.from_numpy(np.ones(3, np.int32))])
    empty = dev.fuse(Traced.input(0).exp(), [dev.from_numpy(np.ones((0, 4), np.float32))])
    assert empty.shape == (0, 4)


def test_large_flat_and_strided(dev):
    """Past L2 (3 x 64 M f32 in, 64 M out): the flat kernel, then the strided one via a broadcast."""
    n = 1 << 26
    rng = np.random.default_rng(19)
    a = rng.standard_normal(n, dtype=np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    c = rng.standard_normal(n, dtype=np.float32)
    expr = Traced.input(0).mul(Traced.input(1)).add(Traced.input(2)).max(0)
    got = run(dev, expr, a, b, c)
    want = (a.astype(np.float64) * b + c).astype(np.float64)
    want = np.where(want >= 0, want, 0.0).astype(np.float32)
    assert same_bits(got, want)
    row = rng.standard_normal(8192, dtype=np.float32)
    got = run(dev, expr, a.reshape(-1, 8192), row, c.reshape(-1, 8192))
    want = (a.reshape(-1, 8192).astype(np.float64) * row + c.reshape(-1, 8192))
    assert same_bits(got, np.where(want >= 0, want, 0.0).astype(np.float32))


def test_unaligned_views_and_collapsed_axes(dev):
    """Views at 4-byte offsets take the one-element kernel; unit axes and axes every input steps
    across contiguously collapse before the launch (the result is the same)."""
    be = dev.backend
    x = np.arange(3 * 37, dtype=np.float32).reshape(3, 37) / 7
    parts = be.split(dev.from_numpy(x).handle, 3, 0)  # rows at byte offsets 0, 148, 296
    y = np.linspace(-1, 1, 37).astype(np.float32)
    expr = Traced.input(0).mul(Traced.input(1)).exp()
    for i, part in enumerate(parts):
        got = be.read_sync(dev.fuse(expr, [part, dev.from_numpy(y).handle])).data
        assert ulps(got, O.eval_ir(expr.node, [x[i], y])).max() <= 1
    a = np.random.default_rng(20).standard_normal((4, 1, 5, 6, 1)).astype(np.float32)
    b = np.random.default_rng(21).standard_normal((1, 1, 5, 6, 1)).astype(np.float32)
    c = np.random.default_rng(22).standard_normal((4, 1, 1, 1, 1)).astype(np.float32)
    expr = Traced.input(0).sub(Traced.input(1)).div(Traced.input(2))
    got = run(dev, expr, a, b, c)
    assert got.shape == (4, 1, 5, 6, 1) and same_bits(got, O.eval_ir(expr.node, [a, b, c]))


# ---- f32 evaluation (precision="f32": every intermediate an f32, as in the WebGPU backend's WGSL,
# packages/tensor-webgpu/src/fusion-wgsl.ts) ------------------------------------------------------

# CUDA's single-precision functions are within a few units in the last place of the correctly
# rounded result (the largest documented bound among those used, normcdff, is 5); composite
# formulas (sigmoid, gelu_tanh, the reciprocal and inverse forms) add a rounding or two.
F32_ULPS = 16


def run32(dev, node, *arrays, dtypes=None):
    ins = [dev.from_numpy(a, d) for a, d in zip(arrays, dtypes or [None] * len(arrays))]
    return dev.to_numpy(dev.fuse(node, ins, precision="f32"))


@pytest.mark.parametrize("op,domain", UNARY_CASES)
def test_unary_ops_f32(dev, op, domain):
    x = random_data(4096, 1, 0.8)
    data = {"x": x, "pos": np.abs(random_data(4096, 2, 0.8)) + 0.1, "pos1": np.abs(random_data(4096, 2, 0.8)) + 1.1,
            "big": np.abs(x) + 1.2, "unit": np.abs(x) * 0.9 + 0.05}[domain]
    node = {"kind": "unary", "op": op, "arg": {"kind": "input", "index": 0}}
    got, want = run32(dev, node, data), O.eval_ir(node, [data])
    if op in EXACT_UNARY:
        assert same_bits(got, want), op
    else:
        assert ulps(got, want).max() <= F32_ULPS, (op, int(ulps(got, want).max()))
    assert np.all(np.abs(got - want) <= 1e-2 * np.maximum(1, np.abs(want)))  # fusion.test.ts:78-85


@pytest.mark.parametrize("op", BINARY_OPS)
def test_binary_ops_f32(dev, op):
    a = random_data(4096, 3, 3)
    b = random_data(4096, 4, 3)
    b[b == 0] = 0.5
    if op == "pow":
        a, b = np.abs(random_data(4096, 5, 2)) + 0.1, random_data(4096, 6, 2)
    node = getattr(Traced.input(0), op)(Traced.input(1)).node
    got, want = run32(dev, node, a, b), O.eval_ir(node, [a, b])
    if op in ("add", "sub", "mul", "div", "min", "max"):
        assert same_bits(got, want), op
    else:
        assert ulps(got, want).max() <= F32_ULPS, (op, int(ulps(got, want).max()))


def test_f32_arithmetic_is_ieee_f32_step_by_step(dev):
    """A chain of +, -, *, / and max equals IEEE f32 arithmetic node by node (no contraction into
    fused multiply-adds), and differs from the f64 evaluation where an intermediate rounds."""
    x, y, z = Traced.input(0), Traced.input(1), Traced.input(2)
    a, b, c = random_data(5000, 23, 3), random_data(5000, 24, 3), random_data(5000, 25, 3)
    e = x.add(y).mul(z).sub(x).div(y.add(3.5)).max(x.mul(0.1)).add(z.mul(z).mul(1.0 / 3.0))
    assert same_bits(run32(dev, e, a, b, c), O.eval_ir(e.node, [a, b, c], precision="f32"))
    lost = x.add(1e-8).sub(x)
    v = np.array([1.0, 3.0, -2.0, 0.75], np.float32)
    assert run32(dev, lost, v).tolist() == [0.0, 0.0, 0.0, 0.0]
    assert np.allclose(run(dev, lost, v), 1e-8, rtol=1e-6)


def test_f32_special_values_and_half_inputs(dev):
    v = np.array([-2.5, -0.5, -0.2, 0.5, 2.5, np.nan, -0.0, 0.0, np.inf, -np.inf, 1.0, -1.0], np.float32)
    w = np.array([np.nan, np.inf, -np.inf, -2.0, 0.5, 1.0, -1.0, np.nan, 0.0, 3.0, np.inf, np.inf], np.float32)
    x, y = Traced.input(0), Traced.input(1)
    for t in (x.round(), x.sign(), x.relu(), x.abs(), x.floor(), x.trunc(), x.neg(), x.min(y), x.max(y), x.eq(y),
              x.ne(y), x.select(y, x), x.div(y), x.sqrt()):
        assert same_bits(run32(dev, t, v, w), O.eval_ir(t.node, [v, w])), t.node
    for t in (x.pow(y), x.hypot(y), x.atan2(y)):  # NaN / infinity cases exact, finite results within bounds
        assert ulps(run32(dev, t, v, w), O.eval_ir(t.node, [v, w])).max() <= F32_ULPS, t.node
    from _helpers import to_device_dtype
    (hx, vx), (hy, vy) = to_device_dtype(random_data(5000, 15, 4), "bf16"), to_device_dtype(random_data(5000, 16, 4), "f16")
    expr = x.mul(y).gelu()
    assert ulps(run32(dev, expr, hx, hy, dtypes=["bf16", "f16"]), O.eval_ir(expr.node, [vx, vy])).max() <= F32_ULPS
    # x * y + 1 cancels where x * y is near -1: its f32 rounding is part of the f32 evaluation, so a
    # composite expression is checked against the oracle's f32 evaluation (every node rounded)
    f = dev.compile(2, lambda p, q: p.mul(q).add(1).gelu(), precision="f32")
    a, b = random_data(1000, 17, 2), random_data(1000, 18, 2)
    got = dev.to_numpy(f(dev.from_numpy(a), dev.from_numpy(b)))
    assert ulps(got, O.eval_ir(x.mul(y).add(1).gelu().node, [a, b], precision="f32")).max() <= F32_ULPS
