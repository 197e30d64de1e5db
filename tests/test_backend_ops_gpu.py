"""The rest of the Backend op set on the B200 against the reference's semantics, stated in numpy:
every op evaluated in f64 on the exactly widened inputs and rounded once to the output type
(CpuBackendImpl, packages/tensor-cpu/src/index.ts:318-735; unaryFlat, nn-kernels.ts:43-60;
sumAxis / extremumAxis / argExtremumAxis / cumsumAxis, kernels.ts:125-187, :543-592).

Exact ops (+, -, *, /, sqrt, maximum, neg, abs, relu, comparisons, where, copies, sums, extrema)
must match bit for bit; transcendental ops within one unit in the last place of the output type.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from tensor_cuda.backend import CudaBackend
    from tensor_cuda.runtime import Device
    return CudaBackend(Device.shared(0))


def bf16_round(x64):
    b = np.asarray(x64, np.float32).view(np.uint32).astype(np.uint64)  # f64 -> f32 first is exact enough here
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def up(be, arr, dtype):
    from tensor_cuda.backend import host
    return be.from_host_sync(host(dtype, arr.shape, arr))


def down(be, t):
    h = be.read_sync(t)
    d = h.data
    if h.dtype == "bf16":
        d = (d.astype(np.uint32) << 16).view(np.float32)
    return np.asarray(d).reshape(h.shape)


def ulps_f32(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


RNG = np.random.default_rng(42)


def data(shape, lo=-3, hi=3):
    return RNG.uniform(lo, hi, shape).astype(np.float32)


@pytest.mark.parametrize("name,fn,lo,exact", [
    ("neg", np.negative, -3, True), ("abs", np.abs, -3, True), ("relu", lambda x: np.where(x > 0, x, 0.0), -3, True),
    ("sqrt", np.sqrt, 0, True), ("exp", np.exp, -3, False), ("log", np.log, 0.01, False),
    ("rsqrt", lambda x: 1 / np.sqrt(x), 0.01, False), ("tanh", np.tanh, -3, False),
    ("sigmoid", lambda x: np.where(x >= 0, 1 / (1 + np.exp(-np.abs(x))), np.exp(-np.abs(x)) / (1 + np.exp(-np.abs(x)))),
     -5, False),
])
def test_unary_ops_f32(be, name, fn, lo, exact):
    x = data((7, 33), lo, 3)
    got = down(be, getattr(be, name)(up(be, x, "f32")))
    want = fn(x.astype(np.float64)).astype(np.float32)
    if exact:
        assert np.array_equal(got, want)
    else:
        assert ulps_f32(got, want).max() <= 1


def test_erf_scale_and_half_outputs(be):
    from scipy.special import erf
    x = data((5, 40))
    assert ulps_f32(down(be, be.erf(up(be, x, "f32"))), erf(x.astype(np.float64)).astype(np.float32)).max() <= 1
    assert np.array_equal(down(be, be.scale(up(be, x, "f32"), -0.375)), (x.astype(np.float64) * -0.375).astype(np.float32))
    # bf16 in -> bf16 out, rounded once from the f64 value
    xb = (bf16_round(x).astype(np.uint32) << 16).view(np.float32)
    got = down(be, be.sqrt(up(be, bf16_round(np.abs(x)), "bf16")))
    want = (bf16_round(np.sqrt(np.abs(xb).astype(np.float64))).astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("name,fn", [("sub", np.subtract), ("mul", np.multiply), ("div", np.divide),
                                     ("maximum", np.maximum)])
def test_binary_ops_broadcast_exact(be, name, fn):
    a = data((3, 1, 5))
    b = data((4, 1)) + 0.5
    a[0, 0, 0] = np.nan if name == "maximum" else a[0, 0, 0]
    got = down(be, getattr(be, name)(up(be, a, "f32"), up(be, b, "f32")))
    want = fn(a.astype(np.float64), b.astype(np.float64)).astype(np.float32)
    assert got.shape == (3, 4, 5)
    assert np.array_equal(got, want, equal_nan=True)


def test_pow_and_integer_arithmetic(be):
    a = data((6, 8), 0.1, 3)
    b = data((8,), -2, 2)
    got = down(be, be.pow(up(be, a, "f32"), up(be, b, "f32")))
    assert ulps_f32(got, np.power(a.astype(np.float64), b.astype(np.float64)).astype(np.float32)).max() <= 1
    i = RNG.integers(-1000, 1000, (4, 5)).astype(np.int32)
    j = RNG.integers(-1000, 1000, (5,)).astype(np.int32)
    for name, fn in (("sub", np.subtract), ("mul", np.multiply), ("maximum", np.maximum)):
        assert np.array_equal(down(be, getattr(be, name)(up(be, i, "i32"), up(be, j, "i32"))), fn(i, j))
    with pytest.raises(TypeError, match="no implicit promotion"):
        be.sub(up(be, a, "f32"), up(be, i, "i32"))


def test_comparisons_logical_and_where(be):
    a = np.round(data((4, 6)))
    b = np.round(data((6,)))
    A, B = up(be, a, "f32"), up(be, b, "f32")
    for name, fn in (("equal", np.equal), ("notEqual", np.not_equal), ("less", np.less),
                     ("lessEqual", np.less_equal), ("greater", np.greater), ("greaterEqual", np.greater_equal)):
        got = down(be, getattr(be, name)(A, B))
        assert got.dtype == np.uint8 and np.array_equal(got.astype(bool), fn(a, b)), name
    p, q = a > 0, b > 0
    P, Q = up(be, p, "bool"), up(be, q, "bool")
    assert np.array_equal(down(be, be.logicalAnd(P, Q)).astype(bool), p & q)
    assert np.array_equal(down(be, be.logicalOr(P, Q)).astype(bool), p | q)
    assert np.array_equal(down(be, be.logicalNot(P)).astype(bool), ~p)
    c = RNG.random((4, 1)) > 0.5
    got = down(be, be.where(up(be, c, "bool"), A, B))
    assert np.array_equal(got, np.where(c, a, b))


def test_reductions_follow_the_reference_order(be):
    x = data((3, 7, 5))
    x[0, 0, 1] = np.nan  # first in its lane: max / argmax keep it
    x[1, 3, 2] = np.nan  # later in its lane: ignored by the strict comparisons
    X = up(be, x, "f32")
    x64 = x.astype(np.float64)
    for axis in (0, 1, 2, -1):
        seq = np.cumsum(np.moveaxis(x64, axis, -1), axis=-1)[..., -1]  # sequential f64 sum
        assert np.array_equal(down(be, be.sum(X, axis)), seq.astype(np.float32), equal_nan=True)
        n = x.shape[axis]
        assert np.array_equal(down(be, be.mean(X, axis)), (seq / n).astype(np.float32), equal_nan=True)

        def sweep(v, want_max):
            best, bi = v[0], 0
            for j in range(1, len(v)):
                if (v[j] > best) if want_max else (v[j] < best):
                    best, bi = v[j], j
            return best, bi
        moved = np.moveaxis(x, axis, -1)
        flat = moved.reshape(-1, moved.shape[-1])
        for want_max, val_op, arg_op in ((True, be.max, be.argmax), (False, be.min, be.argmin)):
            ref = [sweep(r, want_max) for r in flat]
            vals = np.array([r[0] for r in ref], np.float32).reshape(moved.shape[:-1])
            idx = np.array([r[1] for r in ref], np.int32).reshape(moved.shape[:-1])
            assert np.array_equal(down(be, val_op(X, axis)), vals, equal_nan=True)
            assert np.array_equal(down(be, arg_op(X, axis)), idx)
    assert down(be, be.sum(X, 1, keepDims=True)).shape == (3, 1, 5)
    with pytest.raises(ValueError, match="empty axis"):
        be.max(up(be, np.zeros((2, 0), np.float32), "f32"), 1)
    i = RNG.integers(-5, 5, (4, 6)).astype(np.int32)
    assert np.array_equal(down(be, be.sum(up(be, i, "i32"), 1)), i.sum(1))
    assert np.array_equal(down(be, be.cumsum(up(be, i > 0, "bool"), 1)), np.cumsum(i > 0, 1).astype(np.int32))
    assert np.array_equal(down(be, be.cumsum(X, 2)), np.cumsum(x64, 2).astype(np.float32), equal_nan=True)


def test_slice_concat_split(be):
    x = data((5, 6, 7))
    X = up(be, x, "f32")
    assert np.array_equal(down(be, be.slice(X, [1, -4, 0], [4, 100, -2])), x[1:4, -4:, 0:-2])
    assert down(be, be.slice(X, [3], [1])).shape == (0, 6, 7)  # hi clamps to lo
    y = data((5, 2, 7))
    got = down(be, be.concat([X, up(be, y, "f32"), X], 1))
    assert np.array_equal(got, np.concatenate([x, y, x], 1))
    parts = be.split(X, 5, 0)
    assert np.array_equal(down(be, parts[2]), x[2:3])
