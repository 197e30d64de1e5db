"""The chainable device-array API on the B200, mirroring the reference's shared DeviceArray suite
(packages/tensor-cpu/test/device-array-suite.ts) for the ops on the GEMM / attention path:
differential cases in f32 / f16 / bf16 (f16 within 2e-2 and bf16 within 5e-2 on inputs rounded to
them, :8-17; ACCUM 1e-5 for f32 contractions) and the behavioural rules (sync validation errors,
no implicit transfers or promotion, scope / dispose lifetime, lazy-inside / eager-observable)."""
import asyncio

import numpy as np
import pytest

import oracle as O
from _helpers import to_device_dtype

pytestmark = pytest.mark.gpu

TOL = {"f32": (1e-5, 1e-5), "f16": (2e-2, 2e-2), "bf16": (5e-2, 5e-2)}


@pytest.fixture(scope="module")
def dev():
    from tensor_cuda import create_cuda_device
    return create_cuda_device(0)


def run(coro):
    return asyncio.run(coro)


def up(dev, x, dtype):
    arr, exact = to_device_dtype(x, dtype)
    return dev.from_numpy(arr if dtype != "f32" else exact, dtype if dtype == "bf16" else None), exact


def close(got, want, dtype):
    atol, rtol = TOL[dtype]
    assert got.shape == want.shape
    assert np.all(np.abs(got - want) <= atol + rtol * np.abs(want)), np.abs(got - want).max()


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_matmul_softmax_gelu_layernorm_cases(dev, dtype):
    g = lambda shape, s, lo=-1, hi=1: O.lcg_seeded(int(np.prod(shape)), s, lo, hi).astype(np.float32).reshape(shape)
    # device-array-suite.ts:175-176
    for sa, sb in (((4, 8), (8, 5)), ((2, 3, 4), (4, 5))):
        a, ea = up(dev, g(sa, 1), dtype)
        b, eb = up(dev, g(sb, 2), dtype)
        got = run(a.matmul(b).toTensor()).astype(np.float64)
        close(got, O.matmul(ea, eb).astype(np.float64), dtype)
    # :172-173 softmax axis -1 and 0
    for shape, axis in (((3, 7), -1), ((5, 2), 0)):
        x, ex = up(dev, g(shape, 3, -6, 6), dtype)
        close(run(x.softmax(axis).toTensor()).astype(np.float64), O.softmax(ex, axis).astype(np.float64), dtype)
    # gelu (exact erf) on [-4, 4]
    x, ex = up(dev, g((4, 6), 4, -4, 4), dtype)
    close(run(x.gelu().toTensor()).astype(np.float64), O.gelu(ex).astype(np.float64), dtype)
    # layerNorm weight + bias, and no affine
    x, ex = up(dev, g((3, 16), 5), dtype)
    w, ew = up(dev, g((16,), 6), dtype)
    b, eb = up(dev, g((16,), 7), dtype)
    close(run(x.layerNorm(w, b, 1e-5).toTensor()).astype(np.float64), O.layer_norm(ex, ew, eb, 1e-5), dtype)
    x, ex = up(dev, g((2, 2, 8), 8), dtype)
    close(run(x.layerNorm(None, None, 1e-6).toTensor()).astype(np.float64), O.layer_norm(ex, None, None, 1e-6), dtype)


def test_transfers_roundtrip_and_validation(dev):
    x = np.arange(12, dtype=np.float32).reshape(3, 4)
    a = run(dev.fromTensor(x))
    assert a.shape == (3, 4) and a.dtype == "f32"
    assert np.array_equal(run(a.toTensor()), x)
    h = run(a.toHost())
    assert h.dtype == "f32" and h.shape == (3, 4)
    # sync validation before any coroutine (host.ts:58-97): non-contiguous and unsupported dtypes
    with pytest.raises(ValueError, match="C-contiguous"):
        dev.fromTensor(x.T)
    with pytest.raises(TypeError, match="unsupported dtype"):
        dev.fromTensor(x.astype(np.float64))
    # bool normalised to 0/1, f16 exact, bf16 bits round trip
    from tensor_cuda import host
    m = run(dev.fromHost(host("bool", [3], np.array([0, 7, 255], np.uint8))))
    assert run(m.toHost()).data.tolist() == [0, 1, 1]
    f16 = run(dev.fromHost(host("f16", [3], [1.5, -2, 0.0999755859375])))
    assert run(f16.toTensor()).astype(np.float64).tolist() == [1.5, -2, 0.0999755859375]
    bf = run(dev.fromHost(host("bf16", [2], [1.5, -3])))
    assert run(bf.toTensor()).tolist() == [1.5, -3.0]


def test_no_implicit_transfers_or_promotion(dev):
    a = dev.from_numpy(np.ones((2, 2), np.float32))
    b = dev.from_numpy(np.ones((2, 2), np.float16))
    with pytest.raises(TypeError, match="no implicit transfers"):
        a.matmul(np.ones((2, 2), np.float32))
    with pytest.raises(TypeError, match="no implicit promotion"):
        a.matmul(b)
    with pytest.raises(TypeError, match="no implicit promotion"):
        a.add(b)
    with pytest.raises(ValueError, match="inner dimensions"):
        a.matmul(dev.from_numpy(np.ones((3, 2), np.float32)))
    i = dev.from_numpy(np.ones((2, 2), np.int32))
    with pytest.raises(TypeError, match="float"):
        i.gelu()


def test_scope_frees_what_it_does_not_return_and_dispose_is_idempotent(dev):
    x = dev.from_numpy(np.ones((4, 4), np.float32))
    inner = []

    def body():
        t = x.gelu()
        inner.append(t)
        return {"y": t.add(x), "n": 3}

    out = dev.scope(body)
    assert inner[0].disposed and not out["y"].disposed and not x.disposed
    with pytest.raises(RuntimeError, match="after dispose"):
        inner[0].gelu()
    with pytest.raises(ValueError):
        dev.scope(lambda: (x.gelu(), (_ for _ in ()).throw(ValueError("boom"))))
    x.dispose()
    x.dispose()
    with pytest.raises(RuntimeError, match="after dispose"):
        x.gelu()


def test_matmul_add_gelu_chain_runs_as_one_fused_kernel(dev):
    """Lazy inside: x.matmul(w).add(b).gelu() folds into one GEMM launch with the bias + GELU
    epilogue; values appear at toTensor (eager-observable)."""
    m, k, n = 96, 64, 72
    g = lambda shape, s: O.normal_f32(int(np.prod(shape)), s, 0, 0.2).reshape(shape)
    x, ex = up(dev, g((m, k), 1), "bf16")
    w, ew = up(dev, g((k, n), 2), "bf16")
    b, eb = up(dev, g((n,), 3), "bf16")
    before = dev.device.launch_count()
    y = x.matmul(w).add(b).gelu()
    assert dev.device.launch_count() == before  # nothing has run yet
    got = run(y.toTensor()).astype(np.float64)
    # the bias row is cast to f32 for the epilogue (1 launch) and the GEMM runs once (1 launch)
    assert dev.device.launch_count() - before == 2
    want = O.gelu(O.add_f32(O.matmul(ex, ew), eb)).astype(np.float64)
    close(got, want, "bf16")
    # disposing the operands before the pending GEMM runs does not free memory it reads
    x2, _ = up(dev, g((m, k), 4), "f32")
    w2, _ = up(dev, g((k, n), 5), "f32")
    y2 = x2.matmul(w2)
    x2.dispose()
    w2.dispose()
    assert run(y2.toTensor()).shape == (m, n)


def test_resident_chain_matmul_then_linear(dev):
    """gemm.test.ts:292-341: A·B stays on the device and feeds linear (x·Wᵀ); the second hop is
    checked on the device's own intermediate."""
    m, k, n, p = 96, 64, 72, 40
    for dtype in ("f32", "f16"):
        a, ea = up(dev, O.lcg_gemm(m * k, 7).reshape(m, k), dtype)
        b, eb = up(dev, O.lcg_gemm(k * n, 8).reshape(k, n), dtype)
        wt, ewt = up(dev, O.lcg_gemm(p * n, 9).reshape(p, n), dtype)
        ab = a.matmul(b)
        abw = dev.wrap(dev.backend.linear(ab.handle, wt.handle))
        assert abw.shape == (m, p) and abw.dtype == dtype
        ab_host = run(ab.toTensor()).astype(np.float32)
        close(ab_host.astype(np.float64), O.matmul(ea, eb).astype(np.float64), dtype)
        want2 = O.linear(ab_host, ewt).astype(np.float64)
        close(run(abw.toTensor()).astype(np.float64), want2, dtype)


def test_backend_sdpa_and_embedding(dev):
    B, H, L, D = 1, 2, 16, 64
    q, k, v = (O.normal_f32(B * H * L * D, s).reshape(B, H, L, D) for s in (1, 2, 3))
    bq, bk, bv = (dev.from_numpy(t) for t in (q, k, v))
    out = dev.wrap(dev.backend.sdpa(bq.handle, bk.handle, bv.handle, None, 0.125))
    want = O.sdpa(q, k, v, None, 0.125)
    assert np.all(np.abs(run(out.toTensor()) - want) <= 1e-5 + 1e-5 * np.abs(want))
    table = dev.from_numpy(O.normal_f32(11 * 6, 4).reshape(11, 6))
    ids = dev.from_numpy(np.array([[3, 0, 10]], np.int32))
    emb = dev.wrap(dev.backend.embedding(table.handle, ids.handle))
    assert emb.shape == (1, 3, 6)
    with pytest.raises(IndexError, match="out of range"):
        dev.backend.embedding(table.handle, dev.from_numpy(np.array([0, 5, 11], np.int32)).handle)


def test_transpose_like_numpy(dev):
    """device-array-suite.ts:178-179: transpose [2,3,4] -> [2,0,1] and the default reversal, every dtype."""
    x = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    for dtype, arr in (("f32", x), ("f16", x.astype(np.float16)), ("i32", x.astype(np.int32))):
        a = dev.from_numpy(arr)
        assert np.array_equal(run(a.transpose([2, 0, 1]).toTensor()), np.transpose(arr, [2, 0, 1])), dtype
        assert np.array_equal(run(a.transpose().toTensor()), np.transpose(arr)), dtype
    big = O.normal_f32(4 * 64 * 3 * 12 * 64, 3).reshape(4, 64, 3, 12, 64)  # a QKV head split
    got = run(dev.from_numpy(big).transpose([2, 0, 3, 1, 4]).toTensor())
    assert np.array_equal(got, np.transpose(big, [2, 0, 3, 1, 4]))
    with pytest.raises(ValueError, match="permutation"):
        dev.from_numpy(x).transpose([0, 0, 1])


def test_residual_add_folds_into_the_gemm(dev):
    """h.add(x.matmul(w)) and x.matmul(w).add(h): one GEMM launch with the residual in its
    epilogue; values as the oracle's matmul + add."""
    m, k, n = 96, 64, 80
    g = lambda shape, s: O.normal_f32(int(np.prod(shape)), s, 0, 0.3).reshape(shape)
    x, ex = up(dev, g((m, k), 1), "bf16")
    w, ew = up(dev, g((k, n), 2), "bf16")
    h, eh = up(dev, g((m, n), 3), "bf16")
    want = O.add_f32(O.matmul(ex, ew), eh).astype(np.float64)
    for expr in (lambda: h.add(x.matmul(w)), lambda: x.matmul(w).add(h)):
        before = dev.device.launch_count()
        y = expr()
        y.eval()
        assert dev.device.launch_count() - before == 1
        close(run(y.toTensor()).astype(np.float64), want, "bf16")


def test_elementwise_reduction_and_scalar_operands(dev):
    """device-array-suite.ts-style cases of the wider op set: number operands become constants of
    the array's dtype, minimum is -maximum(-a, -b), reductions with no axis cover every element,
    the dtype rules raise before any launch."""
    x = np.array([[1.5, -2.0, 3.0], [0.5, 4.0, -1.0]], np.float32)
    a = dev.from_numpy(x)
    assert np.array_equal(run(a.mul(2).sub(1).toTensor()), x * 2 - 1)
    assert np.array_equal(run(a.minimum(dev.from_numpy(np.zeros(3, np.float32))).toTensor()), np.minimum(x, 0))
    assert run(a.sum().toTensor()).item() == np.float32(x.astype(np.float64).sum())
    assert run(a.max(keepDims=True).toTensor()).shape == (1, 1)
    assert run(a.argmax(1).toTensor()).tolist() == [2, 1]
    assert run(a.cumsum().toTensor()).tolist() == np.cumsum(x.reshape(-1).astype(np.float64)).astype(np.float32).tolist()
    gt = a.greater(0)
    assert run(gt.toTensor()).tolist() == (x > 0).tolist()
    w = dev.where(gt, a, a.neg())
    assert np.array_equal(run(w.toTensor()), np.abs(x))
    assert run(gt.logicalNot().logicalAnd(gt).toTensor()).tolist() == [[False] * 3] * 2
    with pytest.raises(TypeError, match="needs a float dtype"):
        dev.from_numpy(np.ones((2,), np.int32)).exp()
    with pytest.raises(TypeError, match="cast\\(\"bool\"\\) first"):
        a.logicalNot()
    with pytest.raises(TypeError, match="not defined for bool"):
        gt.sum()


def test_gemm_capabilities_record():
    """gemmCapabilities (packages/tensor-webgpu/src/gemm-caps.ts:60-86): what the GEMM and attention
    use on this device."""
    from tensor_cuda.caps import gemm_capabilities
    from tensor_cuda.device import create_cuda_device
    cdev = create_cuda_device(0)
    caps = gemm_capabilities(cdev)
    assert caps.f16 and caps.bf16 and caps.f32_3xtf32 and caps.cta_pairs
    assert caps.sm_count == cdev.info["sm_count"] and caps.pair_min_tiles == caps.sm_count // 2
    assert caps.attention_head_dims == (64, 128) and caps.attention_max_head_dim == 256
    assert caps.max_dim == 1 << 30
