"""The row / element-wise ops of the path on the B200 vs the oracle (tensor-cpu semantics)."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from _helpers import NP_STORAGE, from_device_dtype, to_device_dtype

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    from tensor_cuda.runtime import Device
    return Device.shared(0)


def _call(name, *args):
    from tensor_cuda import _ffi as F
    F.call(name, *args)


def test_gelu_matches_reference_geluErf(dev):
    """Dense grid over [-12, 12] plus the reference test points (backend.test.ts:121-133): the device's
    f32 exact GELU against the oracle's f64 geluErf rounded once."""
    from tensor_cuda import _ffi as F
    x = np.concatenate([np.linspace(-12, 12, 200001), [-3, -0.5, 0, 1e-3, 0.7, 2.5]]).astype(np.float32)
    want = O.gelu(x).astype(np.float64)
    dx = dev.upload(x)
    dy = dev.alloc(x.nbytes)
    _call("mpc_gelu", dev.handle, C.c_void_p(dx.ptr), F.F32, C.c_void_p(dy.ptr), F.F32, x.size, None)
    got = dev.download(dy.ptr, dy.nbytes, np.float32, x.shape).astype(np.float64)
    err = np.abs(got - want)
    # 2e-6 relative where |GELU| is not tiny; 1e-6 absolute where the left tail underflows in f32
    assert np.all(err <= 2e-6 * np.abs(want) + 1e-6 * np.maximum(np.abs(x) * 0, 0) + 2e-7), err.max()
    core = np.abs(x) <= 6
    assert np.all(err[core] <= 2e-6 * np.abs(want[core]) + 1e-12), (err[core] / (np.abs(want[core]) + 1e-30)).max()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_softmax_last_and_middle_axis(dev, dtype):
    from tensor_cuda import _ffi as F
    for shape, axis in (((37, 1000), -1), ((3, 6, 5), 1), ((4, 7), -1), ((2, 3000, 3), 1)):
        x = O.lcg_seeded(int(np.prod(shape)), 77, -40, 40).astype(np.float32).reshape(shape)
        up, ex = to_device_dtype(x, dtype)
        want = O.softmax(ex, axis).astype(np.float64)
        ax = axis % len(shape)
        outer, dim, inner = int(np.prod(shape[:ax])), shape[ax], int(np.prod(shape[ax + 1:]))
        dx = dev.upload(up)
        dy = dev.alloc(x.size * 4)
        _call("mpc_softmax", dev.handle, C.c_void_p(dx.ptr), F.DTYPE_CODES[dtype], C.c_void_p(dy.ptr), outer, dim,
              inner, None)
        got = dev.download(dy.ptr, dy.nbytes, np.float32, shape).astype(np.float64)
        # differential.test.ts:23 TIGHT (1e-6) scaled by the row length for f32 sums
        assert np.all(np.abs(got - want) <= 1e-6 + 2e-6 * np.abs(want)), (shape, np.abs(got - want).max())


def test_add_bias_layernorm_embedding_cast(dev):
    from tensor_cuda import _ffi as F
    rows, d = 70, 768
    x = O.normal_f32(rows * d, 3, 0, 1).reshape(rows, d)
    b = O.normal_f32(d, 4, 0, 0.02)
    dx, db = dev.upload(x), dev.upload(b)
    dy = dev.alloc(x.nbytes)
    _call("mpc_add", dev.handle, C.c_void_p(dx.ptr), C.c_void_p(db.ptr), C.c_void_p(dy.ptr), F.F32, x.size, d, None)
    assert np.array_equal(dev.download(dy.ptr, dy.nbytes, np.float32, x.shape), O.add_f32(x, b))

    w = O.normal_f32(d, 5, 1, 0.1)
    _call("mpc_layer_norm", dev.handle, C.c_void_p(dx.ptr), F.F32, C.c_void_p(dev.upload(w).ptr), C.c_void_p(db.ptr),
          C.c_float(1e-5), C.c_void_p(dy.ptr), F.F32, rows, d, None)
    want = O.layer_norm(x, w, b, 1e-5)
    assert np.abs(dev.download(dy.ptr, dy.nbytes, np.float32, x.shape) - want).max() <= 1e-5

    table = O.normal_f32(11 * 6, 6, 0, 1).reshape(11, 6)
    ids = np.array([[3, 0, 10], [7, 7, 1]], np.int32)
    dt, di = dev.upload(table), dev.upload(ids)
    do = dev.alloc(ids.size * 6 * 4)
    bad = C.c_int64()
    _call("mpc_embedding", dev.handle, C.c_void_p(dt.ptr), F.F32, C.c_void_p(di.ptr), C.c_void_p(do.ptr), ids.size,
          11, 6, C.byref(bad), None)
    assert np.array_equal(dev.download(do.ptr, do.nbytes, np.float32, (2, 3, 6)), O.embedding(table, ids))
    bad_ids = dev.upload(np.array([0, 5, 11, -1], np.int32))
    with pytest.raises(F.MpcError, match="out of range"):
        _call("mpc_embedding", dev.handle, C.c_void_p(dt.ptr), F.F32, C.c_void_p(bad_ids.ptr), C.c_void_p(do.ptr), 4,
              11, 6, C.byref(bad), None)
    assert bad.value == 2

    for dto in ("f16", "bf16"):
        dc = dev.alloc(x.size * 2)
        _call("mpc_cast", dev.handle, C.c_void_p(dx.ptr), F.F32, C.c_void_p(dc.ptr), F.DTYPE_CODES[dto], x.size, None)
        got = from_device_dtype(dev.download(dc.ptr, dc.nbytes, NP_STORAGE[dto], x.shape), dto)
        assert np.array_equal(got, to_device_dtype(x, dto)[1]), dto


@pytest.mark.parametrize("dtype,rows,d", [("f32", 300, 768), ("bf16", 2049, 768), ("f16", 37, 96), ("f32", 70, 2048),
                                          ("bf16", 500, 4096), ("f16", 33, 8200), ("f32", 9, 5000),
                                          ("bf16", 3, 30)])
def test_layer_norm_paths(dev, dtype, rows, d):
    """Every LayerNorm path: one warp per row (short rows, with the next row loaded ahead), one
    256-thread block per row held in registers (long rows), and the general kernel (rows whose
    length is not a multiple of the 16-byte vector): layerNormRows (nn-kernels.ts:108-129), f32
    statistics, one rounding into the storage type."""
    from tensor_cuda import _ffi as F
    x = O.normal_f32(rows * d, 11, 0.5, 2).reshape(rows, d)
    w = O.normal_f32(d, 12, 1, 0.1)
    b = O.normal_f32(d, 13, 0, 0.1)
    xs, xv = to_device_dtype(x, dtype)
    dx = dev.upload(np.ascontiguousarray(xs))
    dy = dev.alloc(dx.nbytes)
    code = {"f32": F.F32, "f16": F.F16, "bf16": F.BF16}[dtype]
    dw, dbias = dev.upload(w), dev.upload(b)  # kept alive until the kernel has run
    _call("mpc_layer_norm", dev.handle, C.c_void_p(dx.ptr), code, C.c_void_p(dw.ptr), C.c_void_p(dbias.ptr),
          C.c_float(1e-5), C.c_void_p(dy.ptr), code, rows, d, None)
    got = from_device_dtype(dev.download(dy.ptr, dy.nbytes, NP_STORAGE[dtype], xs.shape), dtype).reshape(rows, d)
    want = O.layer_norm(xv, w, b, 1e-5)
    _, want_st = to_device_dtype(want, dtype)
    tol = {"f32": 2e-5, "f16": 2e-3, "bf16": 1.6e-2}[dtype]
    assert np.abs(got - want_st.reshape(rows, d)).max() <= tol * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_embedding_vector_rows(dev, dtype):
    """Rows of whole 16-byte vectors take the vector gather; an id out of range still reports its
    first position (takeRows, nn-kernels.ts:277-286)."""
    from tensor_cuda import _ffi as F
    V, D = 50, 64
    table = O.normal_f32(V * D, 21, 0, 1).reshape(V, D)
    up, ex = to_device_dtype(table, dtype)
    ids = np.array([[3, 0, 49, 7], [7, 7, 1, 12]], np.int32)
    dt, di = dev.upload(np.ascontiguousarray(up)), dev.upload(ids)
    code = {"f32": F.F32, "bf16": F.BF16}[dtype]
    eb = F.DTYPE_BYTES[code]
    do = dev.alloc(ids.size * D * eb)
    bad = C.c_int64()
    _call("mpc_embedding", dev.handle, C.c_void_p(dt.ptr), code, C.c_void_p(di.ptr), C.c_void_p(do.ptr), ids.size,
          V, D, C.byref(bad), None)
    got = from_device_dtype(dev.download(do.ptr, do.nbytes, NP_STORAGE[dtype], (ids.size * D,)), dtype)
    assert np.array_equal(got.reshape(ids.size, D), ex.reshape(V, D)[ids.reshape(-1)])
    ids_bad = np.array([1, 2, 50, 3, -1], np.int32)
    dib = dev.upload(ids_bad)
    rc = F.load().mpc_embedding(dev.handle, C.c_void_p(dt.ptr), code, C.c_void_p(dib.ptr), C.c_void_p(do.ptr),
                                ids_bad.size, V, D, C.byref(bad), None)
    assert rc == F.ERR_INVALID and bad.value == 2
