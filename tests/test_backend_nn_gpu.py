"""sort, gatherRows, rope, geglu and meanPool on the B200 against the oracle's restatements of the
reference's kernels (sortAxis, takeRows, ropeHalf, gegluRows, maskedMeanPool;
packages/tensor-cpu/src/index.ts:724-861), on the reference's differential cases
(tensor-cpu/test/differential.test.ts:109-160, from the golden fixture) and on wider sizes.

sort, gatherRows and meanPool must match bit for bit; rope and geglu (cos / sin / Φ in f64 from
CUDA's library against the oracle's) within one unit in the last place of f32."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from tensor_cuda.backend import CudaBackend
    from tensor_cuda.runtime import Device
    return CudaBackend(Device.shared(0))


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


def same_bits(a, b):
    """Equal, NaN matching NaN and -0 distinct from +0."""
    a, b = np.asarray(a), np.asarray(b)
    if a.dtype.kind == "f":
        a32, b32 = a.astype(np.float32), b.astype(np.float32)
        nan = np.isnan(a32)
        return np.array_equal(nan, np.isnan(b32)) and np.array_equal(a32[~nan].view(np.uint32), b32[~nan].view(np.uint32))
    return np.array_equal(a, b)


def fixture_inputs(fx, name):
    gen, shapes, ranks = fx[name + "_gen"], fx[name + "_shapes"], fx[name + "_ranks"]
    shp = tuple(int(d) for d in shapes[0][: ranks[0]])
    s, lo, hi = gen[0]
    return O.lcg_seeded(int(np.prod(shp)), int(s), lo, hi).astype(np.float32).reshape(shp)


@pytest.fixture(scope="module")
def fx(golden_dir):
    import os
    with np.load(os.path.join(golden_dir, "differential_cpu.npz")) as f:
        return {k: f[k] for k in f.files}


# ---- the reference's own cases -------------------------------------------------------------------

def test_reference_backend_cases(be):
    """backend.test.ts:91-92 (sort axis 0), :108 (gatherRows error), :163 / :167 (meanPool, gatherRows)."""
    s = be.sort(up(be, np.array([[3, 1], [-1, -5]], np.float32), "f32"), 0)
    assert down(be, s).reshape(-1).tolist() == [-1, -5, 3, 1]
    x = up(be, np.arange(1, 7, dtype=np.float32).reshape(1, 2, 3), "f32")
    with pytest.raises(IndexError, match="index -3 out of range for length 2"):
        be.gatherRows(x, up(be, np.array([[-3]], np.int32), "i32"))
    x = up(be, np.arange(1, 7, dtype=np.float32).reshape(1, 3, 2), "f32")
    g = be.gatherRows(x, up(be, np.array([[-1, 0]], np.int32), "i32"))
    assert down(be, g).tolist() == [[[5, 6], [1, 2]]]
    m = be.meanPool(x, up(be, np.array([[1, 0, 1]], np.uint8), "bool"))
    assert down(be, m).tolist() == [[3, 4]]


@pytest.mark.parametrize("name", ["rope_base10000_1x3x17x16", "rope_base160000_2x2x70x32", "geglu_3x5x24",
                                  "mean_pool_3x7x5", "sort_axis0_5x3", "gather_rows_2x7x3_idx2x4"])
def test_differential_cases(be, fx, name):
    x = fixture_inputs(fx, name)
    want = fx[name + "_out"]  # the reference's numpy oracle
    xd = up(be, x, "f32")
    if name.startswith("rope"):
        base = float(fx[name + "_base"][0])
        got, ora = down(be, be.rope(xd, base)), O.rope(x, base)
    elif name.startswith("geglu"):
        got, ora = down(be, be.geglu(xd)), O.geglu(x)
    elif name.startswith("mean_pool"):
        mask = fx[name + "_mask"]
        got, ora = down(be, be.meanPool(xd, up(be, mask.astype(np.uint8), "bool"))), O.mean_pool(x, mask)
    elif name.startswith("sort"):
        got, ora = down(be, be.sort(xd, 0)), O.sort_axis(x, 0)
    else:
        idx = fx[name + "_idx"]
        got, ora = down(be, be.gatherRows(xd, up(be, idx, "i32"))), O.gather_rows(x, idx)
    assert got.shape == want.shape
    assert np.all(np.abs(got - want) <= 1e-5 + 1e-5 * np.abs(want)), name
    if name.startswith(("rope", "geglu")):
        assert ulps_f32(got, ora).max() <= 1, name
    else:
        assert same_bits(got, ora), name


# ---- sort ----------------------------------------------------------------------------------------

def special_values(n, rng):
    x = rng.standard_normal(n).astype(np.float32) * 10
    pick = rng.integers(0, 10, n)
    x[pick == 0] = np.nan
    x[pick == 1] = 0.0
    x[pick == 2] = -0.0
    x[pick == 3] = np.inf
    x[pick == 4] = -np.inf
    x[pick == 5] = np.round(x[pick == 5])  # duplicates
    return x


@pytest.mark.parametrize("shape,axis", [
    ((7,), 0), ((300, 5), 1), ((5, 300), 0), ((4, 1000, 3), 1), ((3, 4096), -1), ((2, 5000), 1),
    ((3, 70001), 1), ((20000, 2), 1), ((1, 1), 0), ((6, 1, 2), 1)])
def test_sort_f32_special_values(be, shape, axis):
    rng = np.random.default_rng(sum(shape))
    x = special_values(int(np.prod(shape)), rng).reshape(shape)
    got = down(be, be.sort(up(be, x, "f32"), axis))
    assert same_bits(got, O.sort_axis(x, axis))


@pytest.mark.parametrize("dtype", ["f16", "bf16", "i32", "bool"])
@pytest.mark.parametrize("shape,axis", [((33, 257), 1), ((9000, 3), 0)])
def test_sort_other_dtypes(be, dtype, shape, axis):
    rng = np.random.default_rng(5)
    n = int(np.prod(shape))
    if dtype == "i32":
        x = rng.integers(-2 ** 31, 2 ** 31, n, dtype=np.int64).astype(np.int32).reshape(shape)
        x.reshape(-1)[:4] = [2 ** 31 - 1, -2 ** 31, 0, 2 ** 31 - 1]
        got, want = down(be, be.sort(up(be, x, "i32"), axis)), np.sort(x, axis=axis)
        assert np.array_equal(got, want)
        return
    if dtype == "bool":
        x = rng.integers(0, 2, n).astype(np.uint8).reshape(shape)
        got, want = down(be, be.sort(up(be, x, "bool"), axis)), np.sort(x, axis=axis)
        assert np.array_equal(got, want)
        return
    x = special_values(n, rng).reshape(shape)
    if dtype == "f16":
        x16 = x.astype(np.float16)
        got = np.asarray(be.read_sync(be.sort(up(be, x16, "f16"), axis)).data).reshape(shape)
        assert same_bits(got.astype(np.float32), O.sort_axis(x16.astype(np.float32), axis))
    else:
        from _helpers import bf16_bits_to_f32, f32_to_bf16_bits
        bits = f32_to_bf16_bits(np.nan_to_num(x, nan=0.0, posinf=np.inf, neginf=-np.inf)).reshape(shape)
        bits[np.isnan(x)] = 0x7FC0
        xv = bf16_bits_to_f32(bits).reshape(shape)
        got = down(be, be.sort(up(be, bits.reshape(shape), "bf16"), axis))
        assert same_bits(got, O.sort_axis(xv, axis))


# ---- gatherRows ----------------------------------------------------------------------------------

@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16", "i32"])
def test_gather_rows(be, dtype):
    rng = np.random.default_rng(7)
    B, L, M, D = 3, 50, 77, 130
    x = rng.standard_normal((B, L, D)).astype(np.float32)
    if dtype == "i32":
        x = rng.integers(-1000, 1000, (B, L, D)).astype(np.int32)
    idx = rng.integers(-L, L, (B, M)).astype(np.int32)
    dev = be.gatherRows(up(be, x, dtype), up(be, idx, "i32"))
    got = np.asarray(be.read_sync(dev).data).reshape(B, M, D)
    want_src = np.asarray(be.read_sync(up(be, x, dtype)).data).reshape(B, L, D)
    assert np.array_equal(got, O.gather_rows(want_src, idx))


def test_gather_rows_errors_and_empty(be):
    x = up(be, np.zeros((2, 4, 3), np.float32), "f32")
    with pytest.raises(IndexError, match="index 4 out of range for length 4"):
        be.gatherRows(x, up(be, np.array([[0, 1], [3, 4]], np.int32), "i32"))
    with pytest.raises(IndexError, match="index -5 out of range for length 4"):
        be.gatherRows(up(be, np.zeros((2, 4, 0), np.float32), "f32"), up(be, np.array([[0], [-5]], np.int32), "i32"))
    e = be.gatherRows(up(be, np.zeros((2, 4, 0), np.float32), "f32"), up(be, np.array([[0], [-4]], np.int32), "i32"))
    assert tuple(e.shape) == (2, 1, 0)
    with pytest.raises(ValueError):
        be.gatherRows(x, up(be, np.zeros((3, 1), np.int32), "i32"))


# ---- rope ----------------------------------------------------------------------------------------

@pytest.mark.parametrize("shape,base", [((2, 12, 1024, 64), 10000.0), ((1, 3, 5, 128), 500000.0), ((3, 1, 2000, 2), 10.0)])
def test_rope_f32(be, shape, base):
    x = np.random.default_rng(11).standard_normal(shape).astype(np.float32)
    got = down(be, be.rope(up(be, x, "f32"), base))
    assert ulps_f32(got, O.rope(x, base)).max() <= 1


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_rope_half_storage(be, dtype):
    from _helpers import from_device_dtype, to_device_dtype
    x = np.random.default_rng(12).standard_normal((2, 4, 256, 64)).astype(np.float32)
    arr, xv = to_device_dtype(x, dtype)
    got = from_device_dtype(be.read_sync(be.rope(up(be, arr, dtype), 10000.0)).data, dtype).reshape(x.shape)
    _, want = to_device_dtype(O.rope(xv, 10000.0), dtype)
    # the device rounds the f64 rotation once into the half type, the oracle to f32 first: at
    # most one unit in the last place of the half type apart
    tol = {"bf16": 2 ** -7, "f16": 2 ** -10}[dtype]
    assert np.all(np.abs(got - want) <= tol * np.abs(want) + 1e-30)
    with pytest.raises(ValueError, match="even head dim"):
        be.rope(up(be, np.zeros((1, 1, 2, 3), np.float32), "f32"))


# ---- geglu / meanPool ----------------------------------------------------------------------------

@pytest.mark.parametrize("shape", [(4096, 2 * 1536), (3, 5, 24), (7, 2)])
def test_geglu_f32(be, shape):
    x = np.random.default_rng(13).uniform(-8, 8, shape).astype(np.float32)
    got = down(be, be.geglu(up(be, x, "f32")))
    assert got.shape == shape[:-1] + (shape[-1] // 2,)
    assert ulps_f32(got, O.geglu(x)).max() <= 1


@pytest.mark.parametrize("mask_dtype", ["bool", "f32", "i32"])
def test_mean_pool(be, mask_dtype):
    rng = np.random.default_rng(14)
    B, L, D = 5, 300, 768
    x = rng.standard_normal((B, L, D)).astype(np.float32)
    m = (rng.uniform(0, 1, (B, L)) < 0.6).astype(np.float32)
    m[2] = 0  # a row with nothing kept gives 0
    if mask_dtype == "f32":
        m = m * rng.uniform(0.5, 2, (B, L)).astype(np.float32)
        m[0, :5] = np.nan  # NaN is falsy in the reference's test
    md = up(be, m if mask_dtype == "f32" else m.astype(np.int32 if mask_dtype == "i32" else np.uint8), mask_dtype)
    got = down(be, be.meanPool(up(be, x, "f32"), md))
    want = O.mean_pool(x, m)
    assert same_bits(got, want)
    assert not got[2].any()
