"""GEMM parity on the B200: mpc_gemm (through the C ABI) vs the CPU oracle's Tensor.matmul /
linearNT restatement on the same inputs.

Shapes are the reference's own GEMM test set (packages/tensor-webgpu/test/gemm.test.ts:147-163)
with its LCG inputs (:85-93) and seeds (:109-112), in every input dtype and both B layouts, plus
the fused bias + GELU epilogue, broadcast batches and the large batched configuration.
"""
import numpy as np
import pytest

import oracle as O
from _helpers import NP_STORAGE, from_device_dtype, gemm_bound, to_device_dtype

pytestmark = pytest.mark.gpu

SHAPES = [
    (4, 3, 5, False), (17, 33, 9, False), (128, 128, 128, False), (1, 64, 256, False), (37, 70, 45, True),
    (1, 1024, 300, True), (33, 256, 100, True), (50, 128, 96, True), (65, 64, 64, True), (93, 256, 200, True),
    (300, 268, 130, True), (130, 256, 200, False), (257, 100, 132, False), (130, 256, 202, False),
    (256, 512, 256, False),
]


@pytest.fixture(scope="module")
def dev():
    from tensor_cuda.runtime import Device
    return Device.shared(0)


def run_gemm(dev, a, b, dtype_in, dtype_out, b_layout, m, n, k, bias=None, epilogue=0, alpha=1.0,
             batch_shape=(), a_strides=(), b_strides=()):
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import gemm_desc
    da, db = dev.upload(a), dev.upload(b)
    nb = int(np.prod(batch_shape)) if batch_shape else 1
    out_elems = nb * m * n
    dc = dev.alloc(out_elems * F.DTYPE_BYTES[F.DTYPE_CODES[dtype_out]])
    dbias = dev.upload(np.ascontiguousarray(bias, np.float32)) if bias is not None else None
    desc = gemm_desc(m, n, k, F.DTYPE_CODES[dtype_in], F.DTYPE_CODES[dtype_out], b_layout, epilogue, alpha,
                     batch_shape, a_strides, b_strides)
    dev.gemm(desc, da.ptr, db.ptr, dc.ptr, dbias.ptr if dbias is not None else None)
    dev.sync()
    raw = dev.download(dc.ptr, dc.nbytes, NP_STORAGE[dtype_out], (out_elems,))
    return from_device_dtype(raw, dtype_out)


@pytest.mark.parametrize("dtype_in", ["f32", "f16", "bf16"])
def test_gemm_reference_shapes(dev, dtype_in):
    from tensor_cuda import _ffi as F
    for (m, k, n, trans_b) in SHAPES:
        seed = m * 7919 + k * 104729 + n * 1299709 + (17 if trans_b else 0)
        a32 = O.lcg_gemm(m * k, seed).reshape(m, k)
        b32 = O.lcg_gemm(k * n, seed + 1).reshape((n, k) if trans_b else (k, n))
        a_up, a_ex = to_device_dtype(a32, dtype_in)
        b_up, b_ex = to_device_dtype(b32, dtype_in)
        bkn = b_ex.T if trans_b else b_ex
        want = O.matmul(a_ex, np.ascontiguousarray(bkn)).astype(np.float64)
        absprod = O.matmul(np.abs(a_ex), np.ascontiguousarray(np.abs(bkn))).astype(np.float64)
        for dtype_out in ("f32", dtype_in):
            got = run_gemm(dev, a_up, b_up, dtype_in, dtype_out, F.B_NK if trans_b else F.B_KN, m, n, k)
            got = got.reshape(m, n).astype(np.float64)
            bound = gemm_bound(want, absprod, dtype_in, dtype_out)
            bad = np.argwhere(~(np.abs(got - want) <= bound))
            assert bad.size == 0, (f"{dtype_in}->{dtype_out} {m}x{k}x{n} {'T' if trans_b else 'N'}: "
                                   f"{len(bad)} bad, first {tuple(bad[0])}: got {got[tuple(bad[0])]} "
                                   f"want {want[tuple(bad[0])]}")


def test_gemm_f32_1024_cube_3xtf32(dev):
    """The f32 configuration: A, B uniform[-1,1) (PCG32 uniformSample, seeds 1 and 2), 1024^3,
    held to the reference's f32 bound and to max|C-R|/max|R| <= 1e-5."""
    from tensor_cuda import _ffi as F
    n = 1024
    a = O.uniform_f32(n * n, 1, -1, 1).reshape(n, n)
    b = O.uniform_f32(n * n, 2, -1, 1).reshape(n, n)
    got = run_gemm(dev, a, b, "f32", "f32", F.B_KN, n, n, n).reshape(n, n).astype(np.float64)
    want = O.matmul(a, b, threads=O.default_threads()).astype(np.float64)
    absprod = O.matmul(np.abs(a), np.abs(b), threads=O.default_threads()).astype(np.float64)
    assert np.all(np.abs(got - want) <= 1e-5 * absprod + 1e-7)
    assert np.abs(got - want).max() / np.abs(want).max() <= 1e-5


@pytest.mark.parametrize("dtype_in,b_layout", [("bf16", "kn"), ("f16", "nk"), ("f32", "kn")])
def test_gemm_bias_gelu_epilogue(dev, dtype_in, b_layout):
    """matmul -> add(bias) -> gelu fused (the DeviceArray chain x.matmul(w).add(b).gelu()), alpha."""
    from tensor_cuda import _ffi as F
    m, k, n = 300, 192, 264
    a32 = O.normal_f32(m * k, 11, 0, 1 / np.sqrt(k)).reshape(m, k)
    b32 = O.normal_f32(k * n, 12, 0, 1 / np.sqrt(k)).reshape((k, n) if b_layout == "kn" else (n, k))
    bias = O.normal_f32(n, 13, 0, 0.02)
    a_up, a_ex = to_device_dtype(a32, dtype_in)
    b_up, b_ex = to_device_dtype(b32, dtype_in)
    bkn = b_ex if b_layout == "kn" else b_ex.T
    for alpha in (1.0, 0.5):
        mm = O.matmul(a_ex, np.ascontiguousarray(bkn))
        want = O.gelu(O.add_f32(mm * np.float32(alpha), bias)).astype(np.float64)
        got = run_gemm(dev, a_up, b_up, dtype_in, "f32", F.B_KN if b_layout == "kn" else F.B_NK, m, n, k, bias,
                       F.EPI_BIAS | F.EPI_GELU, alpha).reshape(m, n)
        err = np.abs(got - want)
        if dtype_in == "f32":
            assert np.all(err <= 1e-5 * (1 + np.abs(want))), (alpha, err.max())
        else:
            assert np.all(err <= 2e-3 + 1e-2 * np.abs(want)), (dtype_in, alpha, err.max())


def test_gemm_broadcast_batches(dev):
    """[2,1,5,7] @ [3,7,6] (differential.test.ts:100): batch axes broadcast on both sides."""
    from tensor_cuda import _ffi as F
    a = O.lcg_seeded(70, 101).astype(np.float32).reshape(2, 1, 5, 7)
    b = O.lcg_seeded(126, 102).astype(np.float32).reshape(3, 7, 6)
    want = O.matmul(a, b)
    for dtype in ("f32", "bf16"):
        a_up, a_ex = to_device_dtype(a, dtype)
        b_up, b_ex = to_device_dtype(b, dtype)
        want = O.matmul(a_ex, b_ex).astype(np.float64)
        got = run_gemm(dev, a_up, b_up, dtype, "f32", F.B_KN, 5, 6, 7, batch_shape=(2, 3),
                       a_strides=(35, 0), b_strides=(0, 42)).reshape(2, 3, 5, 6)
        absprod = O.matmul(np.abs(a_ex), np.abs(b_ex)).astype(np.float64)
        assert np.all(np.abs(got - want) <= gemm_bound(want, absprod, dtype, "f32")), dtype


def test_gemm_large_batched_bf16_bias_gelu(dev):
    """The batched configuration's shape (2048^3 per batch, bf16 -> f32, +bias, GELU) on 2 batches,
    checked on 96 sampled rows per batch: <= 1e-2 relative / 2e-3 absolute."""
    from tensor_cuda import _ffi as F
    nb, n = 2, 2048
    a_bits = O.normal_half_bits(nb * n * n, 21, 0, 1 / np.sqrt(n), True).reshape(nb, n, n)
    b_bits = O.normal_half_bits(nb * n * n, 22, 0, 1 / np.sqrt(n), True).reshape(nb, n, n)
    bias = O.normal_f32(n, 23, 0, 0.02)
    got = run_gemm(dev, a_bits, b_bits, "bf16", "f32", F.B_KN, n, n, n, bias, F.EPI_BIAS | F.EPI_GELU, 1.0,
                   (nb,), (n * n,), (n * n,)).reshape(nb, n, n)
    rows = np.random.default_rng(5).choice(n, 96, replace=False)
    for bi in range(nb):
        a = O.half_bits_to_f32(a_bits[bi, rows], True)
        b = O.half_bits_to_f32(b_bits[bi], True)
        want = O.gelu(O.add_f32(O.matmul(a, b, threads=O.default_threads()), bias)).astype(np.float64)
        g = got[bi, rows].astype(np.float64)
        assert np.all(np.abs(g - want) <= 2e-3 + 1e-2 * np.abs(want)), bi


def test_gemm_k_zero_and_empty(dev):
    from tensor_cuda import _ffi as F
    bias = np.arange(5, dtype=np.float32)
    got = run_gemm(dev, np.zeros((3, 0), np.float32), np.zeros((0, 5), np.float32), "f32", "f32", F.B_KN, 3, 5, 0,
                   bias, F.EPI_BIAS)
    assert np.array_equal(got.reshape(3, 5), np.tile(bias, (3, 1)))


@pytest.mark.parametrize("dtype_in,dtype_out,n,in_place", [("bf16", "bf16", 264, False), ("bf16", "bf16", 100, False),
                                                            ("f16", "f32", 264, True), ("bf16", "bf16", 264, True),
                                                            ("f32", "f32", 72, False)])
def test_gemm_residual_epilogue(dev, dtype_in, dtype_out, n, in_place):
    """C = A·Wᵀ + bias + R (the transformer residual) in the epilogue: against the oracle's
    linear + add with the device rounding once; R may be C itself; unaligned rows (n=100 bf16)
    take the scalar path."""
    import ctypes as C
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import gemm_desc
    m, k = 200, 96
    a_up, a_ex = to_device_dtype(O.lcg_gemm(m * k, 31).reshape(m, k), dtype_in)
    w_up, w_ex = to_device_dtype(O.lcg_gemm(n * k, 32).reshape(n, k), dtype_in)
    bias = O.normal_f32(n, 33, 0, 0.5)
    r_up, r_ex = to_device_dtype(O.lcg_gemm(m * n, 34).reshape(m, n), dtype_out)
    da, dw, dbias, dr = dev.upload(a_up), dev.upload(w_up), dev.upload(bias), dev.upload(r_up)
    dc = dr if in_place else dev.alloc(m * n * F.DTYPE_BYTES[F.DTYPE_CODES[dtype_out]])
    desc = gemm_desc(m, n, k, F.DTYPE_CODES[dtype_in], F.DTYPE_CODES[dtype_out], F.B_NK, F.EPI_BIAS | F.EPI_RESIDUAL)
    F.call("mpc_gemm_residual", dev.handle, C.byref(desc), C.c_void_p(da.ptr), C.c_void_p(dw.ptr),
           C.c_void_p(dc.ptr), C.c_void_p(dbias.ptr), C.c_void_p(dr.ptr), None)
    dev.sync()
    got = from_device_dtype(dev.download(dc.ptr, m * n * F.DTYPE_BYTES[F.DTYPE_CODES[dtype_out]],
                                         NP_STORAGE[dtype_out], (m, n)), dtype_out).astype(np.float64)
    want = O.linear(a_ex, w_ex, bias).astype(np.float64) + r_ex.astype(np.float64)
    absprod = O.matmul(np.abs(a_ex), np.ascontiguousarray(np.abs(w_ex).T)).astype(np.float64)
    assert np.all(np.abs(got - want) <= gemm_bound(want, absprod + np.abs(r_ex), dtype_in, dtype_out))
    with pytest.raises(F.MpcError, match="mpc_gemm_residual"):
        dev.gemm(desc, da.ptr, dw.ptr, dc.ptr, dbias.ptr)


@pytest.mark.parametrize("dtype_out,n", [("bf16", 1001), ("f32", 999), ("f16", 50257 // 7)])
def test_gemm_unaligned_rows_batched(dev, dtype_out, n):
    """Outputs whose rows are not 16-byte aligned (the GPT-2 LM head's case) are written by the
    epilogue with plain stores: batched, with bias + GELU and row / column tails."""
    from tensor_cuda import _ffi as F
    bsz, m, k = 3, 150, 64
    a_up, a_ex = to_device_dtype(O.lcg_gemm(bsz * m * k, 41).reshape(bsz, m, k), "bf16")
    w_up, w_ex = to_device_dtype(O.lcg_gemm(n * k, 42).reshape(n, k), "bf16")
    bias = O.normal_f32(n, 43, 0, 0.5)
    got = run_gemm(dev, a_up, w_up, "bf16", dtype_out, F.B_NK, m, n, k, bias, F.EPI_BIAS | F.EPI_GELU,
                   batch_shape=(bsz,), a_strides=(m * k,), b_strides=(0,))
    got = got.reshape(bsz, m, n).astype(np.float64)
    want = np.stack([O.gelu(O.add_f32(O.linear(a_ex[i], w_ex), bias)) for i in range(bsz)]).astype(np.float64)
    tol = {"f32": 2e-3, "f16": 4e-3, "bf16": 2e-2}[dtype_out]
    assert np.all(np.abs(got - want) <= tol * (1 + np.abs(want)))
    # the same products through the aligned path (N padded to 16 bytes, TMA stores): every element
    # has the same K order, so the plain stores must give identical bits, rows of both parities
    npad = -(-n * (4 if dtype_out == "f32" else 2) // 16) * 16 // (4 if dtype_out == "f32" else 2)
    w_pad = np.zeros((npad, k), w_up.dtype)
    w_pad[:n] = w_up
    ref = run_gemm(dev, a_up, w_pad, "bf16", dtype_out, F.B_NK, m, npad, k, np.pad(bias, (0, npad - n)),
                   F.EPI_BIAS | F.EPI_GELU, batch_shape=(bsz,), a_strides=(m * k,), b_strides=(0,))
    assert np.array_equal(got, ref.reshape(bsz, m, npad)[:, :, :n].astype(np.float64))


@pytest.mark.parametrize("b_layout,dtype_in,dtype_out,epi,n,m,b_shared", [
    ("nk", "bf16", "f32", "", 2200, 2200, False),
    ("kn", "f16", "f32", "bias+gelu", 2200, 2200, False),
    ("nk", "bf16", "bf16", "bias+residual", 2200, 2200, False),
    ("kn", "bf16", "bf16", "", 2201, 2200, False),   # rows not 16-byte aligned: plain stores
    ("nk", "bf16", "bf16", "bias", 2100, 2100, True),  # the odd CTA's last rows and B half past M, N
    ("kn", "bf16", "f32", "bias+gelu", 2100, 2100, True),
])
def test_gemm_cta_pair_tiles(dev, b_layout, dtype_in, dtype_out, epi, n, m, b_shared):
    """Problems with at least one 256 x 256 tile per resident CTA pair run on pairs of SMs (M = 256
    tensor-core instructions, half of B per SM): batched (B per batch entry or one B broadcast),
    with row, column and K tails (K = 200; M, N = 2100 leave the odd CTA of the last pair tiles
    no valid row or column), both B layouts, every epilogue and unaligned output rows, against
    the oracle."""
    import ctypes as C
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import gemm_desc
    bsz, k = 2, 200
    lay = F.B_NK if b_layout == "nk" else F.B_KN
    a_up, a_ex = to_device_dtype(O.lcg_gemm(bsz * m * k, 51).reshape(bsz, m, k), dtype_in)
    b_shape = (n, k) if b_layout == "nk" else (k, n)
    nb = 1 if b_shared else bsz
    b_up, b_ex = to_device_dtype(O.lcg_gemm(nb * n * k, 52).reshape((nb,) + b_shape), dtype_in)
    bias = O.normal_f32(n, 53, 0, 0.5)
    flags = (F.EPI_BIAS if "bias" in epi else 0) | (F.EPI_GELU if "gelu" in epi else 0)
    eo = F.DTYPE_BYTES[F.DTYPE_CODES[dtype_out]]
    desc = gemm_desc(m, n, k, F.DTYPE_CODES[dtype_in], F.DTYPE_CODES[dtype_out], lay,
                     flags | (F.EPI_RESIDUAL if "residual" in epi else 0), 1.0, (bsz,), (m * k,),
                     (0 if b_shared else n * k,))
    da, db, dbias = dev.upload(a_up), dev.upload(b_up), dev.upload(bias)
    dc = dev.alloc(bsz * m * n * eo)
    r_ex = None
    if "residual" in epi:
        r_up, r_ex = to_device_dtype(O.lcg_gemm(bsz * m * n, 54).reshape(bsz, m, n), dtype_out)
        dr = dev.upload(r_up)
        F.call("mpc_gemm_residual", dev.handle, C.byref(desc), C.c_void_p(da.ptr), C.c_void_p(db.ptr),
               C.c_void_p(dc.ptr), C.c_void_p(dbias.ptr), C.c_void_p(dr.ptr), None)
    else:
        dev.gemm(desc, da.ptr, db.ptr, dc.ptr, dbias.ptr if flags else None)
    dev.sync()
    got = from_device_dtype(dev.download(dc.ptr, bsz * m * n * eo, NP_STORAGE[dtype_out], (bsz * m * n,)),
                            dtype_out).reshape(bsz, m, n).astype(np.float64)
    for i in range(bsz):
        bi = b_ex[0 if b_shared else i]
        bt = bi.T if b_layout == "nk" else bi
        prod = a_ex[i].astype(np.float64) @ bt.astype(np.float64)
        absprod = np.abs(a_ex[i]).astype(np.float64) @ np.abs(bt).astype(np.float64)
        want = prod
        if "bias" in epi:
            want = want + bias
        if "gelu" in epi:
            want = O.gelu(want.astype(np.float32)).astype(np.float64)
            absprod = absprod + np.abs(bias)
        if r_ex is not None:
            want = want + r_ex[i]
            absprod = absprod + np.abs(r_ex[i]) + np.abs(bias)
        bound = gemm_bound(want, absprod, dtype_in, dtype_out) + (1e-5 * (1 + np.abs(want)) if "gelu" in epi else 0)
        assert np.all(np.abs(got[i] - want) <= bound), i

