"""The allocation-free f32 GEMM entry point (mpc_gemm_f32_noalloc) against mpc_gemm and the oracle.

mpc_gemm_f32_noalloc is for callers that cannot allocate device memory (a host runtime that owns
every device byte or hands the library a fixed budget): its scratch is a static device array
instead of the allocator. The tests call it through the C ABI, twice in a row with different
shapes, and hold each result to mpc_gemm's result for the same inputs and to the oracle's f64
product, within the f32 GEMM bound used by the other tests
(packages/tensor-webgpu/test/gemm.test.ts:125: 1e-5·(|A||B|) + 1e-7); further cases cover a
broadcast batch axis, the bias + GELU epilogue and K = 0; the device's free memory and the
library's allocator are unchanged across calls; a bounded wait that runs out is reported by
mpc_gemm_f32_noalloc_status. This file sorts last so a run that stops at the first failure has run
every other test first.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    from tensor_cuda.runtime import Device
    return Device.shared(0)


def _noalloc(desc, a_ptr, b_ptr, c_ptr, bias_ptr, stream):
    from tensor_cuda import _ffi as F
    F.call("mpc_gemm_f32_noalloc", C.byref(desc), C.c_void_p(a_ptr), C.c_void_p(b_ptr), C.c_void_p(c_ptr),
           C.c_void_p(bias_ptr) if bias_ptr else None, C.c_void_p(stream))


def _gemm_both(dev, a, b, m, n, k, b_layout, batch=None, epi=0, bias=None):
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import gemm_desc
    nb = 1 if batch is None else batch[0]
    da, db = dev.upload(a), dev.upload(b)
    dbias = dev.upload(bias) if bias is not None else None
    c_ref, c_new = dev.alloc(nb * m * n * 4), dev.alloc(nb * m * n * 4)
    kw = {} if batch is None else dict(batch_shape=(nb,), a_batch_strides=(batch[1],), b_batch_strides=(batch[2],))
    desc = gemm_desc(m, n, k, F.F32, F.F32, b_layout, epi, **kw)
    dev.gemm(desc, da.ptr, db.ptr, c_ref.ptr, dbias.ptr if dbias else None)
    dev.sync()
    _noalloc(desc, da.ptr, db.ptr, c_new.ptr, dbias.ptr if dbias else None, dev.stream)
    dev.sync()
    assert F.load().mpc_gemm_f32_noalloc_status(C.c_void_p(dev.stream)) == F.OK, F.last_error()
    shape = (m, n) if batch is None else (nb, m, n)
    ref = dev.download(c_ref.ptr, c_ref.nbytes, np.float32, shape).astype(np.float64)
    got = dev.download(c_new.ptr, c_new.nbytes, np.float32, shape).astype(np.float64)
    return ref, got


def test_noalloc_matches_mpc_gemm_and_the_oracle_on_two_calls_in_a_row(dev):
    from tensor_cuda import _ffi as F
    # call 1: a linear-layout product whose N (130) needs the padded C copy in the static scratch
    m, k, n = 300, 268, 130
    a = O.lcg_gemm(m * k, 11).reshape(m, k)
    b = O.lcg_gemm(n * k, 12).reshape(n, k)
    ref, got = _gemm_both(dev, a, b, m, n, k, F.B_NK)
    absprod = O.matmul(np.abs(a), np.ascontiguousarray(np.abs(b).T)).astype(np.float64)
    want = O.linear(a, b).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-5 * absprod + 1e-7)
    assert np.all(np.abs(got - want) <= 1e-5 * absprod + 1e-7)
    # call 2: the f32 configuration's 1024^3 matmul layout, reusing the same static scratch
    m = k = n = 1024
    a = O.uniform_f32(m * k, 1, -1, 1).reshape(m, k)
    b = O.uniform_f32(k * n, 2, -1, 1).reshape(k, n)
    ref, got = _gemm_both(dev, a, b, m, n, k, F.B_KN)
    absprod = O.matmul(np.abs(a), np.abs(b), threads=O.default_threads()).astype(np.float64)
    want = O.matmul(a, b, threads=O.default_threads()).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-5 * absprod + 1e-7)
    assert np.all(np.abs(got - want) <= 1e-5 * absprod + 1e-7)
    assert np.abs(got - want).max() / np.abs(want).max() <= 1e-5


def test_noalloc_broadcast_batch_bias_gelu_and_k0(dev):
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import gemm_desc
    # three products sharing one B (batch stride 0), + bias, exact GELU
    nb, m, k, n = 3, 200, 96, 136
    a = O.lcg_gemm(nb * m * k, 21).reshape(nb, m, k)
    b = O.lcg_gemm(k * n, 22).reshape(k, n)
    bias = O.lcg_seeded(n, 23, -0.5, 0.5).astype(np.float32)
    ref, got = _gemm_both(dev, a, b, m, n, k, F.B_KN, batch=(nb, m * k, 0), epi=F.EPI_BIAS | F.EPI_GELU, bias=bias)
    want = np.stack([O.gelu(O.add_f32(O.matmul(a[i], b), bias)) for i in range(nb)]).astype(np.float64)
    absprod = np.stack([O.matmul(np.abs(a[i]), np.abs(b)) for i in range(nb)]).astype(np.float64)
    # GELU' is at most 1.13 in magnitude, so the product's bound carries over, plus the f32 GELU rounding
    tol = 1.2e-5 * absprod + 2e-6 * np.abs(want) + 1e-6
    assert np.all(np.abs(got - ref) <= tol)
    assert np.all(np.abs(got - want) <= tol)
    # K = 0: C = GELU(0 + bias)
    m, n = 5, 7
    bias = O.lcg_seeded(n, 24, -1, 1).astype(np.float32)
    dbias, c = dev.upload(bias), dev.alloc(m * n * 4)
    one = dev.alloc(16)
    desc = gemm_desc(m, n, 0, F.F32, F.F32, F.B_KN, F.EPI_BIAS | F.EPI_GELU)
    _noalloc(desc, one.ptr, one.ptr, c.ptr, dbias.ptr, dev.stream)
    dev.sync()
    got = dev.download(c.ptr, c.nbytes, np.float32, (m, n)).astype(np.float64)
    want = np.broadcast_to(O.gelu(bias.reshape(1, n)), (m, n)).astype(np.float64)
    assert np.all(np.abs(got - want) <= 2e-6 * np.abs(want) + 1e-7)


def test_noalloc_allocates_nothing(dev):
    """After a warm-up call (which loads the kernels' code), further calls leave the device's free
    memory and the library's allocator exactly as they were."""
    import torch

    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import gemm_desc
    m, k, n = 512, 384, 260
    da = dev.upload(O.lcg_gemm(m * k, 31).reshape(m, k))
    db = dev.upload(O.lcg_gemm(k * n, 32).reshape(k, n))
    c = dev.alloc(m * n * 4)
    desc = gemm_desc(m, n, k, F.F32, F.F32, F.B_KN)
    _noalloc(desc, da.ptr, db.ptr, c.ptr, None, dev.stream)
    dev.sync()
    free0, _ = torch.cuda.mem_get_info(0)
    stats0 = dev.alloc_stats()
    for _ in range(3):
        _noalloc(desc, da.ptr, db.ptr, c.ptr, None, dev.stream)
    dev.sync()
    assert torch.cuda.mem_get_info(0)[0] == free0
    assert dev.alloc_stats() == stats0


def test_noalloc_reports_a_wait_that_ran_out(dev):
    """A bounded wait in the entry point's error record (the self test: an mbarrier nothing
    releases, 20 ms) is reported once by mpc_gemm_f32_noalloc_status and then cleared; a GEMM
    afterwards is correct and reports nothing."""
    from tensor_cuda import _ffi as F
    lib = F.load()
    assert lib.mpc_gemm_f32_noalloc_status(C.c_void_p(dev.stream)) == F.OK
    assert lib.mpc_gemm_f32_noalloc_selftest(C.c_uint64(20_000_000), C.c_void_p(dev.stream)) == F.OK
    assert lib.mpc_gemm_f32_noalloc_status(C.c_void_p(dev.stream)) == F.ERR_TIMEOUT
    assert "ran out" in F.last_error()
    assert lib.mpc_gemm_f32_noalloc_status(C.c_void_p(dev.stream)) == F.OK  # cleared by the query
    m, k, n = 128, 64, 96
    a = O.lcg_gemm(m * k, 41).reshape(m, k)
    b = O.lcg_gemm(k * n, 42).reshape(k, n)
    ref, got = _gemm_both(dev, a, b, m, n, k, F.B_KN)
    assert np.all(np.abs(got - ref) <= 1e-5 * O.matmul(np.abs(a), np.abs(b)).astype(np.float64) + 1e-7)


def test_noalloc_rejects_requests_beyond_its_static_scratch(dev):
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import gemm_desc
    desc = gemm_desc(2048, 2048, 2048, F.F32, F.F32, F.B_KN)  # 64 MiB of tf32 planes > 32 MiB
    one = dev.alloc(16)
    rc = F.load().mpc_gemm_f32_noalloc(C.byref(desc), C.c_void_p(one.ptr), C.c_void_p(one.ptr),
                                       C.c_void_p(one.ptr), None, C.c_void_p(dev.stream))
    assert rc == F.ERR_INVALID
    assert "static maximum" in F.last_error()
    bad = gemm_desc(4, 4, 4, F.BF16, F.F32, F.B_KN)
    assert F.load().mpc_gemm_f32_noalloc(C.byref(bad), C.c_void_p(one.ptr), C.c_void_p(one.ptr),
                                         C.c_void_p(one.ptr), None, None) == F.ERR_INVALID
