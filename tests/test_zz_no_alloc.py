"""The allocation-free f32 GEMM entry point (mpc_gemm_f32_noalloc) against mpc_gemm.

mpc_gemm_f32_noalloc is for callers that cannot allocate device memory (graph capture, runtimes
that own all device memory): its scratch is a static device array instead of the allocator. The
test calls it twice in a row through the C ABI, with different shapes, and holds each result to
mpc_gemm's result for the same inputs within the f32 GEMM bound used by the other tests
(packages/tensor-webgpu/test/gemm.test.ts:125: 1e-5·(|A||B|) + 1e-7). This file sorts last so a
run that stops at the first failure has run every other test first.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _gemm_both(dev, a, b, m, n, k, b_layout):
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import gemm_desc
    da, db = dev.upload(a), dev.upload(b)
    c_ref, c_new = dev.alloc(m * n * 4), dev.alloc(m * n * 4)
    desc = gemm_desc(m, n, k, F.F32, F.F32, b_layout)
    dev.gemm(desc, da.ptr, db.ptr, c_ref.ptr)
    dev.sync()
    F.call("mpc_gemm_f32_noalloc", C.byref(desc), C.c_void_p(da.ptr), C.c_void_p(db.ptr), C.c_void_p(c_new.ptr),
           None, C.c_void_p(dev.stream))
    dev.sync()
    ref = dev.download(c_ref.ptr, c_ref.nbytes, np.float32, (m, n)).astype(np.float64)
    got = dev.download(c_new.ptr, c_new.nbytes, np.float32, (m, n)).astype(np.float64)
    return ref, got


def test_noalloc_matches_mpc_gemm_on_two_calls_in_a_row():
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import Device
    dev = Device.shared(0)
    # call 1: a linear-layout product whose N (130) needs the padded C copy in the static scratch
    m, k, n = 300, 268, 130
    a = O.lcg_gemm(m * k, 11).reshape(m, k)
    b = O.lcg_gemm(n * k, 12).reshape(n, k)
    ref, got = _gemm_both(dev, a, b, m, n, k, F.B_NK)
    absprod = O.matmul(np.abs(a), np.ascontiguousarray(np.abs(b).T)).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-5 * absprod + 1e-7)
    # call 2: the f32 configuration's 1024^3 matmul layout, reusing the same static scratch
    m = k = n = 1024
    a = O.uniform_f32(m * k, 1, -1, 1).reshape(m, k)
    b = O.uniform_f32(k * n, 2, -1, 1).reshape(k, n)
    ref, got = _gemm_both(dev, a, b, m, n, k, F.B_KN)
    absprod = O.matmul(np.abs(a), np.abs(b), threads=O.default_threads()).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-5 * absprod + 1e-7)


def test_noalloc_rejects_requests_beyond_its_static_scratch():
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import Device, gemm_desc
    dev = Device.shared(0)
    desc = gemm_desc(2048, 2048, 2048, F.F32, F.F32, F.B_KN)  # 64 MiB of tf32 planes > 32 MiB
    one = dev.alloc(16)
    rc = F.load().mpc_gemm_f32_noalloc(C.byref(desc), C.c_void_p(one.ptr), C.c_void_p(one.ptr),
                                       C.c_void_p(one.ptr), None, C.c_void_p(dev.stream))
    assert rc == F.ERR_INVALID
    assert "static maximum" in F.last_error()
    bad = gemm_desc(4, 4, 4, F.BF16, F.F32, F.B_KN)
    assert F.load().mpc_gemm_f32_noalloc(C.byref(bad), C.c_void_p(one.ptr), C.c_void_p(one.ptr),
                                         C.c_void_p(one.ptr), None, None) == F.ERR_INVALID
