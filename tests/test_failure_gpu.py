"""Failure detection on the B200, without faulting, trapping or hanging the GPU.

* an allocation failure injected with the allocator cap: MPC_ERR_OOM, the device stays usable;
* a bounded in-kernel wait that nothing releases (mpc_selftest_wait_timeout): the kernel gives
  up after its limit and returns, the host reads MPC_ERR_TIMEOUT, the handle stays sticky until
  mpc_device_clear_error, and the same context then runs a GEMM correctly (the wasm backend's
  trap-poisoning rule, packages/tensor-wasm/src/index.ts:291-340, with an explicit reset);
* invalid shapes and strides rejected before any launch;
* a rank that never joins the communicator (one GPU; rank 1 is a process that never calls init):
  rank 0's init gives up after its limit with MPC_ERR_TIMEOUT, the half-built communicator is
  aborted on the host, and the device stays usable;
* two ranks (skipped on one GPU): one rank never enters a peer barrier; the other's barrier
  kernel gives up after the short wait limit and its next synchronisation reports MPC_ERR_TIMEOUT.
"""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
from _helpers import gemm_bound

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def dev():
    from tensor_cuda.runtime import Device
    return Device.shared(0)


def test_allocator_cap_injects_oom_and_the_device_stays_usable(dev):
    from tensor_cuda import _ffi as F
    in_use, _ = dev.alloc_stats()
    F.call("mpc_set_alloc_limit", dev.handle, in_use + (4 << 20))
    try:
        ok = dev.alloc(1 << 20)
        with pytest.raises(F.MpcError) as e:
            dev.alloc(64 << 20)
        assert e.value.status == F.ERR_OOM and "allocator cap" in str(e.value)
        ok.free()
    finally:
        F.call("mpc_set_alloc_limit", dev.handle, 0)
    assert dev.status() == F.OK
    dev.alloc(64 << 20).free()


def test_bounded_wait_times_out_and_the_context_recovers(dev):
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import gemm_desc
    rc = F.load().mpc_selftest_wait_timeout(C.c_void_p(dev.handle), C.c_uint64(50_000_000))  # 50 ms
    assert rc == F.ERR_TIMEOUT, F.last_error()
    assert dev.status() == F.ERR_TIMEOUT  # sticky until cleared
    F.call("mpc_device_clear_error", dev.handle)
    assert dev.status() == F.OK
    m = n = k = 128
    a = O.lcg_gemm(m * k, 5).reshape(m, k)
    b = O.lcg_gemm(k * n, 6).reshape(k, n)
    da, db, dc = dev.upload(a), dev.upload(b), dev.alloc(m * n * 4)
    dev.gemm(gemm_desc(m, n, k, F.F32, F.F32), da.ptr, db.ptr, dc.ptr)
    dev.sync()
    got = dev.download(dc.ptr, m * n * 4, np.float32, (m, n)).astype(np.float64)
    want = O.matmul(a, b).astype(np.float64)
    assert np.all(np.abs(got - want) <= gemm_bound(want, O.matmul(np.abs(a), np.abs(b)), "f32", "f32"))


def test_invalid_shapes_and_strides_are_rejected_before_launch(dev):
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import gemm_desc, sdpa_desc
    before = dev.launch_count()
    buf = dev.alloc(1 << 16)
    with pytest.raises(F.MpcError, match="negative dimension"):
        dev.gemm(gemm_desc(-1, 4, 4, F.BF16, F.F32), buf.ptr, buf.ptr, buf.ptr)
    with pytest.raises(F.MpcError, match="whole matrices"):
        dev.gemm(gemm_desc(4, 4, 4, F.BF16, F.F32, batch_shape=(2,), a_batch_strides=(3,), b_batch_strides=(16,)),
                 buf.ptr, buf.ptr, buf.ptr)
    with pytest.raises(F.MpcError, match="multiple of Hk"):
        dev.sdpa(sdpa_desc(1, 3, 2, 8, 8, 64, 64, F.F16), buf.ptr, buf.ptr, buf.ptr, None, buf.ptr)
    shape = (C.c_int64 * 2)(4, 4)
    perm = (C.c_int32 * 2)(0, 0)
    with pytest.raises(F.MpcError, match="permutation"):
        F.call("mpc_transpose", dev.handle, C.c_void_p(buf.ptr), C.c_void_p(buf.ptr), 4, 2, shape, perm, None)
    assert dev.launch_count() == before
    assert dev.status() == F.OK


def test_a_rank_that_never_joins_the_communicator_times_out():
    """Runs in a child process with its own time limit, NVLS off."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=os.pathsep.join(
        [ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "math-plus_b200"), os.path.join(ROOT, "tests")]))
    cmd = ["timeout", "-k", "20", "180", sys.executable, os.path.join(ROOT, "tests", "_comm_init_timeout.py")]
    r = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "rank 0 timed out as expected" in r.stdout and "device usable" in r.stdout


def _gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_a_rank_that_never_arrives_ends_the_peer_barrier_with_a_timeout():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=os.pathsep.join(
        [ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "math-plus_b200"), os.path.join(ROOT, "tests")]))
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29537",
           os.path.join(ROOT, "tests", "_mgpu_timeout.py")]
    r = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "rank 0 timed out as expected" in r.stdout and "rank 1 skipped the barrier" in r.stdout
