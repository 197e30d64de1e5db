"""Child process of test_failure_gpu: rank 0 of a two-rank communicator whose rank 1 never calls
init. The init must give up after its limit with MPC_ERR_TIMEOUT (the half-built communicator
aborted on the host; no kernel involved), and the device must stay usable afterwards: a one-rank
communicator and a GEMM still work."""
import sys
import time

import numpy as np

import oracle as O
from _helpers import gemm_bound


def main() -> int:
    from tensor_cuda import _ffi as F
    from tensor_cuda.parallel import PeerGroup, unique_id
    from tensor_cuda.runtime import Device, gemm_desc
    dev = Device.shared(0)
    uid = unique_id()
    t0 = time.monotonic()
    try:
        PeerGroup(dev, 0, 2, uid, timeout_ms=3000)
    except F.MpcError as e:
        took = time.monotonic() - t0
        if e.status != F.ERR_TIMEOUT or "never joined" not in str(e):
            print(f"unexpected error: {e}")
            return 1
        print(f"rank 0 timed out as expected after {took:.1f} s: {e}")
    else:
        print("init returned although rank 1 never joined")
        return 1
    if not 2.5 <= took <= 60:
        print(f"the limit was 3 s but the call took {took:.1f} s")
        return 1
    g = PeerGroup(dev, 0, 1, unique_id(), timeout_ms=60000)  # a complete group still forms
    g.destroy()
    m = n = k = 256
    a = O.lcg_gemm(m * k, 5).reshape(m, k)
    b = O.lcg_gemm(k * n, 6).reshape(k, n)
    da, db, dc = dev.upload(a), dev.upload(b), dev.alloc(m * n * 4)
    dev.gemm(gemm_desc(m, n, k, F.F32, F.F32), da.ptr, db.ptr, dc.ptr)
    dev.sync()
    got = dev.download(dc.ptr, m * n * 4, np.float32, (m, n)).astype(np.float64)
    want = O.matmul(a, b).astype(np.float64)
    if not np.all(np.abs(got - want) <= gemm_bound(want, O.matmul(np.abs(a), np.abs(b)), "f32", "f32")):
        print("GEMM after the timed-out init is wrong")
        return 1
    print("device usable after the timed-out init")
    return 0


if __name__ == "__main__":
    sys.exit(main())
