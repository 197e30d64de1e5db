"""One rank of the two-GPU column-split check (run under torch.distributed.run).

Every rank builds the same A [m, k] and full B [k, p*n] from seeded generators, keeps its column
block of B, and runs the fused GEMM + all-gather and the NCCL path. Both must give bit-identical
C on every rank (the same kernel computes every block), and 512 sampled entries must match an f64
dot product within the bf16 output rounding."""
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "math-plus_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def main():
    import torch
    import torch.distributed as dist

    from _helpers import from_device_dtype, to_device_dtype
    from tensor_cuda import _ffi as F
    from tensor_cuda.parallel import ColumnSplitGemm, PeerGroup
    from tensor_cuda.runtime import Device

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    dev = Device.shared(local)
    group = PeerGroup.from_torch(dev)
    m, n, k = 1024, 768, 1536  # per-rank block of 768 columns
    rng = np.random.default_rng(11)
    a32 = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b32 = (rng.standard_normal((k, n * world)) / np.sqrt(k)).astype(np.float32)
    a, ea = to_device_dtype(a32, "bf16")
    b, eb = to_device_dtype(b32, "bf16")
    mine = np.ascontiguousarray(b[:, rank * n:(rank + 1) * n])
    da, db = dev.upload(a), dev.upload(mine)
    outs = {}
    for fused in (True, False):
        for layout in ("rows", "blocks"):
            cs = ColumnSplitGemm(group, m, n, k, "bf16", "bf16", F.B_KN, fused=fused, layout=layout)
            for _ in range(3):
                ptr = cs(da.ptr, db.ptr)
            dev.sync()
            if layout == "rows":
                raw = dev.download(ptr, m * n * world * 2, np.uint16, (m, n * world))
            else:  # [p, m, n] -> [m, p, n]
                raw = dev.download(ptr, m * n * world * 2, np.uint16, (world, m, n))
                raw = np.ascontiguousarray(raw.transpose(1, 0, 2)).reshape(m, n * world)
            outs[fused, layout] = from_device_dtype(raw, "bf16")
            cs.destroy()
    for key, c in outs.items():
        assert np.array_equal(c, outs[True, "rows"]), f"{key} differs from the fused row-major result"
    outs[True] = outs[True, "rows"]
    idx = rng.integers(0, [m, n * world], size=(512, 2))
    ref = np.array([np.dot(ea[i].astype(np.float64), eb[:, j].astype(np.float64)) for i, j in idx])
    got = outs[True][idx[:, 0], idx[:, 1]]
    assert np.all(np.abs(got - ref) <= 8e-3 * np.abs(ref) + 1e-3), np.abs(got - ref).max()
    # every rank holds the same C
    h = torch.from_numpy(outs[True].astype(np.float32)).sum(dtype=torch.float64).reshape(1)
    hs = [torch.zeros(1, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(hs, h)
    assert all(float(x) == float(hs[0]) for x in hs)
    group.destroy()
    dist.destroy_process_group()
    print(f"rank {rank} ok", flush=True)


if __name__ == "__main__":
    main()
