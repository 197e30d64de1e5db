"""Rank bodies for the multi-process tests (spawned, one process per rank). Each returns through
a file so the parent test can check every rank's view."""
import os
import sys

import numpy as np


def _paths():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "oracle"), os.path.join(root, "math-plus_b200"), os.path.join(root, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)


def column_split_on_gloo(rank: int, world: int, port: int, out_dir: str, m: int, n_total: int, k: int) -> None:
    """Rank r computes its column block with the oracle, the blocks are all-gathered over gloo in
    shard-major order, and the plan's permutation reassembles the row-major product."""
    _paths()
    import torch
    import torch.distributed as dist

    import oracle as O
    from tensor_cuda import plan as P

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        pl = P.column_split_plan(m, n_total, k, world, "f32")
        a = O.lcg_gemm(m * k, 1).reshape(m, k)
        b = O.lcg_gemm(k * n_total, 2).reshape(k, n_total)
        c0, w = pl.shards[rank]
        mine = O.matmul(a, np.ascontiguousarray(b[:, c0:c0 + w]))  # [m, n_shard]
        blocks = [torch.empty((m, pl.n_shard), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(blocks, torch.from_numpy(mine))
        gathered = torch.stack(blocks).numpy()  # [world, m, n_shard]
        c = np.transpose(gathered, pl.gathered_to_output_perm()).reshape(m, n_total)
        # batch sharding: each rank's contiguous slice, gathered back in rank order
        batch = 13
        s, cnt = P.batch_shard(batch, world, rank)
        counts = [P.batch_shard(batch, world, r)[1] for r in range(world)]
        ids = torch.arange(s, s + cnt, dtype=torch.int64)
        padded = torch.full((max(counts),), -1, dtype=torch.int64)
        padded[:cnt] = ids
        got = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(got, padded)
        order = np.concatenate([g.numpy()[:c] for g, c in zip(got, counts)])
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), c=c, order=order)
    finally:
        dist.destroy_process_group()
