"""The multi-GPU host logic on CPU: the column-split plan's checks, and a world-size-2 gloo run of
the split (oracle column blocks -> shard-major all-gather -> the plan's permutation) against the
oracle's whole product; batch shards cover every entry once, in rank order."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import oracle as O
from tensor_cuda import plan as P


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_column_split_plan_checks():
    pl = P.column_split_plan(16384, 65536, 8192, 8)
    assert pl.n_shard == 8192 and pl.shards[3] == (3 * 8192, 8192)
    with pytest.raises(ValueError, match="do not divide"):
        P.column_split_plan(64, 100, 64, 3)
    with pytest.raises(ValueError, match="16 bytes"):
        P.column_split_plan(64, 12, 64, 2, "bf16")  # 6 bf16 columns = 12 bytes
    with pytest.raises(ValueError, match="ranks"):
        P.column_split_plan(64, 64, 64, 9)
    assert P.column_split_plan(64, 16, 64, 2, "f32").n_shard == 8


def _spawned(rank, world, port, out_dir, m, n, k):
    import _dist_workers
    _dist_workers.column_split_on_gloo(rank, world, port, out_dir, m, n, k)


@pytest.mark.parametrize("world", [2])
def test_column_split_reassembles_on_gloo(tmp_path, world):
    m, n, k = 24, 32, 40
    mp.start_processes(_spawned, args=(world, _free_port(), str(tmp_path), m, n, k), nprocs=world,
                       start_method="spawn", join=True)
    want = O.matmul(O.lcg_gemm(m * k, 1).reshape(m, k), O.lcg_gemm(k * n, 2).reshape(k, n))
    for r in range(world):
        d = np.load(os.path.join(tmp_path, f"rank{r}.npz"))
        assert np.array_equal(d["c"], want), r
        assert d["order"].tolist() == list(range(13))
