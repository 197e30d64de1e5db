"""Host-side shape planning (no GPU): the reference's broadcasting and validation rules as the
integers the C ABI takes."""
import numpy as np
import pytest

from tensor_cuda import plan as P


@pytest.mark.parametrize("a,b", [((4, 8), (8, 5)), ((2, 3, 4), (4, 5)), ((2, 1, 5, 7), (3, 7, 6)),
                                 ((1, 5, 7), (3, 7, 6)), ((3, 2, 4, 4), (3, 1, 4, 2))])
def test_matmul_plan_matches_numpy_broadcasting(a, b):
    pl = P.matmul_plan(a, b)
    x = np.random.default_rng(0).standard_normal(a)
    y = np.random.default_rng(1).standard_normal(b)
    want = np.matmul(x, y)
    assert pl.out_shape == want.shape
    # recompute through the plan's per-axis element strides, as the kernel does
    xf, yf = x.reshape(-1), y.reshape(-1)
    out = np.empty(want.shape)
    for idx in np.ndindex(*pl.batch_shape):
        oa = sum(i * s for i, s in zip(idx, pl.a_batch_strides))
        ob = sum(i * s for i, s in zip(idx, pl.b_batch_strides))
        A = xf[oa:oa + pl.m * pl.k].reshape(pl.m, pl.k)
        B = yf[ob:ob + pl.k * pl.n].reshape(pl.k, pl.n)
        out[idx] = A @ B
    assert np.allclose(out, want)


def test_matmul_plan_errors():
    with pytest.raises(ValueError, match="rank >= 2"):
        P.matmul_plan((6,), (2, 3))
    with pytest.raises(ValueError, match="inner dimensions 3 and 4 do not match"):
        P.matmul_plan((2, 3), (4, 2))
    with pytest.raises(ValueError, match="do not broadcast"):
        P.matmul_plan((2, 3, 4), (3, 4, 5))


def test_linear_plan_matches_tensor_cpu_messages():
    assert P.linear_plan((2, 37, 96), (70, 96), (70,)) == (74, 96, 70, (2, 37, 70))
    # packages/tensor-cpu/test/backend.test.ts:104
    with pytest.raises(ValueError, match=r"linear \[2,3\] with weight \[3,2\]"):
        P.linear_plan((2, 3), (3, 2))
    with pytest.raises(ValueError, match="bias"):
        P.linear_plan((2, 3), (4, 3), (5,))


def test_sdpa_plan_gqa_and_mask_strides():
    pl = P.sdpa_plan((2, 6, 5, 16), (2, 1, 11, 16), (2, 1, 11, 16), (2, 1, 1, 11))
    assert (pl.b, pl.h, pl.hk, pl.lq, pl.lk, pl.d, pl.dv) == (2, 6, 1, 5, 11, 16, 16)
    assert pl.mask_strides == (11, 0, 0, 1)
    assert P.sdpa_plan((1, 3, 13, 8), (1, 3, 13, 8), (1, 3, 13, 8), (13, 13)).mask_strides == (0, 0, 13, 1)
    with pytest.raises(ValueError, match="rank-4"):
        P.sdpa_plan((1, 2, 3), (1, 2, 3, 4), (1, 2, 3, 4))
    with pytest.raises(ValueError, match="does not broadcast"):
        P.sdpa_plan((1, 2, 3, 4), (1, 2, 5, 4), (1, 2, 5, 4), (1, 1, 3, 6))
    with pytest.raises(ValueError):
        P.sdpa_plan((1, 3, 3, 4), (1, 2, 5, 4), (1, 2, 5, 4))  # H % Hk


def test_add_plan_trailing_blocks():
    assert P.add_plan((4, 5, 6), (6,)) == (120, 6)
    assert P.add_plan((4, 5, 6), (1, 5, 6)) == (120, 30)
    assert P.add_plan((4, 5, 6), (4, 5, 6)) == (120, 120)
    with pytest.raises(NotImplementedError):
        P.add_plan((4, 5, 6), (5, 1))
    with pytest.raises(ValueError):
        P.add_plan((4, 5), (7,))


def test_shards_cover_everything_once():
    for n in (1, 7, 64, 65536):
        for w in (1, 2, 3, 4, 8):
            sh = P.column_shards(n, w)
            assert sum(c for _, c in sh) == n
            assert all(sh[i][0] + sh[i][1] == sh[i + 1][0] for i in range(w - 1))
            assert max(c for _, c in sh) - min(c for _, c in sh) <= 1
