"""Shape and stride planning for the device ops (pure Python, no device needed).

Each function turns the reference's shape rules into the plain integers the C ABI takes:

* matmul: ``Tensor.matmul``'s right-aligned batch broadcasting (packages/tensor-core/src/index.ts:1584-1730,
  ``broadcastShapes`` / ``broadcastStrides``) as per-axis element strides with 0 on broadcast axes;
* linear: ``CpuBackendImpl.linear``'s checks (packages/tensor-cpu/src/index.ts:764-774);
* sdpa: ``CpuBackendImpl.sdpa``'s checks and the mask's strides aligned to [B, H, Lq, Lk]
  (index.ts:821-840, ``alignedStrides`` in packages/tensor-core/src/kernels.ts);
* add: the trailing-block broadcast the device kernel supports (bias rows, residuals).

Errors are raised synchronously with the reference's messages' wording.
"""
from __future__ import annotations

from dataclasses import dataclass


def _prod(xs) -> int:
    n = 1
    for x in xs:
        n *= int(x)
    return n


def broadcast_shapes(a, b) -> tuple:
    """NumPy broadcasting of two shapes (tensor-core ``broadcastShapes``)."""
    n = max(len(a), len(b))
    out = []
    for i in range(n):
        da = a[i - (n - len(a))] if i >= n - len(a) else 1
        db = b[i - (n - len(b))] if i >= n - len(b) else 1
        if da != db and da != 1 and db != 1:
            raise ValueError(f"shapes {list(a)} and {list(b)} do not broadcast")
        out.append(db if da == 1 else da)
    return tuple(out)


def aligned_strides(shape, out_shape) -> list:
    """Row-major element strides of ``shape`` aligned to ``out_shape``, 0 on broadcast axes
    (tensor-core ``alignedStrides``)."""
    n = len(out_shape)
    st = [0] * n
    acc = 1
    for i in range(n - 1, -1, -1):
        j = i - (n - len(shape))
        d = shape[j] if j >= 0 else 1
        st[i] = 0 if d == 1 else acc
        acc *= d
    return st


@dataclass(frozen=True)
class MatmulPlan:
    out_shape: tuple
    batch_shape: tuple
    a_batch_strides: tuple
    b_batch_strides: tuple
    m: int
    n: int
    k: int


def matmul_plan(a_shape, b_shape) -> MatmulPlan:
    """``Backend.matmul`` on rank >= 2 operands: [..., m, k] @ [..., k, n]."""
    if len(a_shape) < 2 or len(b_shape) < 2:
        raise ValueError("matmul needs rank >= 2")
    m, k = a_shape[-2], a_shape[-1]
    k2, n = b_shape[-2], b_shape[-1]
    if k != k2:
        raise ValueError(f"matmul: inner dimensions {k} and {k2} do not match "
                         f"(shapes [{','.join(map(str, a_shape))}] @ [{','.join(map(str, b_shape))}])")
    ba, bb = tuple(a_shape[:-2]), tuple(b_shape[:-2])
    batch = broadcast_shapes(ba, bb)
    if len(batch) > 4:
        # fold leading axes that broadcast the same way on both sides
        raise ValueError("matmul: more than 4 batch axes")
    sa = [s * m * k for s in aligned_strides(ba, batch)]
    sb = [s * k * n for s in aligned_strides(bb, batch)]
    return MatmulPlan(batch + (m, n), batch, tuple(sa), tuple(sb), m, n, k)


def linear_plan(x_shape, w_shape, b_shape=None):
    """``Backend.linear``: x [..., in] · w[out, in]ᵀ (+ b[out]) -> (rows, n_in, n_out, out_shape)."""
    if len(w_shape) != 2:
        raise ValueError("linear weight must be [out, in]")
    n_out, n_in = w_shape
    if len(x_shape) < 1 or x_shape[-1] != n_in:
        raise ValueError(f"linear [{','.join(map(str, x_shape))}] with weight [{','.join(map(str, w_shape))}]")
    if b_shape is not None and _prod(b_shape) != n_out:
        raise ValueError(f"linear bias [{','.join(map(str, b_shape))}] for {n_out} outputs")
    rows = _prod(x_shape[:-1])
    return rows, n_in, n_out, tuple(x_shape[:-1]) + (n_out,)


@dataclass(frozen=True)
class SdpaPlan:
    b: int
    h: int
    hk: int
    lq: int
    lk: int
    d: int
    dv: int
    mask_strides: tuple


def sdpa_plan(q_shape, k_shape, v_shape, mask_shape=None) -> SdpaPlan:
    """``Backend.sdpa`` shape rules (tensor-cpu/src/index.ts:821-840)."""
    if len(q_shape) != 4 or len(k_shape) != 4 or len(v_shape) != 4:
        raise ValueError("sdpa expects rank-4 q/k/v")
    B, H, Lq, Dh = q_shape
    Hk, Lk, Dv = k_shape[1], k_shape[2], v_shape[3]
    if k_shape[0] != B or v_shape[0] != B or v_shape[1] != Hk or v_shape[2] != Lk or k_shape[3] != Dh or H % Hk:
        raise ValueError(f"sdpa q [{','.join(map(str, q_shape))}] k [{','.join(map(str, k_shape))}] "
                         f"v [{','.join(map(str, v_shape))}]")
    strides = (0, 0, 0, 0)
    if mask_shape is not None:
        ms = list(mask_shape)
        if len(ms) > 4:
            raise ValueError(f"sdpa mask [{','.join(map(str, mask_shape))}] has rank > 4")
        ms = [1] * (4 - len(ms)) + ms
        target = (B, H, Lq, Lk)
        try:
            ok = broadcast_shapes(ms, target) == target
        except ValueError:
            ok = False
        if not ok:
            raise ValueError(f"sdpa mask [{','.join(map(str, mask_shape))}] does not broadcast to "
                             f"[{','.join(map(str, target))}]")
        strides = tuple(aligned_strides(ms, target))
    return SdpaPlan(B, H, Hk, Lq, Lk, Dh, Dv, strides)


def add_plan(x_shape, y_shape):
    """Element count of x and the repeated trailing block of y for the device add kernel.

    Supported: y's shape (leading 1s dropped) is a suffix of x's shape — a bias row, a residual,
    a per-row block. Other broadcasts raise (the device kernel repeats one trailing block)."""
    out = broadcast_shapes(x_shape, y_shape)
    if tuple(out) != tuple(x_shape):
        raise ValueError(f"add: [{','.join(map(str, y_shape))}] must broadcast into [{','.join(map(str, x_shape))}]")
    ys = list(y_shape)
    while ys and ys[0] == 1:
        ys.pop(0)
    if ys and tuple(ys) != tuple(x_shape[len(x_shape) - len(ys):]):
        raise NotImplementedError(f"add: broadcast of [{','.join(map(str, y_shape))}] into "
                                  f"[{','.join(map(str, x_shape))}] is not a trailing block")
    return _prod(x_shape), max(1, _prod(ys))


def column_shards(n: int, world: int) -> list:
    """Split N columns over ``world`` ranks as evenly as possible: [(start, width), ...]."""
    base, extra = divmod(n, world)
    out, s = [], 0
    for r in range(world):
        w = base + (1 if r < extra else 0)
        out.append((s, w))
        s += w
    return out


def batch_shard(batch: int, world: int, rank: int) -> tuple:
    """Contiguous batch shard (start, count) of rank ``rank``."""
    s, w = column_shards(batch, world)[rank]
    return s, w


_ELEM_BYTES = {"f32": 4, "f16": 2, "bf16": 2}


@dataclass(frozen=True)
class ColumnSplitPlan:
    m: int
    n_total: int
    k: int
    world: int
    n_shard: int
    shards: tuple  # (first column, width) per rank

    def gathered_to_output_perm(self) -> tuple:
        """The permutation that turns the shard-major all-gather result [world, m, n_shard]
        into row-major C [m, world, n_shard] = [m, n_total]."""
        return (1, 0, 2)


def column_split_plan(m: int, n_total: int, k: int, world: int, dtype_out: str = "bf16") -> ColumnSplitPlan:
    """C [m, n_total] = A [m, k] @ B [k, n_total] with B's columns split evenly over ``world``
    ranks. Every rank's column block must start on a 16-byte boundary of C's rows (the epilogue's
    TMA stores and the all-gather blocks), so ``n_total / world`` elements must be a multiple of
    16 bytes."""
    if world < 1 or world > 8:
        raise ValueError(f"column split over {world} ranks (1..8)")
    if m <= 0 or n_total <= 0 or k <= 0:
        raise ValueError(f"column split of a [{m},{k}] @ [{k},{n_total}] product")
    if n_total % world:
        raise ValueError(f"column split: {n_total} columns do not divide over {world} ranks")
    n = n_total // world
    eo = _ELEM_BYTES[dtype_out]
    if (n * eo) % 16:
        raise ValueError(f"column split: a {n}-column block of {dtype_out} is not a multiple of 16 bytes")
    return ColumnSplitPlan(m, n_total, k, world, n, tuple(column_shards(n_total, world)))
