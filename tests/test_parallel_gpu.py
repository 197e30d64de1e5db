"""The GEMM fused with its all-gather, on the B200.

One GPU: mpc_gemm_multi_store writes the product into several matrices at a column offset
(every destination equal to the oracle's product there, every other column untouched), and a
one-rank ColumnSplitGemm (fused and NCCL paths) equals the oracle. Two GPUs (skipped with fewer):
two ranks under torch.distributed.run, fused vs NCCL path bit-identical and sampled entries
against f64 dot products."""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
from _helpers import from_device_dtype, gemm_bound, to_device_dtype

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def dev():
    from tensor_cuda.runtime import Device
    return Device.shared(0)


@pytest.mark.parametrize("dtype_in,dtype_out,layout", [("bf16", "bf16", "kn"), ("f16", "f32", "nk"),
                                                       ("bf16", "f16", "nk")])
def test_multi_store_writes_every_destination_at_its_offset(dev, dtype_in, dtype_out, layout):
    from tensor_cuda import _ffi as F
    from tensor_cuda.parallel import gemm_multi_store
    from tensor_cuda.runtime import gemm_desc
    m, n, k, ldc, off, ndst = 300, 264, 200, 800, 264, 3
    a, ea = to_device_dtype(O.lcg_gemm(m * k, 1).reshape(m, k), dtype_in)
    bmat = O.lcg_gemm(k * n, 2).reshape(k, n)
    b, eb = to_device_dtype(bmat if layout == "kn" else np.ascontiguousarray(bmat.T), dtype_in)
    want = O.matmul(ea, eb) if layout == "kn" else O.linear(ea, eb)
    eo = F.DTYPE_BYTES[F.DTYPE_CODES[dtype_out]]
    sentinel = np.full(m * ldc * eo, 0x5A, np.uint8)
    dsts = [dev.upload(sentinel) for _ in range(ndst)]
    da, db = dev.upload(a), dev.upload(b)
    desc = gemm_desc(m, n, k, F.DTYPE_CODES[dtype_in], F.DTYPE_CODES[dtype_out],
                     F.B_KN if layout == "kn" else F.B_NK)
    gemm_multi_store(dev, desc, da.ptr, db.ptr, [d.ptr for d in dsts], ldc, off)
    dev.sync()
    ebk = eb if layout == "kn" else np.ascontiguousarray(eb.T)
    bound = gemm_bound(want, O.matmul(np.abs(ea), np.abs(ebk)), dtype_in, dtype_out)
    for d in dsts:
        raw = dev.download(d.ptr, m * ldc * eo, np.uint8, (m, ldc * eo))
        inside = raw[:, off * eo:(off + n) * eo].copy()
        got = from_device_dtype(inside.view({4: np.float32, 2: np.uint16 if dtype_out == "bf16" else np.float16}[eo]),
                                dtype_out)
        assert np.all(np.abs(got - want) <= bound)
        assert np.all(raw[:, :off * eo] == 0x5A) and np.all(raw[:, (off + n) * eo:] == 0x5A)


@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_multi_store_cta_pairs(dev, layout):
    """A single-destination product with at least one 256 x 256 tile per resident CTA pair takes
    the paired kernel (the column-split workload on one GPU): the block lands at its column
    offset, the columns around it stay untouched."""
    from tensor_cuda import _ffi as F
    from tensor_cuda.parallel import gemm_multi_store
    from tensor_cuda.runtime import gemm_desc
    m, n, k, ldc, off, ndst = 2200, 2304, 200, 6912, 2304, 1
    a, ea = to_device_dtype(O.lcg_gemm(m * k, 5).reshape(m, k), "bf16")
    bmat = O.lcg_gemm(k * n, 6).reshape(k, n)
    b, eb = to_device_dtype(bmat if layout == "kn" else np.ascontiguousarray(bmat.T), "bf16")
    ebk = eb if layout == "kn" else np.ascontiguousarray(eb.T)
    want = ea.astype(np.float64) @ ebk.astype(np.float64)
    sentinel = np.full(m * ldc * 2, 0x5A, np.uint8)
    dsts = [dev.upload(sentinel) for _ in range(ndst)]
    da, db = dev.upload(a), dev.upload(b)
    desc = gemm_desc(m, n, k, F.BF16, F.BF16, F.B_KN if layout == "kn" else F.B_NK)
    gemm_multi_store(dev, desc, da.ptr, db.ptr, [d.ptr for d in dsts], ldc, off)
    dev.sync()
    bound = gemm_bound(want, np.abs(ea).astype(np.float64) @ np.abs(ebk).astype(np.float64), "bf16", "bf16")
    for d in dsts:
        raw = dev.download(d.ptr, m * ldc * 2, np.uint8, (m, ldc * 2))
        got = from_device_dtype(raw[:, off * 2:(off + n) * 2].copy().view(np.uint16), "bf16")
        assert np.all(np.abs(got - want) <= bound)
        assert np.all(raw[:, :off * 2] == 0x5A) and np.all(raw[:, (off + n) * 2:] == 0x5A)


def test_multi_store_rejects_misaligned_offsets(dev):
    from tensor_cuda import _ffi as F
    from tensor_cuda.parallel import gemm_multi_store
    from tensor_cuda.runtime import gemm_desc
    d = dev.alloc(64 * 64 * 2)
    a = dev.alloc(64 * 64 * 2)
    desc = gemm_desc(64, 16, 64, F.BF16, F.BF16, F.B_KN)
    with pytest.raises(F.MpcError, match="16 bytes"):
        gemm_multi_store(dev, desc, a.ptr, a.ptr, [d.ptr], 64, 3)
    with pytest.raises(F.MpcError, match="do not fit"):
        gemm_multi_store(dev, desc, a.ptr, a.ptr, [d.ptr], 64, 56)
    with pytest.raises(F.MpcError, match="destinations"):
        gemm_multi_store(dev, desc, a.ptr, a.ptr, [d.ptr] * 9, 64, 0)


@pytest.mark.parametrize("fused,layout", [(True, "rows"), (False, "rows"), (True, "blocks"), (False, "blocks")])
def test_one_rank_column_split_equals_the_oracle(dev, fused, layout):
    from tensor_cuda import _ffi as F
    from tensor_cuda.parallel import ColumnSplitGemm, PeerGroup, unique_id
    m, n, k = 256, 512, 320
    a, ea = to_device_dtype(O.lcg_gemm(m * k, 3).reshape(m, k), "bf16")
    b, eb = to_device_dtype(O.lcg_gemm(k * n, 4).reshape(k, n), "bf16")
    g = PeerGroup(dev, 0, 1, unique_id())
    try:
        cs = ColumnSplitGemm(g, m, n, k, "bf16", "f32", F.B_KN, fused=fused, layout=layout)
        da, db = dev.upload(a), dev.upload(b)
        for _ in range(2):  # the second call reuses the buffers and barriers
            ptr = cs(da.ptr, db.ptr)
        dev.sync()
        got = dev.download(ptr, m * n * 4, np.float32, (m, n))
        want = O.matmul(ea, eb)
        assert np.all(np.abs(got - want) <= gemm_bound(want, O.matmul(np.abs(ea), np.abs(eb)), "bf16", "f32"))
        cs.destroy()
    finally:
        g.destroy()


def _normal_bf16_rows(rows, cols, seed, std, block=512):
    """[rows, cols] bf16 bits from the oracle's seeded normal generator, row blocks of `block` rows
    seeded seed * 100003 + block index, generated on host threads (the generator releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor
    out = np.empty((rows, cols), np.uint16)

    def fill(i):
        r0, r1 = i * block, min(rows, (i + 1) * block)
        out[r0:r1] = O.normal_half_bits((r1 - r0) * cols, seed * 100003 + i, 0, std, True).reshape(r1 - r0, cols)

    with ThreadPoolExecutor(max_workers=O.default_threads()) as ex:
        list(ex.map(fill, range((rows + block - 1) // block)))
    return out


def test_column_split_at_the_large_gemm_configuration_sampled(dev):
    """The single large GEMM configuration on one rank: A [16384, 8192] @ B [8192, 65536] bf16 -> bf16
    through ColumnSplitGemm (fused path: peer barrier, the paired GEMM storing into the peer buffer,
    barrier). 4096 random (i, j) entries are held to f64 dot products of the same bf16 inputs within
    1e-2 relative / 2e-3 absolute, and to the f32-accumulation bound of the other GEMM tests; every
    entry of C is finite."""
    from tensor_cuda import _ffi as F
    from tensor_cuda.parallel import ColumnSplitGemm, PeerGroup, unique_id
    M, N, K = 16384, 65536, 8192
    a_bits = _normal_bf16_rows(M, K, 71, 1 / np.sqrt(K))
    b_bits = _normal_bf16_rows(K, N, 72, 1 / np.sqrt(K))
    g = PeerGroup(dev, 0, 1, unique_id())
    try:
        cs = ColumnSplitGemm(g, M, N, K, "bf16", "bf16", F.B_KN, fused=True)
        da, db = dev.upload(a_bits), dev.upload(b_bits)
        ptr = cs(da.ptr, db.ptr)
        dev.sync()
        c_bits = dev.download(ptr, M * N * 2, np.uint16, (M, N))
        cs.destroy()
        da.free()
        db.free()
    finally:
        g.destroy()
    got_all = from_device_dtype(c_bits, "bf16")
    assert np.isfinite(got_all).all()
    rng = np.random.default_rng(5)
    i = rng.integers(0, M, 4096)
    j = rng.integers(0, N, 4096)
    a = from_device_dtype(a_bits[i], "bf16").astype(np.float64)                            # [4096, K]
    b = from_device_dtype(np.ascontiguousarray(b_bits[:, j].T), "bf16").astype(np.float64)  # [4096, K]
    want = (a * b).sum(1)
    absprod = (np.abs(a) * np.abs(b)).sum(1)
    got = got_all[i, j].astype(np.float64)
    assert np.all(np.abs(got - want) <= 2e-3 + 1e-2 * np.abs(want)), np.abs(got - want).max()
    assert np.all(np.abs(got - want) <= gemm_bound(want, absprod, "bf16", "bf16"))


def _gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_two_rank_fused_allgather_matches_nccl_and_f64():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=os.pathsep.join(
        [ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "math-plus_b200"), os.path.join(ROOT, "tests")]))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29531",
           os.path.join(ROOT, "tests", "_mgpu_check.py")]
    r = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "rank 0 ok" in r.stdout and "rank 1 ok" in r.stdout
