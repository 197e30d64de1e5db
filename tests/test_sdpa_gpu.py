"""Fused attention on the B200 (mpc_sdpa through the C ABI) vs the oracle's restatement of
tensor-core `attention` (packages/tensor-core/src/nn-kernels.ts:179-239) and the reference's own
attention_oracle.py fixtures (tests/golden/attention_webgpu.npz)."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
from _helpers import NP_STORAGE, from_device_dtype, to_device_dtype

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    from tensor_cuda.runtime import Device
    return Device.shared(0)


def run_sdpa(dev, q, k, v, dtype, scale, causal=False, mask=None, want_lse=False):
    """q [B,H,Lq,D], k/v [B,Hk,Lk,D*] f32 arrays (exact in `dtype`); mask bool/f32 broadcastable."""
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import sdpa_desc
    B, H, Lq, D = q.shape
    Hk, Lk, Dv = k.shape[1], k.shape[2], v.shape[3]
    dq, dk, dv = (dev.upload(to_device_dtype(x, dtype)[0]) for x in (q, k, v))
    do = dev.alloc(B * H * Lq * Dv * F.DTYPE_BYTES[F.DTYPE_CODES[dtype]])
    dl = dev.alloc(B * H * Lq * 4) if want_lse else None
    kind, strides, dm = F.MASK_NONE, (0, 0, 0, 0), None
    if mask is not None:
        m = np.asarray(mask)
        shape = (1,) * (4 - m.ndim) + m.shape
        st, acc = [0] * 4, 1
        for d in range(3, -1, -1):
            st[d] = 0 if shape[d] == 1 else acc
            acc *= shape[d]
        strides = tuple(st)
        if m.dtype == np.bool_:
            kind, dm = F.MASK_BOOL, dev.upload(np.ascontiguousarray(m, np.uint8))
        else:
            kind, dm = F.MASK_ADD, dev.upload(np.ascontiguousarray(m, np.float32))
    desc = sdpa_desc(B, H, Hk, Lq, Lk, D, Dv, F.DTYPE_CODES[dtype], causal, scale, kind, strides)
    dev.sdpa(desc, dq.ptr, dk.ptr, dv.ptr, dm.ptr if dm is not None else None, do.ptr, dl.ptr if dl else None)
    dev.sync()
    out = from_device_dtype(dev.download(do.ptr, do.nbytes, NP_STORAGE[dtype], (B, H, Lq, Dv)), dtype)
    if want_lse:
        return out, dev.download(dl.ptr, dl.nbytes, np.float32, (B, H, Lq))
    return out


def exact(x, dtype):
    return to_device_dtype(x, dtype)[1]


def half_tol(q, k, v, mask, scale, want, dtype):
    """Per-element bound for f16 / bf16 attention: 2e-3 + 1e-2·|want|, and for bf16 the effect of
    bf16 attention weights on top: P.V multiplies probabilities rounded to 8 significant bits, which
    moves a normalised output by at most 2 * 2^-9 times the weighted spread of the V rows it averages,
    sqrt(E_w[v^2] - O^2) (E_w[v^2] is attention with V squared). Rows that average a few very
    different V rows (the first rows under a causal mask) need that term; long rows barely do."""
    tol = 2e-3 + 1e-2 * np.abs(want)
    if dtype == "bf16":
        ev2 = O.sdpa(q, k, (v.astype(np.float64) ** 2).astype(np.float32), mask, scale, threads=O.default_threads())
        tol = tol + 2.0 ** -8 * np.sqrt(np.maximum(ev2.astype(np.float64) - want.astype(np.float64) ** 2, 0.0))
    return tol


def ref_lse(q, k, scale, causal):
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), np.repeat(k, q.shape[1] // k.shape[1], 1).astype(np.float64))
    s = s * scale
    if causal:
        Lq, Lk = s.shape[-2:]
        s = np.where(np.tril(np.ones((Lq, Lk), bool)), s, -np.inf)
    mx = s.max(-1, keepdims=True)
    return (mx + np.log(np.exp(s - mx).sum(-1, keepdims=True)))[..., 0]


def test_reference_attention_fixtures(dev, golden_dir):
    """flash-attention.test.ts:257-336 cases (attention_oracle.py outputs), f32 and f16 storage;
    max |err| <= 1e-4 (the test's own bound) for f32, fully masked rows compared too (zeros)."""
    fx = np.load(os.path.join(golden_dir, "attention_webgpu.npz"))
    names = sorted({k[: -len("_dims")] for k in fx.files if k.endswith("_dims")})
    for name in names:
        B, LQ, LK, D, seed = (int(v) for v in fx[name + "_dims"])
        q = O.lcg_gemm(B * LQ * D, seed).reshape(B, 1, LQ, D)
        k = O.lcg_gemm(B * LK * D, seed + 1).reshape(B, 1, LK, D)
        v = O.lcg_gemm(B * LK * D, seed + 2).reshape(B, 1, LK, D)
        mask = None
        if name + "_mask" in fx.files:
            ms = tuple(int(s) for s in fx[name + "_maskshape"])
            m3 = (1,) * (3 - len(ms)) + ms
            mask = (fx[name + "_mask"].reshape(m3) != 0).reshape(m3[0], 1, m3[1], m3[2])
        scale = float(fx[name + "_scale"][0])
        got = run_sdpa(dev, q, k, v, "f32", scale, mask=mask).reshape(-1).astype(np.float64)
        assert np.abs(got - fx[name + "_out"]).max() <= 1e-4, name
        got16 = run_sdpa(dev, exact(q, "f16"), exact(k, "f16"), exact(v, "f16"), "f16", scale, mask=mask)
        want16 = O.sdpa(exact(q, "f16"), exact(k, "f16"), exact(v, "f16"), mask, scale)
        assert np.all(np.abs(got16 - want16) <= 2e-3 + 1e-2 * np.abs(want16)), name


def test_differential_sdpa_cases(dev, golden_dir):
    """differential.test.ts:103-107 (numpy_oracle.py outputs): GQA, key padding, causal and
    additive masks, the B=1 H=16 L=128 D=64 encoder shape; ACCUM tolerance for f32."""
    fx = np.load(os.path.join(golden_dir, "differential_cpu.npz"))
    for name in (str(n) for n in fx["_names"]):
        if not name.startswith("sdpa"):
            continue
        gen, shapes, ranks = fx[name + "_gen"], fx[name + "_shapes"], fx[name + "_ranks"]
        ins = [O.lcg_seeded(int(np.prod(shapes[i][: ranks[i]])), int(s), lo, hi).astype(np.float32)
               .reshape(tuple(int(d) for d in shapes[i][: ranks[i]])) for i, (s, lo, hi) in enumerate(gen)]
        mask = fx[name + "_mask"] if name + "_mask" in fx.files else None
        scale = float(fx[name + "_scale"][0])
        got = run_sdpa(dev, ins[0], ins[1], ins[2], "f32", scale, mask=mask)
        want = fx[name + "_out"]
        assert np.all(np.abs(got - want) <= 1e-5 + 1e-5 * np.abs(want)), name
        for dt in ("f16", "bf16"):
            e = [exact(x, dt) for x in ins[:3]]
            got = run_sdpa(dev, *e, dt, scale, mask=mask)
            want = O.sdpa(*e, mask, scale)
            tol = half_tol(*e, mask, scale, want, dt)
            assert np.all(np.abs(got - want) <= tol), (name, dt, np.abs(got - want).max())


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("B,H,Hk,Lq,Lk,D,causal", [
    (2, 4, 4, 1000, 1000, 128, True),    # ragged length, diagonal tiles, two Q tiles per CTA
    (1, 2, 2, 300, 700, 128, False),     # Lq != Lk, K/V tail tile
    (2, 8, 2, 384, 384, 64, True),       # GQA, head dim 64
    (1, 3, 1, 130, 257, 64, False),      # one row in the second Q tile
    (3, 25, 5, 800, 800, 64, True),      # 300 units on a persistent grid: CTAs walk several unit
                                         # pairs; the last q-block of each head has no second tile
])
def test_tensor_core_path_shapes(dev, dtype, B, H, Hk, Lq, Lk, D, causal):
    """For every causal case here the heavy / light unit pairs leave CTAs unevenly loaded, so the
    host deals the units in the cost-sorted snake order instead; the non-causal cases and the full
    causal configuration (test_causal_attention_full_config_sampled) take the pairs."""
    q = exact(O.normal_f32(B * H * Lq * D, 31).reshape(B, H, Lq, D), dtype)
    k = exact(O.normal_f32(B * Hk * Lk * D, 32).reshape(B, Hk, Lk, D), dtype)
    v = exact(O.normal_f32(B * Hk * Lk * D, 33).reshape(B, Hk, Lk, D), dtype)
    scale = 1 / np.sqrt(D)
    got, lse = run_sdpa(dev, q, k, v, dtype, scale, causal=causal, want_lse=True)
    mask = np.tril(np.ones((Lq, Lk), np.bool_)).reshape(1, 1, Lq, Lk) if causal else None
    want = O.sdpa(q, k, v, mask, scale, threads=O.default_threads())
    tol = half_tol(q, k, v, mask, scale, want, dtype)
    assert np.all(np.abs(got - want) <= tol), float((np.abs(got - want) / tol).max())
    assert np.abs(lse - ref_lse(q, k, scale, causal)).max() <= 2e-3


def test_tensor_core_bool_and_additive_masks(dev):
    B, H, L, D = 2, 2, 200, 64
    q, k, v = (exact(O.normal_f32(B * H * L * D, s).reshape(B, H, L, D), "f16") for s in (41, 42, 43))
    pad = np.ones((B, 1, 1, L), np.bool_)
    pad[0, ..., 150:] = False
    pad[1, ..., 37:] = False
    add = (O.lcg_seeded(B * H * L * L, 44, -3, 1).astype(np.float32)).reshape(B, H, L, L)
    for mask in (pad, add):
        got = run_sdpa(dev, q, k, v, "f16", 0.125, mask=mask)
        want = O.sdpa(q, k, v, mask, 0.125, threads=O.default_threads())
        assert np.all(np.abs(got - want) <= 2e-3 + 1e-2 * np.abs(want)), np.abs(got - want).max()


def test_generic_path_skips_masked_non_finite_values(dev):
    """flash-attention.test.ts:338: keys no query can see may hold NaN in V; the output stays finite.
    (The f32 path skips masked keys; a fully masked row yields zeros, backend.test.ts:112-119.)"""
    B, L, D = 2, 128, 32
    q, k, v = (O.lcg_gemm(B * L * D, s).reshape(B, 1, L, D) for s in (1, 2, 3))
    lens = [40, 70]
    mask = np.zeros((B, 1, 1, L), np.bool_)
    for b, n in enumerate(lens):
        mask[b, ..., :n] = True
        v[b, 0, (n + 31) // 32 * 32:] = np.nan
    got = run_sdpa(dev, q, k, v, "f32", 1 / np.sqrt(D), mask=mask)
    assert np.isfinite(got).all()
    full = np.zeros((1, 1, 2, 4), np.bool_)
    full[..., 0, 0] = True
    qq, kk, vv = (O.lcg_seeded(8, s).astype(np.float32).reshape(1, 1, 2, 4) for s in (1, 2, 3))
    out = run_sdpa(dev, qq, kk, vv, "f32", 0.5, mask=full).reshape(-1)
    assert out[4:].tolist() == [0, 0, 0, 0] and np.isfinite(out[:4]).all()


def test_causal_attention_full_config_sampled(dev):
    """The causal f16 configuration [16, 32, 2048, 128], scale 1/sqrt(128): every output is finite
    and 3 sampled (b, h) heads match the oracle (1e-2 relative / 2e-3 absolute)."""
    B, H, L, D = 16, 32, 2048, 128
    n = B * H * L * D
    q = O.normal_half_bits(n, 51, 0, 1, False).view(np.float16).reshape(B, H, L, D)
    k = O.normal_half_bits(n, 52, 0, 1, False).view(np.float16).reshape(B, H, L, D)
    v = O.normal_half_bits(n, 53, 0, 1, False).view(np.float16).reshape(B, H, L, D)
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import sdpa_desc
    dq, dk, dv = dev.upload(q), dev.upload(k), dev.upload(v)
    do = dev.alloc(q.nbytes)
    dev.sdpa(sdpa_desc(B, H, H, L, L, D, D, F.F16, True, 1 / np.sqrt(D)), dq.ptr, dk.ptr, dv.ptr, None, do.ptr)
    dev.sync()
    got = dev.download(do.ptr, do.nbytes, np.float16, (B, H, L, D)).astype(np.float32)
    assert np.isfinite(got).all()
    mask = np.tril(np.ones((L, L), np.bool_)).reshape(1, 1, L, L)
    for (b, h) in ((0, 0), (7, 19), (15, 31)):
        want = O.sdpa(q[b:b + 1, h:h + 1].astype(np.float32), k[b:b + 1, h:h + 1].astype(np.float32),
                      v[b:b + 1, h:h + 1].astype(np.float32), mask, 1 / np.sqrt(D), threads=O.default_threads())
        g = got[b:b + 1, h:h + 1]
        assert np.all(np.abs(g - want) <= 2e-3 + 1e-2 * np.abs(want)), (b, h, np.abs(g - want).max())


@pytest.mark.parametrize("dtype,D,causal", [("bf16", 64, True), ("f16", 128, False), ("f32", 64, True)])
def test_packed_qkv_layout_matches_the_contiguous_oracle(dev, dtype, D, causal):
    """mpc_sdpa_strided on a packed [B, L, 3, H, D] projection writing [B, L, H, D] (the tensor-core
    path for f16 / bf16, the CUDA-core path for f32) against the oracle on the split heads."""
    from tensor_cuda import _ffi as F
    from tensor_cuda.backend import CudaBackend, host
    B, L, H = 2, 300, 3
    x = exact(O.normal_f32(B * L * 3 * H * D, 61).reshape(B, L, 3, H, D), dtype)
    be = CudaBackend(dev)
    if dtype == "bf16":
        bits = (x.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
        t = be.from_host_sync(host("bf16", (B, L, 3 * H * D), bits))
    else:
        t = be.from_host_sync(host(dtype, (B, L, 3 * H * D), x.reshape(B, L, -1)))
    out = be.read_sync(be.sdpa_packed(t, H, 1 / np.sqrt(D), causal=causal))
    got = out.data
    if dtype == "bf16":
        got = (got.astype(np.uint32) << 16).view(np.float32)
    got = np.asarray(got, np.float32).reshape(B, L, H, D)
    q, k, v = (np.ascontiguousarray(np.transpose(x[:, :, i].astype(np.float32), (0, 2, 1, 3))) for i in range(3))
    mask = np.tril(np.ones((L, L), np.bool_)).reshape(1, 1, L, L) if causal else None
    want_h = O.sdpa(q, k, v, mask, 1 / np.sqrt(D), threads=O.default_threads())  # [B, H, L, D]
    want = np.transpose(want_h, (0, 2, 1, 3))
    tol = (1e-5 + 1e-5 * np.abs(want) if dtype == "f32"
           else np.transpose(half_tol(q, k, v, mask, 1 / np.sqrt(D), want_h, dtype), (0, 2, 1, 3)))
    assert np.all(np.abs(got - want) <= tol), np.abs(got - want).max()
