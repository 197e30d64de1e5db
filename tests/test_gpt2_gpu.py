"""The GPT-2-shaped forward on the B200 against the same forward composed from the oracle's
restatements of the reference's CPU ops (linearNT, attention, layerNormRows, takeRows, geluErf),
rounded to bf16 at every op output as the device stores it (the residual adds inside the
projections' epilogues, as the device fuses them).

Every comparison is per element: |got - want| <= 8·sigma + 1e-2·|want|, where sigma is the RMS of
what bf16 storage itself changes on these inputs (the same composition stored in bf16 against it
stored in f32, the reference's own storage). A device that rounds one op's result the other way from
the oracle diverges from it by about that much, and the oracle's own bf16-vs-f32 deviations reach ~5
sigma; a wrong kernel is off by the signal's own scale (hundreds of sigma). Reduced sizes (2 layers,
batch 2, 128 tokens; one full-width layer with the real 50257-token vocabulary), the residual stream
after block 1 (layer-wise), then the full 12-layer model at 1024 tokens against the oracle's full
forward: per element, per-position checksums of the logits, and a bit-identical second run."""
import math

import numpy as np
import pytest

import oracle as O
from _helpers import bf16_bits_to_f32

pytestmark = pytest.mark.gpu


def oracle_forward(cfg, w, ids, stop_after=None, f32_storage=False):
    f = {k: (bf16_bits_to_f32(v).reshape(v.shape) if v.dtype == np.uint16 else v) for k, v in w.items()}
    kw = dict(store=lambda x: np.asarray(x, np.float32)) if f32_storage else {}
    return O.gpt2_forward(f, ids, cfg.n_layer, cfg.n_head, cfg.eps, threads=O.default_threads(),
                          residual_in_epilogue=True, stop_after=stop_after, **kw)


def storage_sigma(cfg, w, ids, want, stop_after=None, ref32=None):
    """RMS of (bf16-stored composition - f32-stored composition): the rounding noise of bf16 storage."""
    if ref32 is None:
        ref32 = oracle_forward(cfg, w, ids, stop_after, f32_storage=True)
    sigma = math.sqrt(float(np.mean((want.astype(np.float64) - ref32) ** 2)))
    rms = math.sqrt(float(np.mean(ref32.astype(np.float64) ** 2)))
    assert sigma <= 0.02 * rms, (sigma, rms)  # the bound stays far below the signal
    return sigma


@pytest.fixture(scope="module")
def be():
    from tensor_cuda.backend import CudaBackend
    from tensor_cuda.runtime import Device
    return CudaBackend(Device.shared(0))


def run_model(be, cfg, w, ids, stop_after=None):
    from tensor_cuda.backend import host
    from tensor_cuda.gpt2 import GPT2
    model = GPT2(be, cfg, w)
    t = be.from_host_sync(host("i32", ids.shape, ids))
    out = be.read_sync(model.forward(t, stop_after=stop_after))
    return bf16_bits_to_f32(out.data).reshape(out.shape)


def within(got, want, sigma, k=8.0, rel=1e-2):
    """Per element: |got - want| <= k·sigma + rel·|want|. Returns (ok, worst ratio)."""
    want = want.astype(np.float64)
    ratio = np.abs(got.astype(np.float64) - want) / (k * sigma + rel * np.abs(want))
    return bool(np.all(ratio <= 1.0)), float(ratio.max())


SMALL = dict(n_layer=2, d_model=128, n_head=2, d_ff=512, vocab=1001, n_ctx=256, B=2, L=128)
WIDE = dict(n_layer=1, d_model=768, n_head=12, d_ff=3072, vocab=50257, n_ctx=1024, B=1, L=64)


@pytest.mark.parametrize("dims", [SMALL, WIDE])
def test_forward_matches_the_oracle_composition(be, dims):
    from tensor_cuda.gpt2 import GPT2Config, random_weights
    dims = dict(dims)
    B, L = dims.pop("B"), dims.pop("L")
    cfg = GPT2Config(**dims)
    w = random_weights(cfg, seed=5)
    ids = O.randint_i32(B * L, 9, cfg.vocab).reshape(B, L)
    got = run_model(be, cfg, w, ids)
    want = oracle_forward(cfg, w, ids)
    assert got.shape == want.shape and np.all(np.isfinite(got))
    sigma = storage_sigma(cfg, w, ids, want)
    ok, worst = within(got, want, sigma)
    assert ok, (worst, sigma)


@pytest.mark.parametrize("dims", [SMALL, WIDE])
def test_residual_stream_after_block_one(be, dims):
    """Layer-wise: the residual stream after the first block (embeddings, LN, QKV, attention,
    out-projection + residual, LN, fc + GELU, projection + residual), per element."""
    from tensor_cuda.gpt2 import GPT2Config, random_weights
    dims = dict(dims)
    B, L = dims.pop("B"), dims.pop("L")
    cfg = GPT2Config(**dims)
    w = random_weights(cfg, seed=6)
    ids = O.randint_i32(B * L, 10, cfg.vocab).reshape(B, L)
    got = run_model(be, cfg, w, ids, stop_after=1)
    want = oracle_forward(cfg, w, ids, stop_after=1)
    assert got.shape == (B, L, cfg.d_model)
    sigma = storage_sigma(cfg, w, ids, want, stop_after=1)
    ok, worst = within(got, want, sigma)
    assert ok, (worst, sigma)


def test_full_size_forward_against_the_oracle_and_deterministic(be):
    """The full 12-layer model at 1024 tokens (one sequence) against the oracle's full forward:
    every logit within the per-element bound, the per-position checksums (sums over the
    vocabulary) within 8 times their own bf16 storage noise; a second run is bit-identical."""
    from tensor_cuda.gpt2 import GPT2Config, random_weights
    cfg = GPT2Config()
    w = random_weights(cfg, seed=1)
    ids = O.randint_i32(1024, 3, cfg.vocab).reshape(1, 1024)
    a = run_model(be, cfg, w, ids)
    b = run_model(be, cfg, w, ids)
    assert a.shape == (1, 1024, cfg.vocab) and np.all(np.isfinite(a))
    assert np.array_equal(a, b)
    want = oracle_forward(cfg, w, ids)
    ref32 = oracle_forward(cfg, w, ids, f32_storage=True)
    sigma = storage_sigma(cfg, w, ids, want, ref32=ref32)
    ok, worst = within(a, want, sigma)
    assert ok, (worst, sigma)
    # per-position checksums: the same noise yardstick, taken over the checksums themselves
    cs_got, cs_want, cs_32 = (x.astype(np.float64).sum(-1) for x in (a, want, ref32))
    cs_sigma = math.sqrt(float(np.mean((cs_want - cs_32) ** 2)))
    cs_rms = math.sqrt(float(np.mean(cs_32 ** 2)))
    assert cs_sigma <= 0.1 * cs_rms, (cs_sigma, cs_rms)
    assert np.abs(cs_got - cs_want).max() <= 8 * cs_sigma, (np.abs(cs_got - cs_want).max(), cs_sigma, cs_rms)
