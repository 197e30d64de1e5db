"""The GPT-2-shaped forward on the B200 against the same forward composed from the oracle's
restatements of the reference's CPU ops (linearNT, attention, layerNormRows, takeRows, geluErf),
rounded to bf16 at every op output as the device stores it. Reduced sizes for parity (2 layers,
batch 2, 128 tokens; and one full-width layer with the real 50257-token vocabulary), then the full
12-layer model at 1024 tokens: finite logits and a bit-identical second run."""
import math

import numpy as np
import pytest

import oracle as O
from _helpers import bf16_bits_to_f32

pytestmark = pytest.mark.gpu


def oracle_forward(cfg, w, ids):
    f = {k: (bf16_bits_to_f32(v).reshape(v.shape) if v.dtype == np.uint16 else v) for k, v in w.items()}
    return O.gpt2_forward(f, ids, cfg.n_layer, cfg.n_head, cfg.eps, threads=8)


@pytest.fixture(scope="module")
def be():
    from tensor_cuda.backend import CudaBackend
    from tensor_cuda.runtime import Device
    return CudaBackend(Device.shared(0))


def run_model(be, cfg, w, ids):
    from tensor_cuda.backend import host
    from tensor_cuda.gpt2 import GPT2
    model = GPT2(be, cfg, w)
    t = be.from_host_sync(host("i32", ids.shape, ids))
    out = be.read_sync(model.forward(t))
    return bf16_bits_to_f32(out.data).reshape(out.shape)


@pytest.mark.parametrize("dims", [dict(n_layer=2, d_model=128, n_head=2, d_ff=512, vocab=1001, n_ctx=256, B=2, L=128),
                                  dict(n_layer=1, d_model=768, n_head=12, d_ff=3072, vocab=50257, n_ctx=1024, B=1,
                                       L=64)])
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
    err = np.abs(got.astype(np.float64) - want)
    scale = np.abs(want).max()
    rms = math.sqrt(float(np.mean(err ** 2)) / float(np.mean(want.astype(np.float64) ** 2)))
    assert err.max() <= 3e-2 * scale, (err.max(), scale)
    assert rms <= 1e-2, rms


def test_full_size_forward_is_finite_and_deterministic(be):
    from tensor_cuda.gpt2 import GPT2Config, random_weights
    cfg = GPT2Config()
    w = random_weights(cfg, seed=1)
    ids = O.randint_i32(2 * 1024, 3, cfg.vocab).reshape(2, 1024)
    a = run_model(be, cfg, w, ids)
    b = run_model(be, cfg, w, ids)
    assert a.shape == (2, 1024, cfg.vocab) and np.all(np.isfinite(a))
    assert np.array_equal(a, b)
