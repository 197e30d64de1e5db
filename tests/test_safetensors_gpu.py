"""safetensors files into device memory on the B200: every device dtype read back bit for bit,
dtypes without a device form refused before anything is copied, and a GPT-2 checkpoint in the
Hugging Face layout (``Conv1D`` weights [in, out], f32) loaded, transposed and cast on the device,
giving logits bit-identical to the same weights prepared on the host."""
import numpy as np
import pytest

from tensor_cuda import safetensors as st

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from tensor_cuda.backend import CudaBackend
    from tensor_cuda.runtime import Device
    return CudaBackend(Device.shared(0))


def test_every_device_dtype_round_trips(be, tmp_path):
    rng = np.random.default_rng(0)
    tensors = {
        "f32": ("F32", rng.standard_normal((37, 129)).astype(np.float32)),
        "f16": ("F16", rng.standard_normal(1001).astype(np.float16)),
        "bf16": ("BF16", rng.integers(0, 2 ** 16, (3, 5, 7), dtype=np.uint16)),
        "i32": ("I32", rng.integers(-2 ** 31, 2 ** 31, 77, dtype=np.int32)),
        "mask": ("BOOL", rng.integers(0, 2, (4, 4), dtype=np.uint8)),
        "empty": ("F32", np.zeros((0, 5), np.float32)),
        "scalar": ("F32", np.array(2.5, np.float32)),
    }
    p = tmp_path / "mixed.safetensors"
    st.write(p, tensors)
    dev = st.load_to_device(str(p), be)
    try:
        assert sorted(dev) == sorted(tensors)
        for name, (dtype, arr) in tensors.items():
            h = be.read_sync(dev[name])
            assert h.dtype == st.DEVICE[dtype] and tuple(h.shape) == arr.shape, name
            assert h.data.tobytes() == arr.tobytes(), name
        # a subset, from bytes in memory
        sub = st.load_to_device(p.read_bytes(), be, ["bf16"])
        assert list(sub) == ["bf16"] and be.read_sync(sub["bf16"]).data.tobytes() == tensors["bf16"][1].tobytes()
    finally:
        for t in dev.values():
            be.dispose(t)


def test_dtype_without_device_form_is_refused(be):
    data = st.serialize({"a": ("F32", np.ones(4, np.float32)), "d": ("F64", np.ones(2))})
    with pytest.raises(st.SafetensorsError) as e:
        st.load_to_device(data, be)
    assert e.value.code == "InvalidDtype"
    assert be.read_sync(st.load_to_device(data, be, ["a"])["a"]).data.tolist() == [1, 1, 1, 1]


def hf_checkpoint(cfg, seed=0, prefix=""):
    """A GPT-2 checkpoint in the Hugging Face layout: Conv1D weights [in, out], everything f32."""
    rng = np.random.default_rng(seed)
    d, f = cfg.d_model, cfg.d_ff
    r = lambda *s: (rng.standard_normal(s) * 0.02).astype(np.float32)
    w = {"wte.weight": r(cfg.vocab, d), "wpe.weight": r(cfg.n_ctx, d),
         "ln_f.weight": 1 + r(d), "ln_f.bias": r(d)}
    for i in range(cfg.n_layer):
        p = f"h.{i}."
        w.update({p + "ln_1.weight": 1 + r(d), p + "ln_1.bias": r(d), p + "ln_2.weight": 1 + r(d),
                  p + "ln_2.bias": r(d), p + "attn.c_attn.weight": r(d, 3 * d), p + "attn.c_attn.bias": r(3 * d),
                  p + "attn.c_proj.weight": r(d, d), p + "attn.c_proj.bias": r(d),
                  p + "mlp.c_fc.weight": r(d, f), p + "mlp.c_fc.bias": r(f),
                  p + "mlp.c_proj.weight": r(f, d), p + "mlp.c_proj.bias": r(d)})
    return {prefix + k: v for k, v in w.items()}


def host_weights(cfg, hf):
    """The same weights prepared on the host: Conv1D transposed to [out, in], matrices rounded to
    bf16 (nearest even)."""
    from tensor_cuda.gpt2 import _bf16_bits
    w = {"wte": _bf16_bits(hf["wte.weight"]), "wpe": _bf16_bits(hf["wpe.weight"]),
         "ln_f.weight": hf["ln_f.weight"], "ln_f.bias": hf["ln_f.bias"]}
    names = {"attn.c_attn": ("attn.in_proj_weight", "attn.in_proj_bias"),
             "attn.c_proj": ("attn.out_proj.weight", "attn.out_proj.bias"),
             "mlp.c_fc": ("mlp.fc.weight", "mlp.fc.bias"), "mlp.c_proj": ("mlp.proj.weight", "mlp.proj.bias")}
    for i in range(cfg.n_layer):
        p = f"h.{i}."
        for n in ("ln_1.weight", "ln_1.bias", "ln_2.weight", "ln_2.bias"):
            w[p + n] = hf[p + n]
        for src, (wn, bn) in names.items():
            w[p + wn] = _bf16_bits(np.ascontiguousarray(hf[p + src + ".weight"].T)).reshape(hf[p + src + ".weight"].T.shape)
            w[p + bn] = hf[p + src + ".bias"]
    return w


@pytest.mark.parametrize("prefix", ["", "transformer."])
def test_gpt2_checkpoint_matches_host_prepared_weights(be, tmp_path, prefix):
    from tensor_cuda.backend import host
    from tensor_cuda.gpt2 import GPT2, GPT2Config
    cfg = GPT2Config(n_layer=2, d_model=128, n_head=2, d_ff=512, vocab=1000, n_ctx=256)
    hf = hf_checkpoint(cfg, seed=1)
    tensors = {prefix + k: ("F32", v) for k, v in hf.items()}
    if prefix:
        tensors["lm_head.weight"] = ("F32", hf["wte.weight"])  # tied, not loaded
    p = tmp_path / "gpt2.safetensors"
    st.write(p, tensors, {"format": "pt"})
    ids = np.random.default_rng(2).integers(0, cfg.vocab, (2, 128)).astype(np.int32)
    dev_ids = be.from_host_sync(host("i32", ids.shape, ids))
    a = GPT2.from_safetensors(be, cfg, str(p))
    b = GPT2(be, cfg, host_weights(cfg, hf))
    for k in b.w:
        assert a.w[k].dtype == b.w[k].dtype and tuple(a.w[k].shape) == tuple(b.w[k].shape), k
        assert be.read_sync(a.w[k]).data.tobytes() == be.read_sync(b.w[k]).data.tobytes(), k
    la, lb = be.read_sync(a.forward(dev_ids)).data, be.read_sync(b.forward(dev_ids)).data
    assert la.tobytes() == lb.tobytes()
    assert np.isfinite((la.view(np.uint16).astype(np.uint32) << 16).view(np.float32)).all()


def test_gpt2_checkpoint_missing_tensor(be):
    from tensor_cuda.gpt2 import GPT2Config
    cfg = GPT2Config(n_layer=1, d_model=64, n_head=1, d_ff=256, vocab=100, n_ctx=64)
    hf = hf_checkpoint(cfg)
    del hf["h.0.mlp.c_fc.bias"]
    with pytest.raises(st.SafetensorsError) as e:
        st.gpt2_device_weights(st.serialize({k: ("F32", v) for k, v in hf.items()}), be, cfg.n_layer)
    assert e.value.code == "TensorNotFound"
