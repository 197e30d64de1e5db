"""A GPT-2-small-shaped forward pass on the device, composed from the Backend ops of the GEMM /
attention path.

The block is the reference's pre-norm transformer layer (``TransformerEncoderLayer.forward`` with
``normFirst``, packages/tensor-autograd/src/transformer.ts:320-333: ``x = x + sa(norm1(x))``,
``x = x + ff(norm2(x))``, exact-erf GELU) with causal self-attention laid out like its
``MultiheadAttention`` (transformer.ts:173-242: packed ``in_proj_weight [3E, E]``, heads split as
``[N, L, H, D] -> [N, H, L, D]``, ``out_proj`` on the merged heads). GPT-2's token + position
embeddings lead in and a final LayerNorm and the tied LM head (``linear`` with the token table)
lead out.

Every step is one device op: ``embedding``, ``add``, ``layerNorm``, ``linear`` (bias, GELU for the
first MLP projection and the residual adds in the GEMM's epilogue) and ``sdpa_packed`` (causal
attention reading Q / K / V straight from the packed in-projection and writing the heads merged). Activations and weight matrices are bf16; biases and LayerNorm
parameters f32; every GEMM accumulates in f32.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from .backend import CudaBackend, CudaTensor, host


@dataclass(frozen=True)
class GPT2Config:
    n_layer: int = 12
    d_model: int = 768
    n_head: int = 12
    d_ff: int = 3072
    vocab: int = 50257
    n_ctx: int = 1024
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_head

    def forward_flop(self, batch: int, seq: int) -> float:
        """Dense FLOP of one forward: the four linears per layer, causal attention (half of
        4*L^2*D per head) and the LM head."""
        d, f = self.d_model, self.d_ff
        per_token = self.n_layer * 2 * (d * 3 * d + d * d + 2 * d * f) + 2 * d * self.vocab
        attn = self.n_layer * 0.5 * 4 * seq * seq * d  # per sequence, all heads
        return batch * (seq * per_token + attn)


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def random_weights(cfg: GPT2Config, seed: int = 0, std: float = 0.02) -> dict:
    """Host weights: matrices ~ N(0, std) rounded to bf16 (uint16 bits), biases ~ N(0, std) and
    LayerNorm weight 1 / bias 0 in f32. Keys follow GPT-2's parameter names."""
    rng = np.random.default_rng(seed)
    d, f = cfg.d_model, cfg.d_ff
    mat = lambda *shape: _bf16_bits(rng.standard_normal(shape, dtype=np.float32) * std)
    vec = lambda n: (rng.standard_normal(n, dtype=np.float32) * std).astype(np.float32)
    w = {"wte": mat(cfg.vocab, d), "wpe": mat(cfg.n_ctx, d),
         "ln_f.weight": np.ones(d, np.float32), "ln_f.bias": np.zeros(d, np.float32)}
    for i in range(cfg.n_layer):
        p = f"h.{i}."
        w[p + "ln_1.weight"] = np.ones(d, np.float32)
        w[p + "ln_1.bias"] = np.zeros(d, np.float32)
        w[p + "attn.in_proj_weight"] = mat(3 * d, d)
        w[p + "attn.in_proj_bias"] = vec(3 * d)
        w[p + "attn.out_proj.weight"] = mat(d, d)
        w[p + "attn.out_proj.bias"] = vec(d)
        w[p + "ln_2.weight"] = np.ones(d, np.float32)
        w[p + "ln_2.bias"] = np.zeros(d, np.float32)
        w[p + "mlp.fc.weight"] = mat(f, d)
        w[p + "mlp.fc.bias"] = vec(f)
        w[p + "mlp.proj.weight"] = mat(d, f)
        w[p + "mlp.proj.bias"] = vec(d)
    return w


class GPT2:
    """The model's weights resident on one device and its forward pass."""

    def __init__(self, backend: CudaBackend, cfg: GPT2Config, weights: dict):
        """``weights``: host arrays (uint16 = bf16 bits, else f32), uploaded here, or device
        tensors (``CudaTensor``, e.g. from ``safetensors.gpt2_device_weights``), taken as they are."""
        self.backend, self.cfg = backend, cfg
        self.w: dict[str, CudaTensor] = {}
        for name, arr in weights.items():
            if isinstance(arr, CudaTensor):
                self.w[name] = arr
                continue
            dtype = "bf16" if arr.dtype == np.uint16 else "f32"
            self.w[name] = backend.from_host_sync(host(dtype, arr.shape, arr))
        self._pos: dict[int, CudaTensor] = {}

    @classmethod
    def from_safetensors(cls, backend: CudaBackend, cfg: GPT2Config, source) -> "GPT2":
        """A Hugging Face GPT-2 checkpoint (a ``.safetensors`` path or its bytes) on the device."""
        from .safetensors import gpt2_device_weights
        return cls(backend, cfg, gpt2_device_weights(source, backend, cfg.n_layer))

    def _positions(self, seq: int) -> CudaTensor:
        if seq not in self._pos:
            self._pos[seq] = self.backend.from_host_sync(host("i32", (seq,), np.arange(seq, dtype=np.int32)))
        return self._pos[seq]

    def forward(self, ids: CudaTensor, stop_after: int | None = None) -> CudaTensor:
        """ids i32 [B, L] -> logits bf16 [B, L, vocab]; with ``stop_after`` = n, the residual stream
        bf16 [B, L, d_model] after the first n blocks instead (no final LayerNorm or LM head)."""
        be, cfg, w = self.backend, self.cfg, self.w
        B, L = ids.shape
        if L > cfg.n_ctx:
            raise ValueError(f"GPT2: sequence of {L} tokens is longer than the context ({cfg.n_ctx})")
        if stop_after is not None and not 0 <= stop_after <= cfg.n_layer:
            raise ValueError(f"GPT2: stop_after={stop_after} outside 0..{cfg.n_layer}")
        D, H, Dh = cfg.d_model, cfg.n_head, cfg.head_dim
        tok = be.embedding(w["wte"], ids)                      # [B, L, D]
        pos = be.embedding(w["wpe"], self._positions(L))      # [L, D]
        s = be.add(tok, pos)
        x = be.reshape(s, (B * L, D))
        for t in (tok, pos, s):
            be.dispose(t)
        for i in range(cfg.n_layer if stop_after is None else stop_after):
            p = f"h.{i}."
            x = self._block(x, p, B, L, D, H, Dh)
        if stop_after is not None:
            out = be.reshape(x, (B, L, D))
            be.dispose(x)
            return out
        h = be.layerNorm(x, w["ln_f.weight"], w["ln_f.bias"], cfg.eps)
        be.dispose(x)
        logits = be.linear(h, w["wte"])                        # tied LM head: x . wte^T
        out = be.reshape(logits, (B, L, cfg.vocab))
        be.dispose(logits)
        be.dispose(h)
        return out

    def _block(self, x: CudaTensor, p: str, B: int, L: int, D: int, H: int, Dh: int) -> CudaTensor:
        be, w, eps = self.backend, self.w, self.cfg.eps
        tmp = []
        h = be.layerNorm(x, w[p + "ln_1.weight"], w[p + "ln_1.bias"], eps)
        qkv = be.linear(h, w[p + "attn.in_proj_weight"], w[p + "attn.in_proj_bias"])      # [B*L, 3D]
        qkv3 = be.reshape(qkv, (B, L, 3 * D))                                              # [B, L, 3, H, Dh]
        a = be.sdpa_packed(qkv3, H, 1.0 / math.sqrt(Dh), causal=True)                     # [B, L, H*Dh]
        merged = be.reshape(a, (B * L, D))
        o = be.linear(merged, w[p + "attn.out_proj.weight"], w[p + "attn.out_proj.bias"])
        x1 = be.add(x, o)
        tmp += [h, qkv, qkv3, a, merged, o]
        h2 = be.layerNorm(x1, w[p + "ln_2.weight"], w[p + "ln_2.bias"], eps)
        f = be.linear(h2, w[p + "mlp.fc.weight"], w[p + "mlp.fc.bias"], activation="gelu")  # [B*L, d_ff]
        g = be.linear(f, w[p + "mlp.proj.weight"], w[p + "mlp.proj.bias"])
        x2 = be.add(x1, g)
        tmp += [h2, f, g, x1, x]
        for t in tmp:
            be.dispose(t)
        return x2
