"""Shared helpers for the tests: half-precision encodings and error bounds."""
import numpy as np


def f32_to_bf16_bits(x) -> np.ndarray:
    """Round f32 to bfloat16 bits, nearest-even (finite inputs)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.ascontiguousarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_device_dtype(x, dtype: str):
    """(array to upload, exact f32 value of what the device sees)."""
    x = np.ascontiguousarray(x, np.float32)
    if dtype == "f32":
        return x, x
    if dtype == "f16":
        h = x.astype(np.float16)
        return h, h.astype(np.float32)
    bits = f32_to_bf16_bits(x)
    return bits, bf16_bits_to_f32(bits)


def from_device_dtype(arr, dtype: str) -> np.ndarray:
    if dtype == "f32":
        return np.asarray(arr, np.float32)
    if dtype == "f16":
        return np.asarray(arr).view(np.float16).astype(np.float32)
    return bf16_bits_to_f32(np.asarray(arr).view(np.uint16))


NP_STORAGE = {"f32": np.float32, "f16": np.float16, "bf16": np.uint16}

# Relative rounding of one store into the output dtype.
OUT_ROUND = {"f32": 6e-8, "f16": 4.9e-4, "bf16": 3.9e-3}


def gemm_bound(want, absprod, dtype_in: str, dtype_out: str):
    """Per-element bound of packages/tensor-webgpu/test/gemm.test.ts:120-129, generalised:
    f32 accumulation over exact inputs (1e-5·(|A||B|) for 3xTF32 f32 inputs, 2e-5·(|A||B|) for
    half inputs) plus one rounding of the result into the output dtype."""
    acc = 1e-5 if dtype_in == "f32" else 2e-5
    return OUT_ROUND[dtype_out] * np.abs(want) + acc * absprod + 1e-7
