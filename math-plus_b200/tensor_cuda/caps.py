"""What the GEMM uses on a device, and when a host-array GEMM is worth sending to it.

The reference's WebGPU facade keeps the same two pieces: ``gemmCapabilities(device)``, a record of
the optional features its GEMM may use on a device (packages/tensor-webgpu/src/gemm-caps.ts:60-86),
and ``chooseGemmBackend(m, n, k)``, a MEASURED crossover below which a host-array matmul stays on
the CPU because the device's per-call floor dominates (packages/tensor-webgpu/src/threshold.ts:67-85).

Both are advisory, as in the reference: nothing here routes work anywhere. ``DeviceArray.matmul``
and every Backend op always run on the device; a caller holding host arrays may consult
``choose_gemm_backend`` to decide whether to upload at all.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _ffi as F


class GemmCapsStruct(C.Structure):
    """mpc_gemm_caps (include/mathplus_cuda.h)."""
    _fields_ = [("f16", C.c_int32), ("bf16", C.c_int32), ("f32_3xtf32", C.c_int32), ("cta_pairs", C.c_int32),
                ("sm_count", C.c_int32), ("pair_min_tiles", C.c_int32), ("tf32_narrow_below", C.c_int32),
                ("attention_tc_head_dims", C.c_int32), ("attention_max_head_dim", C.c_int32),
                ("reserved", C.c_int32), ("max_dim", C.c_int64)]


@dataclass(frozen=True)
class GemmCapabilities:
    """What GEMM (and attention) will use on a device."""
    f16: bool                    # f16 operands on tcgen05 (f32 accumulation)
    bf16: bool                   # bf16 operands on tcgen05 (f32 accumulation)
    f32_3xtf32: bool             # f32 operands as 3xTF32 (held to f32 accuracy)
    cta_pairs: bool              # 256 x 256 tiles on two SMs (cta_group::2)
    sm_count: int
    pair_min_tiles: int          # f16 / bf16 problems with at least this many 256 x 256 tiles run on pairs
    tf32_narrow_below: int       # f32 problems with fewer 128 x 128 tiles run 128 x 64 tiles
    attention_head_dims: tuple   # head dims of the tensor-core attention path
    attention_max_head_dim: int  # largest head dim of the CUDA-core attention path
    max_dim: int                 # largest M, N, K


def gemm_capabilities(device) -> GemmCapabilities:
    """The record for a ``Device`` (runtime) or a ``CudaDevice`` (facade)."""
    dev = getattr(device, "device", device)
    s = GemmCapsStruct()
    F.call("mpc_gemm_capabilities", dev.handle, C.byref(s))
    dims = tuple(d for bit, d in ((1, 64), (2, 128)) if s.attention_tc_head_dims & bit)
    return GemmCapabilities(bool(s.f16), bool(s.bf16), bool(s.f32_3xtf32), bool(s.cta_pairs), s.sm_count,
                            s.pair_min_tiles, s.tf32_narrow_below, dims, s.attention_max_head_dim, s.max_dim)


gemmCapabilities = gemm_capabilities

# ---- the measured crossover ------------------------------------------------------------------
# Measured with ``python bench.py --threshold-sweep`` on a B200 box: end to end per call, as
# threshold.ts prices a host-array matmul (upload A and B from host memory, the f32 GEMM, read C
# back) against the reference's CPU algorithm (tensor-core gemmNT, restated in C) on one host
# thread. The shapes and times are summarised in profiles/gemm_threshold_sweep.txt. Re-run the
# sweep on other hardware before trusting these numbers.

#: Output elements (m·n) below which the CPU path beat the device end to end, whatever k was.
#: (Not binding on the measured shapes: the work test alone separated them.)
GEMM_ELEMENT_THRESHOLD = 8 * 8
#: Multiply-adds (m·n·k) below which the CPU path beat the device end to end: 96^3. The device's
#: per-call floor from host arrays was 62-68 us (two uploads, the split prologue and GEMM, the
#: read-back, a synchronisation); 96^3 took 76 us there against 141 us on one CPU thread, 64^3
#: 67 against 49.
GEMM_WORK_THRESHOLD = 96 ** 3


def choose_gemm_backend(m: int, n: int, k: int | None = None) -> str:
    """``"cuda"`` when BOTH ``m·n >= GEMM_ELEMENT_THRESHOLD`` and ``m·n·k >= GEMM_WORK_THRESHOLD``,
    else ``"cpu"`` (chooseGemmBackend, threshold.ts:67-85: ``k`` optional; omitted, only the m·n
    test applies). Prices host-array calls: operands already on the device make the device the
    better choice at every size. Advisory only."""
    for name, v in (("m", m), ("n", n)) + ((("k", k),) if k is not None else ()):
        if not isinstance(v, int) or v < 0:
            raise ValueError(f"choose_gemm_backend: {name} must be a non-negative integer, got {v!r}")
    elements = m * n
    if elements < GEMM_ELEMENT_THRESHOLD:
        return "cpu"
    if k is not None and elements * k < GEMM_WORK_THRESHOLD:
        return "cpu"
    return "cuda"


chooseGemmBackend = choose_gemm_backend
