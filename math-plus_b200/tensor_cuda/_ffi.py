"""ctypes binding of libmathplus_cuda.so (include/mathplus_cuda.h).

This is the Python twin of the symbol table a math-plus TypeScript facade would hand to
``Deno.dlopen`` / ``bun:ffi`` (the style of packages/tensor-wasm/src/native.ts:48-70): one
entry per exported C function, with its argument and result types. There is no fallback: if
the library is missing, loading raises, and every non-zero status raises :class:`MpcError`
carrying ``mpc_last_error()``.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
_PKG = os.path.dirname(_HERE)
DEFAULT_LIB = os.path.join(_PKG, "lib", "libmathplus_cuda.so")

# mpc_status
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_OOM, ERR_CUDA, ERR_TIMEOUT, ERR_POISONED, ERR_NO_DEVICE, ERR_COMM, ERR_COMPILE = range(10)
STATUS_NAMES = {0: "OK", 1: "INVALID", 2: "UNSUPPORTED", 3: "OOM", 4: "CUDA", 5: "TIMEOUT", 6: "POISONED",
                7: "NO_DEVICE", 8: "COMM", 9: "COMPILE"}
# mpc_dtype
F32, F16, BF16, I32, BOOL = range(5)
FUSED_F32 = 1  # MPC_FUSED_F32
DTYPE_CODES = {"f32": F32, "f16": F16, "bf16": BF16, "i32": I32, "bool": BOOL}
DTYPE_BYTES = {F32: 4, F16: 2, BF16: 2, I32: 4, BOOL: 1}
EPI_BIAS, EPI_GELU, EPI_RESIDUAL = 1, 2, 4
B_KN, B_NK = 0, 1
MASK_NONE, MASK_BOOL, MASK_ADD = 0, 1, 2
# mpc op codes (include/mathplus_cuda.h)
UNARY_OPS = {name: i + 1 for i, name in enumerate(
    ["neg", "abs", "exp", "log", "sqrt", "rsqrt", "tanh", "sigmoid", "relu", "erf", "scale", "pow_scalar",
     "logicalNot"])}
BINARY_OPS = {name: i + 32 for i, name in enumerate(
    ["add", "sub", "mul", "div", "maximum", "pow", "equal", "notEqual", "less", "lessEqual", "greater",
     "greaterEqual", "logicalAnd", "logicalOr"])}
REDUCE_OPS = {name: i + 64 for i, name in enumerate(["sum", "mean", "max", "min", "argmax", "argmin"])}


class MpcError(RuntimeError):
    def __init__(self, status: int, where: str, message: str):
        self.status = status
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}: {message}")


class DeviceInfo(C.Structure):
    _fields_ = [("name", C.c_char * 128), ("ordinal", C.c_int), ("cc_major", C.c_int), ("cc_minor", C.c_int),
                ("sm_count", C.c_int), ("total_bytes", C.c_size_t), ("smem_per_block_optin", C.c_size_t),
                ("runtime_version", C.c_int), ("driver_version", C.c_int)]


class SdpaLayout(C.Structure):
    """mpc_sdpa_layout: element strides of (batch, head, row) for Q, K, V and O."""
    _fields_ = [("q", C.c_int64 * 3), ("k", C.c_int64 * 3), ("v", C.c_int64 * 3), ("o", C.c_int64 * 3)]


class GemmDesc(C.Structure):
    _fields_ = [("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64), ("dtype_in", C.c_int32),
                ("dtype_out", C.c_int32), ("b_layout", C.c_int32), ("epilogue", C.c_int32), ("alpha", C.c_float),
                ("batch_rank", C.c_int32), ("batch_shape", C.c_int64 * 4), ("a_batch_stride", C.c_int64 * 4),
                ("b_batch_stride", C.c_int64 * 4)]


class SdpaDesc(C.Structure):
    _fields_ = [("b", C.c_int64), ("h", C.c_int64), ("hk", C.c_int64), ("lq", C.c_int64), ("lk", C.c_int64),
                ("d", C.c_int64), ("dv", C.c_int64), ("dtype", C.c_int32), ("causal", C.c_int32),
                ("scale", C.c_float), ("mask_kind", C.c_int32), ("mask_strides", C.c_int64 * 4)]


_vp, _sz, _i32, _i64, _u64 = C.c_void_p, C.c_size_t, C.c_int32, C.c_int64, C.c_uint64
_dev = C.c_void_p

# name -> argtypes (every function returns an int status unless listed in _RESTYPE)
SIGNATURES = {
    "mpc_version": [],
    "mpc_device_count": [C.POINTER(C.c_int)],
    "mpc_device_create": [C.c_int, C.c_uint, C.POINTER(_dev)],
    "mpc_device_destroy": [_dev],
    "mpc_device_info": [_dev, C.POINTER(DeviceInfo)],
    "mpc_last_error": [_dev],
    "mpc_device_status": [_dev],
    "mpc_set_wait_timeout_ns": [_dev, _u64],
    "mpc_device_clear_error": [_dev],
    "mpc_selftest_wait_timeout": [_dev, _u64],
    "mpc_alloc": [_dev, _sz, C.POINTER(_vp)],
    "mpc_free": [_dev, _vp],
    "mpc_set_alloc_limit": [_dev, _sz],
    "mpc_alloc_stats": [_dev, C.POINTER(_sz), C.POINTER(_sz)],
    "mpc_trim": [_dev],
    "mpc_host_alloc": [_dev, _sz, C.POINTER(_vp)],
    "mpc_host_free": [_dev, _vp],
    "mpc_memcpy_h2d_async": [_dev, _vp, _vp, _sz, _vp],
    "mpc_memcpy_d2h_async": [_dev, _vp, _vp, _sz, _vp],
    "mpc_memcpy_d2d_async": [_dev, _vp, _vp, _sz, _vp],
    "mpc_memset_async": [_dev, _vp, C.c_int, _sz, _vp],
    "mpc_stream_create": [_dev, C.POINTER(_vp)],
    "mpc_stream_destroy": [_dev, _vp],
    "mpc_stream_sync": [_dev, _vp],
    "mpc_device_stream": [_dev, C.POINTER(_vp)],
    "mpc_event_create": [_dev, C.POINTER(_vp)],
    "mpc_event_destroy": [_dev, _vp],
    "mpc_event_record": [_dev, _vp, _vp],
    "mpc_stream_wait_event": [_dev, _vp, _vp],
    "mpc_event_elapsed_ms": [_dev, _vp, _vp, C.POINTER(C.c_float)],
    "mpc_sync": [_dev],
    "mpc_launch_count": [_dev, C.POINTER(_u64)],
    "mpc_gemm": [_dev, C.POINTER(GemmDesc), _vp, _vp, _vp, _vp, _vp],
    "mpc_sdpa_strided": [_dev, C.POINTER(SdpaDesc), _vp, _vp, _vp, _vp, _vp, _vp, C.POINTER(SdpaLayout), _vp],
    "mpc_unary": [_dev, _i32, _vp, _i32, _vp, _i32, _i64, C.c_float, _vp],
    "mpc_binary": [_dev, _i32, _vp, _vp, _i32, _vp, _i32, _i32, C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64), _vp],
    "mpc_where": [_dev, _vp, _vp, _vp, _i32, _vp, _i32, C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64),
                  C.POINTER(_i64), _vp],
    "mpc_reduce": [_dev, _i32, _vp, _i32, _vp, _i32, _i64, _i64, _i64, _vp],
    "mpc_cumsum": [_dev, _vp, _i32, _vp, _i32, _i64, _i64, _i64, _vp],
    "mpc_strided_copy": [_dev, _vp, C.POINTER(_i64), _vp, C.POINTER(_i64), _i32, _i32, C.POINTER(_i64), _vp],
    "mpc_sort": [_dev, _vp, _i32, _vp, _i64, _i64, _i64, _vp],
    "mpc_fused_create": [_dev, C.POINTER(_i32), _i32, C.POINTER(C.c_double), _i32, _i32, C.POINTER(_i32),
                         C.POINTER(_vp)],
    "mpc_fused_create_ex": [_dev, C.POINTER(_i32), _i32, C.POINTER(C.c_double), _i32, _i32, C.POINTER(_i32),
                            C.c_uint32, C.POINTER(_vp)],
    "mpc_fused_run": [_vp, C.POINTER(_vp), _i32, C.POINTER(_i64), C.POINTER(_i64), _vp, _vp],
    "mpc_fused_destroy": [_vp],
    "mpc_fused_lower": [C.POINTER(_i32), _i32, C.POINTER(C.c_double), _i32, _i32, C.POINTER(_i32), C.c_uint32, _i32,
                        C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)],
    "mpc_gather_rows": [_dev, _vp, _i32, _vp, _vp, _i64, _i64, _i64, _i64, C.POINTER(_i64), _vp],
    "mpc_rope": [_dev, _vp, _i32, _vp, _i64, _i64, _i64, C.c_double, _vp],
    "mpc_geglu": [_dev, _vp, _i32, _vp, _i64, _i64, _vp],
    "mpc_mean_pool": [_dev, _vp, _i32, _vp, _i32, _vp, _i64, _i64, _i64, _vp],
    "mpc_gemm_residual": [_dev, C.POINTER(GemmDesc), _vp, _vp, _vp, _vp, _vp, _vp],
    "mpc_gemm_capabilities": [_dev, _vp],
    "mpc_gemm_f32_noalloc": [C.POINTER(GemmDesc), _vp, _vp, _vp, _vp, _vp],
    "mpc_gemm_f32_noalloc_status": [_vp],
    "mpc_gemm_f32_noalloc_selftest": [_u64, _vp],
    "mpc_sdpa": [_dev, C.POINTER(SdpaDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "mpc_softmax": [_dev, _vp, _i32, _vp, _i64, _i64, _i64, _vp],
    "mpc_gelu": [_dev, _vp, _i32, _vp, _i32, _i64, _vp],
    "mpc_add": [_dev, _vp, _vp, _vp, _i32, _i64, _i64, _vp],
    "mpc_layer_norm": [_dev, _vp, _i32, _vp, _vp, C.c_float, _vp, _i32, _i64, _i64, _vp],
    "mpc_embedding": [_dev, _vp, _i32, _vp, _vp, _i64, _i64, _i64, C.POINTER(_i64), _vp],
    "mpc_cast": [_dev, _vp, _i32, _vp, _i32, _i64, _vp],
    "mpc_transpose": [_dev, _vp, _vp, _i32, _i32, C.POINTER(_i64), C.POINTER(_i32), _vp],
    "mpc_comm_unique_id": [_vp],
    "mpc_comm_init": [_dev, C.c_int, C.c_int, _vp, C.POINTER(_vp)],
    "mpc_comm_init_timeout": [_dev, C.c_int, C.c_int, _vp, _i64, C.POINTER(_vp)],
    "mpc_comm_destroy": [_vp],
    "mpc_comm_abort": [_vp],
    "mpc_allgather": [_vp, _vp, _vp, _sz, _vp],
    "mpc_peer_buffer_create": [_vp, _sz, C.POINTER(_vp)],
    "mpc_peer_buffer_ptr": [_vp, C.c_int, C.POINTER(_vp)],
    "mpc_peer_barrier": [_vp, _vp],
    "mpc_peer_buffer_destroy": [_vp],
    "mpc_gemm_multi_store": [_dev, C.POINTER(GemmDesc), _vp, _vp, _vp, C.POINTER(_vp), _i32, _i64, _i64, _vp],
    "mpc_gemm_allgather": [_dev, C.POINTER(GemmDesc), _vp, _vp, _vp, _vp, _vp, _vp],
}
_RESTYPE = {"mpc_last_error": C.c_char_p}

_lib = None
_lib_path = None


def library_path() -> str:
    """Resolution order of packages/tensor-wasm/src/native.ts:78-89: explicit env var, then in-tree."""
    return os.environ.get("MATH_PLUS_CUDA_LIB_PATH") or DEFAULT_LIB


def load(path: str | None = None) -> C.CDLL:
    global _lib, _lib_path
    if _lib is not None and (path is None or path == _lib_path):
        return _lib
    p = path or library_path()
    if not os.path.exists(p):
        raise OSError(f"libmathplus_cuda.so not found at {p} (build it: python math-plus_b200/build.py)")
    lib = C.CDLL(p)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, C.c_int)
    _lib, _lib_path = lib, p
    return lib


def last_error() -> str:
    msg = load().mpc_last_error(None)
    return msg.decode("utf-8", "replace") if msg else ""


def check(status: int, where: str) -> None:
    if status != OK:
        raise MpcError(status, where, last_error())


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
