"""The C ABI boundary without a GPU: the library loads, exports exactly what include/*.h declares,
and the ctypes layouts match the C structs."""
import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mathplus_cuda.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mpc_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from tensor_cuda import _ffi as F
    return F.load()


def test_library_loads_and_reports_version(lib):
    assert lib.mpc_version() == 1


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 40
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", lib._name], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (\w+)$", out, flags=re.M)))
    assert exported == names, set(exported) ^ set(names)


def test_ctypes_signature_table_covers_the_header():
    from tensor_cuda import _ffi as F
    assert sorted(F.SIGNATURES) == declared_functions()


def test_struct_layouts_match_the_header():
    from tensor_cuda import _ffi as F
    prog = r'''
#include <stdio.h>
#include <stddef.h>
#include "mathplus_cuda.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu\n", sizeof(mpc_gemm_desc), offsetof(mpc_gemm_desc, alpha),
         offsetof(mpc_gemm_desc, batch_shape), offsetof(mpc_gemm_desc, b_batch_stride), sizeof(mpc_sdpa_desc));
  printf("%zu %zu %zu\n", offsetof(mpc_sdpa_desc, scale), offsetof(mpc_sdpa_desc, mask_strides),
         sizeof(mpc_device_info_t));
  printf("%zu %zu\n", sizeof(mpc_gemm_caps), offsetof(mpc_gemm_caps, max_dim));
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(prog)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()
    vals = [int(v) for v in out]
    assert vals[0] == C.sizeof(F.GemmDesc)
    assert vals[1] == F.GemmDesc.alpha.offset
    assert vals[2] == F.GemmDesc.batch_shape.offset
    assert vals[3] == F.GemmDesc.b_batch_stride.offset
    assert vals[4] == C.sizeof(F.SdpaDesc)
    assert vals[5] == F.SdpaDesc.scale.offset
    assert vals[6] == F.SdpaDesc.mask_strides.offset
    assert vals[7] == C.sizeof(F.DeviceInfo)
    from tensor_cuda.caps import GemmCapsStruct
    assert vals[8] == C.sizeof(GemmCapsStruct)
    assert vals[9] == GemmCapsStruct.max_dim.offset


def test_calls_fail_with_status_not_abort(lib):
    """Every call returns a status (lib.rs:17-38 'defined failure, not panic'), with a message."""
    from tensor_cuda import _ffi as F
    n = C.c_int(-1)
    assert lib.mpc_device_count(C.byref(n)) == F.OK and n.value >= 0
    h = C.c_void_p()
    rc = lib.mpc_device_create(0, 0, C.byref(h))
    if n.value == 0:
        assert rc == F.ERR_NO_DEVICE and h.value is None
        assert "no CUDA device" in F.last_error()
    assert lib.mpc_gemm(None, None, None, None, None, None, None) == F.ERR_INVALID
    assert "null device" in F.last_error()
    assert lib.mpc_device_count(None) == F.ERR_INVALID
    assert lib.mpc_comm_init(None, 2, 0, None, None) == F.ERR_INVALID
    assert lib.mpc_comm_init_timeout(None, 2, 0, None, C.c_int64(1000), None) == F.ERR_INVALID
    assert lib.mpc_gemm_capabilities(None, None) == F.ERR_INVALID


def test_missing_library_raises_instead_of_falling_back(tmp_path):
    from tensor_cuda import _ffi as F
    with pytest.raises(OSError, match="not found"):
        F.load(str(tmp_path / "nope.so"))


def test_typescript_symbol_tables_cover_the_header():
    """The Deno.dlopen / bun:ffi tables generated for the TypeScript package name every function
    of the header with one FFI type per C parameter; descriptor structs and out-parameters are
    buffers, device pointers and handles opaque pointers, the waits nonblocking."""
    from tensor_cuda import ts_symbols as T
    deno, bun = T.table(), T.table(bun=True)
    assert sorted(deno) == declared_functions() == sorted(bun)
    assert deno["mpc_gemm"] == {"parameters": ["pointer", "buffer", "pointer", "pointer", "pointer", "pointer",
                                                "pointer"], "result": "i32"}
    assert deno["mpc_device_create"]["parameters"] == ["i32", "u32", "buffer"]
    assert deno["mpc_alloc"]["parameters"] == ["pointer", "usize", "buffer"]
    assert deno["mpc_layer_norm"]["parameters"][5] == "f32" and deno["mpc_rope"]["parameters"][7] == "f64"
    assert deno["mpc_stream_sync"].get("nonblocking") and deno["mpc_sync"].get("nonblocking")
    assert deno["mpc_last_error"]["result"] == "pointer" and bun["mpc_last_error"]["returns"] == "ptr"
    assert bun["mpc_gemm"]["args"][1] == "ptr" and bun["mpc_alloc"]["args"][1] == "u64"
    src = T.render()
    assert src.count("parameters:") == len(deno) and src.count("{") == src.count("}")
    assert T.render(bun=True).count("FFIType.i32") >= len(bun)
