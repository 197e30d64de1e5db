"""safetensors header validation and writer on the CPU.

The cases are those of the reference's header tests (packages/safetensors/test/header.test.ts:
18-100) and writer tests (writer.test.ts:7-75), on hand-built files; the reader and writer are
also checked against the Python ``safetensors`` package (the reference's own oracle,
packages/safetensors/scripts/safetensors_oracle.py) where it is installed: files it writes read
back with the same bytes, and ``serialize`` gives its bytes exactly."""
import json
import struct

import numpy as np
import pytest

from tensor_cuda import safetensors as st
from tensor_cuda.safetensors import MAX_HEADER, SafetensorsError, SafetensorsFile, parse_header


def craft(header, data=b"", pad=False) -> bytes:
    """u64 LE header length + header text (+ space padding) + data (the reference's test helper)."""
    text = header if isinstance(header, str) else json.dumps(header, separators=(",", ":"))
    raw = text.encode()
    if pad:
        raw += b" " * ((8 - len(raw) % 8) % 8)
    return struct.pack("<Q", len(raw)) + raw + bytes(data)


def code(fn, expected):
    with pytest.raises(SafetensorsError) as e:
        fn()
    assert e.value.code == expected, str(e.value)


def f32(*v):
    return np.array(v, np.float32).tobytes()


def u8(b, e):
    return {"dtype": "U8", "shape": [e - b], "data_offsets": [b, e]}


def test_minimal_valid_file():
    f = SafetensorsFile(craft({"__metadata__": {"a": "b"}, "x": {"dtype": "F32", "shape": [2],
                                                                 "data_offsets": [0, 8]}}, f32(1, 2), True))
    assert f.metadata == {"a": "b"}
    assert f.names() == ["x"] and f.has("x") and not f.has("y")
    assert f.info("x") == st.TensorInfo("x", "F32", (2,), (0, 8))
    assert f.numpy("x").tolist() == [1.0, 2.0]
    assert f.header.data_length == 8 and f.header.data_start % 8 == 0
    code(lambda: f.info("y"), "TensorNotFound")


def test_empty_header_and_null_metadata():
    assert SafetensorsFile(craft("{}")).names() == []
    f = SafetensorsFile(craft({"__metadata__": None, "x": u8(0, 1)}, bytes([7])))
    assert f.metadata == {} and f.numpy("x").tolist() == [7]


def test_header_length():
    code(lambda: parse_header(bytes(4)), "HeaderTooSmall")
    code(lambda: parse_header(struct.pack("<Q", MAX_HEADER + 1)), "HeaderTooLarge")
    full = craft({"x": u8(0, 1)}, bytes([1]))
    code(lambda: parse_header(full[:20]), "InvalidHeaderLength")
    lying = bytearray(craft("{}"))
    lying[:8] = struct.pack("<Q", 1000)
    code(lambda: SafetensorsFile(bytes(lying)), "InvalidHeaderLength")


def test_header_text():
    bad = bytearray(craft("{}"))
    bad[8] = 0xFF
    code(lambda: SafetensorsFile(bytes(bad)), "InvalidHeader")
    code(lambda: SafetensorsFile(craft(' {"a":1}')), "InvalidHeaderStart")
    code(lambda: SafetensorsFile(craft("[]")), "InvalidHeaderStart")
    code(lambda: SafetensorsFile(craft('{"x": {"dtype": "F32",')), "InvalidHeaderDeserialization")
    code(lambda: SafetensorsFile(craft('{"x": 5}')), "InvalidHeaderDeserialization")
    code(lambda: SafetensorsFile(craft('{"x": []}')), "InvalidHeaderDeserialization")
    code(lambda: SafetensorsFile(craft('{"__metadata__": {"k": 1}}')), "InvalidHeaderDeserialization")
    code(lambda: SafetensorsFile(craft('{"__metadata__": [1]}')), "InvalidHeaderDeserialization")
    code(lambda: SafetensorsFile(craft('{"x": {"dtype": "U8", "shape": [NaN]}}')), "InvalidHeaderDeserialization")
    # an empty object entry is an object: it fails on its dtype
    code(lambda: SafetensorsFile(craft('{"x": {}}')), "InvalidDtype")


def test_duplicate_names():
    text = '{"x":{"dtype":"U8","shape":[1],"data_offsets":[0,1]},"x":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}'
    code(lambda: SafetensorsFile(craft(text, bytes([1]))), "DuplicateTensor")
    # a nested key equal to a tensor name, and escaped quotes in names, are not duplicates
    ok = ('{"__metadata__":{"x":"dtype \\"x\\""},"x":{"dtype":"U8","shape":[1],"data_offsets":[0,1]},'
          '"x\\"":{"dtype":"U8","shape":[0],"data_offsets":[1,1]}}')
    assert SafetensorsFile(craft(ok, bytes([1]))).names() == ["x", 'x"']


def test_per_tensor_validation():
    one = bytes(4)
    code(lambda: SafetensorsFile(craft({"x": {"dtype": "F8_E4M3", "shape": [4], "data_offsets": [0, 4]}}, one)), "InvalidDtype")
    code(lambda: SafetensorsFile(craft({"x": {"dtype": "toString", "shape": [4], "data_offsets": [0, 4]}}, one)), "InvalidDtype")
    code(lambda: SafetensorsFile(craft({"x": {"dtype": "U8", "shape": [-4], "data_offsets": [0, 4]}}, one)), "InvalidShape")
    code(lambda: SafetensorsFile(craft({"x": {"dtype": "U8", "shape": [2.5], "data_offsets": [0, 4]}}, one)), "InvalidShape")
    code(lambda: SafetensorsFile(craft({"x": {"dtype": "U8", "shape": [4], "data_offsets": [0]}}, one)), "InvalidOffset")
    code(lambda: SafetensorsFile(craft({"x": {"dtype": "U8", "shape": [4], "data_offsets": [4, 0]}}, one)), "InvalidOffset")
    code(lambda: SafetensorsFile(craft({"x": {"dtype": "F32", "shape": [2], "data_offsets": [0, 4]}}, one)), "TensorInvalidInfo")
    code(lambda: SafetensorsFile(craft({"x": {"dtype": "F64", "shape": [2 ** 30, 2 ** 30], "data_offsets": [0, 4]}}, one)),
         "ValidationOverflow")
    # integral numbers written as floats are integers (as JSON.parse reads them)
    f = SafetensorsFile(craft('{"x": {"dtype": "U8", "shape": [4.0], "data_offsets": [0, 4e0]}}', one))
    assert f.info("x").shape == (4,)


def test_offsets_tile_the_data_section():
    eight = bytes(8)
    code(lambda: SafetensorsFile(craft({"x": u8(2, 8)}, eight)), "InvalidOffset")
    code(lambda: SafetensorsFile(craft({"x": u8(0, 3), "y": u8(4, 8)}, eight)), "InvalidOffset")
    code(lambda: SafetensorsFile(craft({"x": u8(0, 5), "y": u8(4, 8)}, eight)), "InvalidOffset")
    code(lambda: SafetensorsFile(craft({"x": u8(0, 16)}, eight)), "MetadataIncompleteBuffer")
    code(lambda: SafetensorsFile(craft({"x": u8(0, 4)}, eight)), "MetadataIncompleteBuffer")
    # the header alone (no file size) still catches gaps and overlaps, not trailing bytes
    assert parse_header(craft({"x": u8(0, 4)}, eight)).data_length == 4
    # out-of-order JSON with contiguous offsets is fine; empty tensors can sit anywhere
    f = SafetensorsFile(craft({"y": u8(4, 8), "e": {"dtype": "F32", "shape": [0, 3], "data_offsets": [4, 4]},
                               "x": u8(0, 4)}, eight))
    assert f.names() == ["y", "e", "x"] and f.numpy("e").shape == (0, 3)


def test_misaligned_data_reads():
    h = {"x": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}
    data = craft(h, f32(1.5, -2))
    assert (8 + len(json.dumps(h, separators=(",", ":")))) % 4 != 0
    assert SafetensorsFile(data).numpy("x").tolist() == [1.5, -2.0]


def test_file_path_and_mmap(tmp_path):
    p = tmp_path / "a.safetensors"
    st.write(p, {"w": ("F32", np.arange(6, dtype=np.float32).reshape(2, 3)), "b": ("BF16", np.array([0x3FC0], np.uint16))})
    with SafetensorsFile(str(p)) as f:
        assert f.numpy("w").tolist() == [[0, 1, 2], [3, 4, 5]]
        assert f.numpy("b").tolist() == [0x3FC0]
    p.write_bytes(p.read_bytes() + b"\0")  # trailing bytes
    code(lambda: SafetensorsFile(str(p)), "MetadataIncompleteBuffer")


ALL = {
    "f32": ("F32", np.array([[1, 2], [3, 4]], np.float32)),
    "f16": ("F16", np.array([1.5, -0.25], np.float16)),
    "bf16": ("BF16", np.array([0x3FC0], np.uint16)),
    "f64": ("F64", np.array([np.pi])),
    "i64": ("I64", np.array([-(2 ** 60), 7], np.int64)),
    "u64": ("U64", np.array([2 ** 63], np.uint64)),
    "i32": ("I32", np.array([-1], np.int32)),
    "u32": ("U32", np.array([4_000_000_000], np.uint32)),
    "i16": ("I16", np.array([-2], np.int16)),
    "u16": ("U16", np.array([65535], np.uint16)),
    "i8": ("I8", np.array([-3], np.int8)),
    "u8": ("U8", np.array([1, 2, 3], np.uint8)),
    "bool": ("BOOL", np.array([1, 0], np.uint8)),
    "empty": ("F32", np.zeros((0, 5), np.float32)),
    "scalar": ("F32", np.array(9, np.float32)),
}


def test_writer_round_trip_every_dtype():
    meta = {"format": "pt", "note": "é ünïcode"}
    f = SafetensorsFile(st.serialize(ALL, meta))
    assert f.metadata == meta and f.header.data_start % 8 == 0
    for name, (dtype, arr) in ALL.items():
        assert f.info(name).dtype == dtype and f.info(name).shape == arr.shape
        assert f.numpy(name).tobytes() == arr.tobytes(), name
        assert (f.header.data_start + f.info(name).data_offsets[0]) % st.BYTES[dtype] == 0, name


def test_writer_order_and_errors():
    f = SafetensorsFile(st.serialize({"b": ("U8", np.array([1], np.uint8)), "10": ("F32", np.array([1], np.float32)),
                                      "a": ("U8", np.array([2], np.uint8)), "2": ("F32", np.array([2], np.float32)),
                                      "z": ("I64", np.array([3], np.int64))}))
    assert f.names() == ["z", "10", "2", "a", "b"]
    code(lambda: st.serialize({"x": ("F16", np.zeros(2, np.float32))}), "TensorInvalidInfo")
    code(lambda: st.serialize({"x": ("Q4", np.zeros(1, np.uint8))}), "InvalidDtype")
    code(lambda: st.serialize({"__metadata__": ("U8", np.zeros(1, np.uint8))}), "InvalidHeaderDeserialization")
    code(lambda: st.serialize({}, {"k": 1}), "InvalidHeaderDeserialization")


safetensors_lib = pytest.importorskip("safetensors", reason="the Python safetensors package is not installed")


def _lib_serialize(tensors, metadata):
    """The safetensors package's low-level serializer (the reference oracle's ``serialize``)."""
    names = {"BOOL": "bool", "U8": "uint8", "I8": "int8", "U16": "uint16", "I16": "int16", "F16": "float16",
             "BF16": "bfloat16", "U32": "uint32", "I32": "int32", "F32": "float32", "U64": "uint64",
             "I64": "int64", "F64": "float64"}
    spec = {n: {"dtype": names[d], "shape": list(a.shape), "data": np.ascontiguousarray(a).tobytes()}
            for n, (d, a) in tensors.items()}
    return safetensors_lib.serialize(spec, metadata)


# one metadata key: the package keeps metadata in a hash map, so the order of several keys varies
@pytest.mark.parametrize("metadata", [None, {"format": "pt"}])
def test_serialize_matches_the_safetensors_package_byte_for_byte(metadata):
    tensors = {k: v for k, v in ALL.items()}
    tensors["bool"] = ("BOOL", np.array([True, False]))
    tensors["0"] = ("U8", np.array([1, 2, 3], np.uint8))
    tensors["layers.10.attn"] = ("F32", np.zeros(0, np.float32))
    tensors["nan"] = ("F32", np.array([0.5, -1, 2, np.nan, np.inf, -0.0], np.float32).reshape(2, 3))
    assert st.serialize(tensors, metadata) == bytes(_lib_serialize(tensors, metadata))


def test_reads_files_the_safetensors_package_writes(tmp_path):
    from safetensors.numpy import save_file
    rng = np.random.default_rng(3)
    arrs = {"a": rng.standard_normal((3, 5)).astype(np.float32),
            "h": np.array([1e-7, 65504, -0.0, np.inf, np.nan], np.float16),
            "d": rng.standard_normal(4), "i": np.arange(-3, 3, dtype=np.int64), "m": np.array([True, False, True]),
            "z": np.zeros((2, 0), np.float32), "s": np.array(2.5, np.float32)}
    p = tmp_path / "lib.safetensors"
    save_file(arrs, str(p), metadata={"k": "v"})
    with SafetensorsFile(str(p)) as f:
        assert f.metadata == {"k": "v"} and sorted(f.names()) == sorted(arrs)
        for k, a in arrs.items():
            got = f.numpy(k)
            assert got.shape == a.shape and got.tobytes() == a.astype(got.dtype).tobytes(), k
    # and the package reads what this writer writes, with the same bytes
    back = safetensors_lib.deserialize(st.serialize(ALL))
    got = {name: (info["dtype"], info["shape"], bytes(info["data"])) for name, info in back}
    for name, (dtype, arr) in ALL.items():
        assert got[name] == (dtype, list(arr.shape), arr.tobytes()), name
