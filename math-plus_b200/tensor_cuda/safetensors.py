"""safetensors files straight into device memory.

The header is parsed and validated as the reference's reader does it (packages/safetensors/src/
header.ts:76-245, itself following huggingface/safetensors ``Metadata::validate``): a u64
little-endian header length N (at most 100 MB), N bytes of UTF-8 JSON starting with ``{``, no
duplicate names, known dtypes, non-negative integer shapes, ``[begin, end]`` offsets that tile the
data section exactly (sorted, no gaps, no overlaps, each spanning ``prod(shape) * sizeof(dtype)``),
and the last tensor ending at the end of the file. Errors carry the reference's codes.

``load_to_device`` memory-maps the file and uploads each tensor with one host-to-device copy;
``gpt2_device_weights`` turns a Hugging Face GPT-2 checkpoint (``Conv1D`` weights stored
[in, out]) into the parameter names and [out, in] bf16 layout of :mod:`tensor_cuda.gpt2`, the
transposes and casts running on the device. ``serialize`` / ``write`` produce the reference
writer's layout.
"""
from __future__ import annotations

import json
import mmap
import os
from dataclasses import dataclass

import numpy as np

MAX_HEADER = 100 * 1024 * 1024

BYTES = {"BOOL": 1, "U8": 1, "I8": 1, "U16": 2, "I16": 2, "F16": 2, "BF16": 2,
         "U32": 4, "I32": 4, "F32": 4, "U64": 8, "I64": 8, "F64": 8}
NUMPY = {"BOOL": np.uint8, "U8": np.uint8, "I8": np.int8, "U16": np.uint16, "I16": np.int16, "F16": np.float16,
         "BF16": np.uint16, "U32": np.uint32, "I32": np.int32, "F32": np.float32, "U64": np.uint64,
         "I64": np.int64, "F64": np.float64}
# safetensors dtype -> device dtype (the device keeps f32, f16, bf16, i32 and bool)
DEVICE = {"F32": "f32", "F16": "f16", "BF16": "bf16", "I32": "i32", "BOOL": "bool"}


class SafetensorsError(ValueError):
    def __init__(self, code: str, message: str):
        super().__init__(f"safetensors: {message}")
        self.code = code


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dtype: str
    shape: tuple
    data_offsets: tuple


@dataclass(frozen=True)
class Header:
    tensors: dict
    metadata: dict
    data_start: int
    data_length: int


def _count(v):
    """A JSON number that is a non-negative safe integer (integral floats such as ``2.0`` count, as
    they do for JavaScript's ``Number.isSafeInteger``), as an int; None otherwise."""
    if isinstance(v, bool) or not isinstance(v, (int, float)):
        return None
    if isinstance(v, float) and not v.is_integer():
        return None
    return int(v) if 0 <= v < 2 ** 53 else None


class _Obj(list):
    """A JSON object as its (key, value) pairs in source order, duplicates kept."""


def _reject_constant(name):
    raise ValueError(f"{name} is not JSON")


def parse_header(data, file_size: int | None = None) -> Header:
    """Parses and validates the header from bytes holding at least the first 8 + N bytes
    (header.ts:124-245). ``file_size``, when known, enables the check that the offsets cover the
    data section exactly."""
    if len(data) < 8:
        raise SafetensorsError("HeaderTooSmall", f"need 8 bytes for the header length, got {len(data)}")
    n = int.from_bytes(bytes(data[:8]), "little")
    if n > MAX_HEADER:
        raise SafetensorsError("HeaderTooLarge", f"header length {n} exceeds {MAX_HEADER}")
    if len(data) < 8 + n:
        raise SafetensorsError("InvalidHeaderLength", f"truncated header: need {8 + n} bytes, have {len(data)}")
    if file_size is not None and file_size < 8 + n:
        raise SafetensorsError("InvalidHeaderLength", f"header length {n} exceeds file size {file_size}")
    try:
        text = bytes(data[8:8 + n]).decode("utf-8")
    except UnicodeDecodeError as e:
        raise SafetensorsError("InvalidHeader", "header is not valid UTF-8") from e
    if not text.startswith("{"):
        raise SafetensorsError("InvalidHeaderStart", "header must start with '{'")
    # Objects are kept as (key, value) lists so that duplicate keys stay visible (JSON.parse keeps
    # the last); NaN / Infinity are not JSON.
    try:
        top = json.loads(text, object_pairs_hook=_Obj, parse_constant=_reject_constant)
    except (ValueError, RecursionError) as e:
        raise SafetensorsError("InvalidHeaderDeserialization", f"header is not valid JSON ({e})") from e
    if not isinstance(top, _Obj):
        raise SafetensorsError("InvalidHeaderDeserialization", "header JSON must be an object")
    seen = set()
    for k, _ in top:
        if k in seen:
            raise SafetensorsError("DuplicateTensor", f"duplicate entry {json.dumps(k)} in header")
        seen.add(k)

    tensors, metadata = [], {}
    for name, raw in top:
        if name == "__metadata__":
            if raw is None:
                continue
            if not isinstance(raw, _Obj):
                raise SafetensorsError("InvalidHeaderDeserialization", "__metadata__ must be an object of strings")
            for k, v in raw:
                if not isinstance(v, str):
                    kind = "object" if isinstance(v, list) or v is None else \
                        "boolean" if isinstance(v, bool) else "number"
                    raise SafetensorsError("InvalidHeaderDeserialization", f"__metadata__.{k} must be a string, got {kind}")
            metadata = dict(raw)
            continue
        if not isinstance(raw, _Obj):
            raise SafetensorsError("InvalidHeaderDeserialization", f"entry {name} must be an object")
        r = dict(raw)
        dtype = r.get("dtype")
        if not isinstance(dtype, str) or dtype not in BYTES:
            raise SafetensorsError("InvalidDtype", f"unsupported dtype {json.dumps(dtype)} for {name}")
        shape = r.get("shape")
        dims = [_count(d) for d in shape] if isinstance(shape, list) and not isinstance(shape, _Obj) else None
        if dims is None or any(d is None for d in dims):
            raise SafetensorsError("InvalidShape", f"{name}: shape must be an array of non-negative integers")
        offs = r.get("data_offsets")
        bounds = [_count(v) for v in offs] if isinstance(offs, list) and not isinstance(offs, _Obj) else None
        if bounds is None or len(bounds) != 2 or any(v is None for v in bounds):
            raise SafetensorsError("InvalidOffset", f"{name}: data_offsets must be [begin, end] non-negative integers")
        begin, end = bounds
        if end < begin:
            raise SafetensorsError("InvalidOffset", f"{name}: data_offsets end {end} < begin {begin}")
        expected = BYTES[dtype]
        for d in dims:
            expected *= d
            if expected >= 2 ** 53:
                raise SafetensorsError("ValidationOverflow", f"{name}: byte size overflows")
        if end - begin != expected:
            raise SafetensorsError("TensorInvalidInfo",
                                   f"{name} spans {end - begin} bytes, expected {expected} for {dtype}{dims}")
        tensors.append(TensorInfo(name, dtype, tuple(dims), (begin, end)))

    # The offsets must tile [0, data length) exactly: no gaps, no overlaps (header.ts:221-233).
    cursor = 0
    for t in sorted(tensors, key=lambda t: t.data_offsets):
        b, e = t.data_offsets
        if b != cursor:
            raise SafetensorsError(
                "InvalidOffset",
                f"{t.name} overlaps the previous tensor (begins at {b}, previous ends at {cursor})" if b < cursor
                else f"gap before {t.name} (begins at {b}, previous ends at {cursor})")
        cursor = e
    if file_size is not None and 8 + n + cursor != file_size:
        raise SafetensorsError("MetadataIncompleteBuffer",
                               f"data section is {file_size - 8 - n} bytes but the header's offsets cover {cursor}")
    return Header({t.name: t for t in tensors}, metadata, 8 + n, cursor)


class SafetensorsFile:
    """A safetensors file, memory-mapped (a path) or in memory (bytes), with its validated header
    (the reference's ``readSafetensors`` / ``openSafetensors`` for a path, index.ts and lazy.ts)."""

    def __init__(self, source):
        self._f = None
        if isinstance(source, (str, os.PathLike)):
            self._f = open(source, "rb")
            size = os.fstat(self._f.fileno()).st_size
            self._buf = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ) if size else b""
        else:
            self._buf = source
        try:
            self.header = parse_header(self._buf, file_size=len(self._buf))
        except Exception:
            self.close()
            raise

    @property
    def metadata(self) -> dict:
        return self.header.metadata

    def names(self) -> list:
        return list(self.header.tensors)

    def has(self, name: str) -> bool:
        return name in self.header.tensors

    def info(self, name: str) -> TensorInfo:
        if name not in self.header.tensors:
            raise SafetensorsError("TensorNotFound", f"no tensor named {json.dumps(name)}")
        return self.header.tensors[name]

    def numpy(self, name: str) -> np.ndarray:
        """A host view of the tensor's bytes (BF16 as uint16 bits, BOOL as uint8); zero-copy over
        the mapping (numpy reads unaligned data as it is)."""
        t = self.info(name)
        b, e = t.data_offsets
        count = (e - b) // BYTES[t.dtype]
        if count == 0:
            return np.zeros(t.shape, NUMPY[t.dtype])
        arr = np.frombuffer(self._buf, dtype=NUMPY[t.dtype], count=count, offset=self.header.data_start + b)
        return arr.reshape(t.shape)

    def close(self) -> None:
        """Closes the file; a mapping that host views from ``numpy`` still point into is unmapped
        when the last of them goes."""
        if self._f is not None:
            if isinstance(self._buf, mmap.mmap):
                try:
                    self._buf.close()
                except BufferError:
                    pass
            self._buf = b""
            self._f.close()
            self._f = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def load_to_device(source, backend, names=None) -> dict:
    """Uploads the named tensors (default: all) into device memory and returns {name: CudaTensor}.

    Each tensor gets its own allocation (so every base address keeps the allocator's 256-byte
    alignment that TMA operands need) and one host-to-device copy straight from the mapped file,
    all queued on the backend's stream with a single synchronisation at the end. The dtype mapping
    is the reference's ``toTensor`` one (tensor.ts:19-22) restricted to what the device keeps:
    F32, F16, BF16 (bits), I32 and BOOL; any other dtype raises ``InvalidDtype`` before anything
    is copied."""
    f = source if isinstance(source, SafetensorsFile) else SafetensorsFile(source)
    out = {}
    try:
        names = f.names() if names is None else list(names)
        for name in names:
            t = f.info(name)
            if t.dtype not in DEVICE:
                raise SafetensorsError("InvalidDtype", f"{name}: dtype {t.dtype} has no device form "
                                                       "(F32, F16, BF16, I32, BOOL)")
        for name in names:
            t = f.info(name)
            x = backend._alloc(t.shape, DEVICE[t.dtype])
            out[name] = x
            if x.size:
                backend.device.copy_h2d(x._buf.ptr, f.numpy(name).reshape(-1))
        backend.device.stream_sync()  # the mapping may close once this returns
    except Exception:
        for x in out.values():
            backend.dispose(x)
        raise
    finally:
        if not isinstance(source, SafetensorsFile):
            f.close()
    return out


_CONV1D = ("attn.c_attn", "attn.c_proj", "mlp.c_fc", "mlp.c_proj")
_GPT2_NAMES = {"attn.c_attn": "attn.in_proj", "attn.c_proj": "attn.out_proj", "mlp.c_fc": "mlp.fc",
               "mlp.c_proj": "mlp.proj"}


def gpt2_device_weights(source, backend, n_layer: int) -> dict:
    """The device weights of :class:`tensor_cuda.gpt2.GPT2` from a Hugging Face GPT-2 checkpoint.

    The file is uploaded as stored; on the device, the ``Conv1D`` matrices (stored [in, out]) are
    transposed to the [out, in] layout ``linear`` takes, matrices are cast to bf16 (round to
    nearest even) and vectors to f32. A ``transformer.`` name prefix is accepted; the tied
    ``lm_head.weight``, when present, is not loaded."""
    f = source if isinstance(source, SafetensorsFile) else SafetensorsFile(source)
    try:
        prefix = "transformer." if f.has("transformer.wte.weight") else ""
        wanted = ["wte.weight", "wpe.weight", "ln_f.weight", "ln_f.bias"]
        for i in range(n_layer):
            p = f"h.{i}."
            wanted += [p + n for n in ("ln_1.weight", "ln_1.bias", "ln_2.weight", "ln_2.bias")]
            wanted += [p + c + ".weight" for c in _CONV1D] + [p + c + ".bias" for c in _CONV1D]
        missing = [n for n in wanted if not f.has(prefix + n)]
        if missing:
            raise SafetensorsError("TensorNotFound", f"GPT-2 checkpoint lacks {missing[:4]}"
                                                     f"{' ...' if len(missing) > 4 else ''}")
        raw = load_to_device(f, backend, [prefix + n for n in wanted])
    finally:
        if not isinstance(source, SafetensorsFile):
            f.close()

    def take(name, transpose=False, dtype="f32"):
        x = raw.pop(prefix + name)
        if transpose:
            y = backend.transpose(x)
            backend.dispose(x)
            x = y
        y = backend.cast(x, dtype)
        backend.dispose(x)
        return y

    w = {"wte": take("wte.weight", dtype="bf16"), "wpe": take("wpe.weight", dtype="bf16"),
         "ln_f.weight": take("ln_f.weight"), "ln_f.bias": take("ln_f.bias")}
    for i in range(n_layer):
        p = f"h.{i}."
        for n in ("ln_1.weight", "ln_1.bias", "ln_2.weight", "ln_2.bias"):
            w[p + n] = take(p + n)
        for c in _CONV1D:
            dst = p + _GPT2_NAMES[c]
            w[dst + ("_weight" if c == "attn.c_attn" else ".weight")] = take(p + c + ".weight", True, "bf16")
            w[dst + ("_bias" if c == "attn.c_attn" else ".bias")] = take(p + c + ".bias")
    backend.device.stream_sync()
    return w


# Sort key of the writer: the position of each dtype in the safetensors ``Dtype`` enum, larger first
# (writer.ts:32-35), so that every tensor starts at a multiple of its element size.
_ORDER = {"BOOL": 0, "U8": 1, "I8": 2, "I16": 3, "U16": 4, "F16": 5, "BF16": 6, "I32": 7, "U32": 8, "F32": 9,
          "F64": 10, "I64": 11, "U64": 12}


def serialize(tensors: dict, metadata: dict | None = None) -> bytes:
    """{name: (dtype, ndarray)} as safetensors bytes laid out like the reference's writer
    (writer.ts:38-97): tensors by dtype (larger element first) then name, compact JSON with
    ``__metadata__`` first, the header padded with spaces to an 8-byte boundary."""
    entries = []
    for name, (dtype, arr) in tensors.items():
        if name == "__metadata__":
            raise SafetensorsError("InvalidHeaderDeserialization",
                                   '"__metadata__" is reserved and cannot name a tensor')
        if dtype not in BYTES:
            raise SafetensorsError("InvalidDtype", f"unsupported dtype {json.dumps(dtype)} for {name}")
        a = np.asarray(arr)
        if a.dtype.itemsize != BYTES[dtype]:
            raise SafetensorsError("TensorInvalidInfo", f"{name}: {a.dtype} elements for {dtype}")
        entries.append((name, dtype, a.shape, np.ascontiguousarray(a).tobytes()))
    if metadata is not None:
        for k, v in metadata.items():
            if not isinstance(v, str):
                raise SafetensorsError("InvalidHeaderDeserialization", f"metadata.{k} must be a string")
    entries.sort(key=lambda e: (-_ORDER[e[1]], e[0]))
    parts = []
    if metadata is not None:
        parts.append('"__metadata__":' + json.dumps(metadata, ensure_ascii=False, separators=(",", ":")))
    off = 0
    for name, dtype, shape, blob in entries:
        info = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(blob)]}
        parts.append(json.dumps(name, ensure_ascii=False) + ":" + json.dumps(info, separators=(",", ":")))
        off += len(blob)
    text = ("{" + ",".join(parts) + "}").encode()
    text += b" " * ((8 - len(text) % 8) % 8)
    return len(text).to_bytes(8, "little") + text + b"".join(e[3] for e in entries)


def write(path, tensors: dict, metadata: dict | None = None) -> None:
    with open(path, "wb") as fh:
        fh.write(serialize(tensors, metadata))
