"""GGUF v2/v3 reader and writer (host side).

The reader mirrors ``GgufReader.Parse`` / ``GgufFile``
(src/DotNetFoundryLLM.ModelFormats.Gguf/GgufReader.cs:55-111,
GgufFile.cs:76-123): little-endian header, metadata key/values, tensor infos,
data start aligned to ``general.alignment`` (default 32), tensor offsets
relative to that start.  It works on any buffer (bytes, numpy array,
``np.memmap``) without copying tensor payloads.

The writer produces files that reader (and the reference loader) accepts; it is
used to build the seeded synthetic models.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Any, Callable

import numpy as np

# GgufValueType.cs
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)

# GgufTensorType.cs
T_F32, T_F16, T_Q4_0, T_Q4_1, T_Q5_0, T_Q5_1, T_Q8_0, T_Q8_1 = 0, 1, 2, 3, 6, 7, 8, 9
T_Q2_K, T_Q3_K, T_Q4_K, T_Q5_K, T_Q6_K, T_Q8_K, T_BF16 = 10, 11, 12, 13, 14, 15, 30

TYPE_NAMES = {T_F32: "F32", T_F16: "F16", T_Q4_0: "Q4_0", T_Q8_0: "Q8_0", T_Q4_K: "Q4_K", T_Q5_K: "Q5_K",
              T_Q6_K: "Q6_K", T_Q8_K: "Q8_K", T_BF16: "BF16"}

# GgufFile.ComputeByteSize (GgufFile.cs:100-123): (block elements, block bytes)
BLOCK = {T_F32: (1, 4), T_F16: (1, 2), T_BF16: (1, 2), T_Q4_0: (32, 18), T_Q4_1: (32, 20), T_Q5_0: (32, 22),
         T_Q5_1: (32, 24), T_Q8_0: (32, 34), T_Q8_1: (32, 36), T_Q4_K: (256, 144), T_Q5_K: (256, 176),
         T_Q6_K: (256, 210), T_Q8_K: (256, 292)}

_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", U64: "<Q", I64: "<q",
           F64: "<d"}


class ModelLoadError(Exception):
    """DotNetFoundryLLM.Core.ModelLoadException."""


@dataclass
class MetaValue:
    type: int
    value: Any = None
    array_type: int | None = None  # element type when type == ARR


@dataclass
class TensorInfo:
    name: str
    dims: list[int]
    type: int
    offset: int

    @property
    def element_count(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n


def byte_size(info: TensorInfo) -> int:
    if info.type not in BLOCK:
        raise NotImplementedError(f"Cannot compute byte size for tensor type {info.type}.")
    be, bb = BLOCK[info.type]
    return info.element_count // be * bb


class _Reader:
    def __init__(self, buf):
        self.mv = memoryview(buf).cast("B")
        self.pos = 0

    def take(self, n: int) -> memoryview:
        if n < 0 or self.pos + n > len(self.mv):
            raise ModelLoadError("Truncated GGUF header.")
        b = self.mv[self.pos:self.pos + n]
        self.pos += n
        return b

    def scalar(self, t: int):
        fmt = _SCALAR[t]
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.scalar(U64)
        return bytes(self.take(n)).decode("utf-8", "replace")

    def value(self, t: int):
        if t in _SCALAR:
            return self.scalar(t)
        if t == BOOL:
            return self.take(1)[0] != 0
        if t == STR:
            return self.string()
        raise NotImplementedError(f"Unsupported array element type: {t}")


class GgufFile:
    """Parsed GGUF image: ``metadata``, ``tensors`` and zero-copy ``tensor_bytes``."""

    def __init__(self, buf, version: int, metadata: dict[str, MetaValue], tensors: list[TensorInfo],
                 data_start: int):
        self.buf = buf
        self.version = version
        self.metadata = metadata
        self.tensors = tensors
        self.data_start = data_start
        self._index = {t.name: t for t in tensors}

    def find_tensor(self, name: str) -> TensorInfo | None:
        return self._index.get(name)

    def tensor_bytes(self, info: TensorInfo) -> np.ndarray:
        """GgufFile.GetTensorBytes: a view of the raw (quantized) payload."""
        n = byte_size(info)
        off = self.data_start + info.offset
        arr = np.frombuffer(self.buf, dtype=np.uint8, count=n, offset=off) if not isinstance(self.buf, np.ndarray) \
            else self.buf[off:off + n]
        if arr.size != n:
            raise ModelLoadError(f"Tensor '{info.name}' data lies outside the file.")
        return arr

    # GgufModelLoader metadata helpers (GgufModelLoader.cs:433-478)
    def get_string(self, key: str, default: str = "") -> str:
        v = self.metadata.get(key)
        return v.value if v is not None and v.type == STR else default

    def get_uint(self, key: str, default: int = 0, array_length: bool = False) -> int:
        v = self.metadata.get(key)
        if v is None:
            return default
        if array_length and v.type == ARR:
            return len(v.value)
        if v.type in (U8, U16, U32, U64):
            return int(v.value)
        if v.type in (I32, I64):
            return int(v.value) & 0xFFFFFFFFFFFFFFFF
        return default

    def get_float(self, key: str, default: float = 0.0) -> float:
        v = self.metadata.get(key)
        return float(v.value) if v is not None and v.type == F32 else default


def parse(buf) -> GgufFile:
    """GgufReader.Parse (GgufReader.cs:55-111)."""
    r = _Reader(buf)
    if len(r.mv) < 4 or bytes(r.mv[:4]) != b"GGUF":
        raise ModelLoadError("Not a GGUF file: invalid magic bytes.")
    r.pos = 4
    version = r.scalar(U32)
    if version not in (2, 3):
        raise ModelLoadError(f"Unsupported GGUF version {version}. Expected 2 or 3.")
    n_tensors = r.scalar(U64)
    n_kv = r.scalar(U64)
    meta: dict[str, MetaValue] = {}
    for _ in range(n_kv):
        key = r.string()
        t = r.scalar(U32)
        if t == ARR:
            et = r.scalar(U32)
            cnt = r.scalar(U64) if version >= 3 else r.scalar(U32)
            meta[key] = MetaValue(ARR, [r.value(et) for _ in range(cnt)], et)
        elif t in _SCALAR or t in (BOOL, STR):
            meta[key] = MetaValue(t, r.value(t))
        else:
            raise NotImplementedError(f"Unknown GGUF metadata value type: {t}")
    tensors = []
    for _ in range(n_tensors):
        name = r.string()
        nd = r.scalar(U32)
        dims = [r.scalar(U64) for _ in range(nd)]
        t = r.scalar(U32)
        off = r.scalar(U64)
        tensors.append(TensorInfo(name, dims, t, off))
    align = 32
    a = meta.get("general.alignment")
    if a is not None and a.type in (U32, U64):
        align = int(a.value) & 0xFFFFFFFF
    if align == 0:
        raise ModelLoadError("Attempted to divide by zero (general.alignment = 0).")
    start = (r.pos + align - 1) // align * align
    return GgufFile(buf, version, meta, tensors, start)


# ── writer ────────────────────────────────────────────────────────────────

def _enc_str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _enc_value(t: int, v) -> bytes:
    if t in _SCALAR:
        return struct.pack(_SCALAR[t], v)
    if t == BOOL:
        return struct.pack("<B", 1 if v else 0)
    if t == STR:
        return _enc_str(v)
    raise ValueError(t)


@dataclass
class PlannedTensor:
    name: str
    dims: list[int]
    type: int
    nbytes: int
    fill: Callable[[np.ndarray], None]
    offset: int = 0


@dataclass
class GgufWriter:
    """Two-phase writer: add metadata and tensor plans, then ``build()`` into
    one buffer (or ``write(path)``).  ``fill`` callbacks write each payload in
    place, so multi-GB models never hold a second copy."""

    version: int = 3
    alignment: int = 32
    meta: list[tuple[str, int, Any, int | None]] = field(default_factory=list)
    tensors: list[PlannedTensor] = field(default_factory=list)

    def add(self, key: str, t: int, value, array_type: int | None = None) -> None:
        self.meta.append((key, t, value, array_type))

    def add_tensor(self, name: str, dims: list[int], t: int, fill: Callable[[np.ndarray], None]) -> None:
        n = 1
        for d in dims:
            n *= d
        be, bb = BLOCK[t]
        if n % be:
            raise ValueError(f"{name}: {n} elements is not a multiple of the {be}-element block")
        self.tensors.append(PlannedTensor(name, list(dims), t, n // be * bb, fill))

    def _header(self) -> bytes:
        out = bytearray(b"GGUF")
        out += struct.pack("<I", self.version)
        out += struct.pack("<QQ", len(self.tensors), len(self.meta))
        for key, t, v, at in self.meta:
            out += _enc_str(key) + struct.pack("<I", t)
            if t == ARR:
                out += struct.pack("<I", at)
                out += struct.pack("<Q", len(v)) if self.version >= 3 else struct.pack("<I", len(v))
                for e in v:
                    out += _enc_value(at, e)
            else:
                out += _enc_value(t, v)
        off = 0
        for tp in self.tensors:
            off = (off + self.alignment - 1) // self.alignment * self.alignment
            tp.offset = off
            off += tp.nbytes
            out += _enc_str(tp.name) + struct.pack("<I", len(tp.dims))
            for d in tp.dims:
                out += struct.pack("<Q", d)
            out += struct.pack("<IQ", tp.type, tp.offset)
        self._data_len = off
        return bytes(out)

    def build(self, out: np.ndarray | None = None) -> np.ndarray:
        hdr = self._header()
        start = (len(hdr) + self.alignment - 1) // self.alignment * self.alignment
        total = start + self._data_len
        buf = np.zeros(total, dtype=np.uint8) if out is None else out[:total]
        buf[:len(hdr)] = np.frombuffer(hdr, dtype=np.uint8)
        for tp in self.tensors:
            tp.fill(buf[start + tp.offset:start + tp.offset + tp.nbytes])
        return buf

    def write(self, path: str) -> int:
        buf = self.build()
        buf.tofile(path)
        return int(buf.size)
