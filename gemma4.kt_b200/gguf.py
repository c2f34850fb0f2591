"""GGUF v2/v3 files: the reader the model loader needs and the writer the
synthetic-model generator uses.

Format (as the reference parses it, gguf/GGUF.kt:89-212, MetadataValueType.kt,
GGMLType.kt): little-endian; magic 0x46554747 ("GGUF"), version, tensor count
(u64), metadata count (u64); metadata key/value pairs (u64-length UTF-8 key,
u32 value type, value; arrays carry an element type and a u64 length); tensor
infos (name, u32 n_dims, u64 dims innermost first, u32 GGML type, u64 offset
relative to the data section, a multiple of the alignment); padding to
`general.alignment` (default 32); tensor data.

The reader memory-maps the file once and hands out zero-copy numpy views of
each tensor's block stream, like GGUF.loadTensors slicing its MemorySegment
(GGUF.kt:195-212).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from enum import IntEnum
from pathlib import Path

import numpy as np

from .floattensor import GGMLType

GGUF_MAGIC = 0x46554747  # GGUF.kt:476
DEFAULT_ALIGNMENT = 32   # GGUF.kt:477
SUPPORTED_VERSIONS = (2, 3)


class ValueType(IntEnum):
    """MetadataValueType.kt: the wire ids are the enum ordinals."""

    UINT8 = 0
    INT8 = 1
    UINT16 = 2
    INT16 = 3
    UINT32 = 4
    INT32 = 5
    FLOAT32 = 6
    BOOL = 7
    STRING = 8
    ARRAY = 9
    UINT64 = 10
    INT64 = 11
    FLOAT64 = 12


_SCALAR = {
    ValueType.UINT8: "<B", ValueType.INT8: "<b", ValueType.UINT16: "<H", ValueType.INT16: "<h",
    ValueType.UINT32: "<I", ValueType.INT32: "<i", ValueType.FLOAT32: "<f", ValueType.BOOL: "<?",
    ValueType.UINT64: "<Q", ValueType.INT64: "<q", ValueType.FLOAT64: "<d",
}
_NP = {
    ValueType.UINT8: np.uint8, ValueType.INT8: np.int8, ValueType.UINT16: np.uint16, ValueType.INT16: np.int16,
    ValueType.UINT32: np.uint32, ValueType.INT32: np.int32, ValueType.FLOAT32: np.float32,
    ValueType.BOOL: np.bool_, ValueType.UINT64: np.uint64, ValueType.INT64: np.int64,
    ValueType.FLOAT64: np.float64,
}


@dataclass
class TensorInfo:
    """GGUFTensorInfo.kt: name, dims (innermost first), GGML type, data offset."""

    name: str
    dims: tuple
    ggml_type: GGMLType
    offset: int

    @property
    def n_elems(self) -> int:
        n = 1
        for d in self.dims:
            n *= int(d)
        return n

    @property
    def nbytes(self) -> int:
        return self.ggml_type.byte_size_for(self.n_elems)


class Typed:
    """A metadata value with an explicit wire type (for the writer)."""

    def __init__(self, vtype: ValueType, value, elem: ValueType | None = None):
        self.vtype, self.value, self.elem = vtype, value, elem


def u32(v) -> Typed:
    return Typed(ValueType.UINT32, int(v))


def i32(v) -> Typed:
    return Typed(ValueType.INT32, int(v))


def f32(v) -> Typed:
    return Typed(ValueType.FLOAT32, float(v))


def arr(elem: ValueType, values) -> Typed:
    return Typed(ValueType.ARRAY, values, elem)


# ---------------------------------------------------------------------- reader
class GGUFFile:
    """Parsed GGUF header + mmap of the file (GGUF.kt:89-212)."""

    def __init__(self, path):
        self.path = Path(path)
        self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        self._pos = 0
        magic, = self._read("<I")
        if magic != GGUF_MAGIC:
            raise ValueError(f"unsupported header.magic {magic}")
        self.version, = self._read("<I")
        if self.version not in SUPPORTED_VERSIONS:
            raise ValueError(f"unsupported header.version {self.version}")
        n_tensors, n_kv = self._read("<QQ")
        self.metadata: dict = {}
        for _ in range(n_kv):
            key = self._string()
            if key in self.metadata:
                raise ValueError(f"duplicate metadata key {key}")
            self.metadata[key] = self._value(ValueType(self._read("<I")[0]))
        self.alignment = int(self.metadata.get("general.alignment", DEFAULT_ALIGNMENT))
        if self.alignment <= 0 or self.alignment & (self.alignment - 1):
            raise ValueError("alignment must be a power of two")
        self.tensors: dict[str, TensorInfo] = {}
        for _ in range(n_tensors):
            name = self._string()
            nd, = self._read("<I")
            dims = tuple(int(d) for d in self._read("<" + "Q" * nd))
            t = GGMLType.from_id(self._read("<I")[0])
            off, = self._read("<Q")
            if off % self.alignment:
                raise ValueError(f"tensor {name}: offset {off} not aligned")
            self.tensors[name] = TensorInfo(name, dims, t, off)
        pad = (self.alignment - self._pos % self.alignment) % self.alignment
        self.data_offset = self._pos + pad

    def _read(self, fmt: str):
        n = struct.calcsize(fmt)
        v = struct.unpack_from(fmt, self._mm, self._pos)
        self._pos += n
        return v

    def _string(self) -> str:
        n, = self._read("<Q")
        s = bytes(self._mm[self._pos:self._pos + n]).decode("utf-8")
        self._pos += n
        return s

    def _value(self, vt: ValueType):
        if vt in _SCALAR:
            return self._read(_SCALAR[vt])[0]
        if vt == ValueType.STRING:
            return self._string()
        if vt == ValueType.ARRAY:
            et = ValueType(self._read("<I")[0])
            n, = self._read("<Q")
            if et in _NP:
                a = np.frombuffer(self._mm, dtype=np.dtype(_NP[et]).newbyteorder("<"), count=n,
                                  offset=self._pos).copy()
                self._pos += a.nbytes
                return a
            return [self._value(et) for _ in range(n)]
        raise ValueError(f"metadata value type {vt}")

    def tensor_bytes(self, name: str) -> np.ndarray:
        """Zero-copy uint8 view of the tensor's block stream."""
        ti = self.tensors[name]
        start = self.data_offset + ti.offset
        return self._mm[start:start + ti.nbytes]

    def tensor_f32(self, name: str) -> np.ndarray:
        ti = self.tensors[name]
        if ti.ggml_type != GGMLType.F32:
            raise ValueError(f"Conversion to {ti.ggml_type.name}")  # ModelLoader.toFloatBuffer
        return self.tensor_bytes(name).view(np.float32)


# ---------------------------------------------------------------------- writer
def _enc_value(vt: ValueType, v, elem: ValueType | None = None) -> bytes:
    if vt in _SCALAR:
        return struct.pack(_SCALAR[vt], v)
    if vt == ValueType.STRING:
        b = v.encode("utf-8")
        return struct.pack("<Q", len(b)) + b
    if vt == ValueType.ARRAY:
        if elem in _NP:
            a = np.ascontiguousarray(np.asarray(v, dtype=np.dtype(_NP[elem]).newbyteorder("<")))
            return struct.pack("<IQ", int(elem), a.size) + a.tobytes()
        parts = [struct.pack("<IQ", int(elem), len(v))]
        parts += [_enc_value(elem, x) for x in v]
        return b"".join(parts)
    raise ValueError(vt)


def _typed(v) -> Typed:
    if isinstance(v, Typed):
        return v
    if isinstance(v, bool):
        return Typed(ValueType.BOOL, v)
    if isinstance(v, int):
        return Typed(ValueType.INT32, v)
    if isinstance(v, float):
        return Typed(ValueType.FLOAT32, v)
    if isinstance(v, str):
        return Typed(ValueType.STRING, v)
    raise TypeError(f"give {v!r} an explicit metadata type")


def write_gguf(path, metadata: dict, tensors: list, alignment: int = DEFAULT_ALIGNMENT) -> None:
    """Write a GGUF v3 file.  `tensors`: (name, dims innermost first, GGMLType,
    block-stream bytes) in file order; every offset is aligned."""
    header = [struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(metadata))]
    for k, v in metadata.items():
        t = _typed(v)
        kb = k.encode("utf-8")
        header.append(struct.pack("<Q", len(kb)) + kb + struct.pack("<I", int(t.vtype)) +
                      _enc_value(t.vtype, t.value, t.elem))
    off = 0
    offsets = []
    for name, dims, gt, raw in tensors:
        gt = GGMLType(int(gt))
        n = 1
        for d in dims:
            n *= int(d)
        if len(raw) != gt.byte_size_for(n):
            raise ValueError(f"{name}: {len(raw)} bytes for {n} {gt.name} elements")
        nb = name.encode("utf-8")
        header.append(struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims)) +
                      struct.pack("<" + "Q" * len(dims), *dims) + struct.pack("<IQ", int(gt), off))
        offsets.append(off)
        off += len(raw)
        off += (alignment - off % alignment) % alignment
    with open(path, "wb") as f:
        h = b"".join(header)
        f.write(h)
        f.write(b"\0" * ((alignment - len(h) % alignment) % alignment))
        pos = 0
        for (name, dims, gt, raw), o in zip(tensors, offsets):
            if o > pos:
                f.write(b"\0" * (o - pos))
                pos = o
            mv = memoryview(np.ascontiguousarray(raw).view(np.uint8).reshape(-1))
            f.write(mv)
            pos += len(mv)
