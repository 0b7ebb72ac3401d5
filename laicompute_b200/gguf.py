"""GGUF v3 container: a minimal writer and reader.

The reader follows the parse rules of the reference loader
(``src/gguf.cpp:9-18``): little-endian fields, metadata value types 0..12,
tensor infos ``name, n_dims, dims (ne0 first), ggml_type, offset`` and a data
section that starts at the next multiple of ``general.alignment`` (default 32).
The writer emits exactly what that loader accepts; it is used to build the
synthetic Llama models the engine and the oracle both decode.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Any, Dict, List, Sequence, Tuple

import numpy as np

GGUF_MAGIC = 0x46554747  # "GGUF"

# GGML tensor types used by the reference (include/laic/gguf.hpp:9).
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q5_0: "Q5_0", Q8_0: "Q8_0"}
BLOCK_BYTES = {Q4_0: 18, Q4_1: 20, Q5_0: 22, Q5_1: 24, Q8_0: 34}

# metadata value type codes (src/gguf.cpp:10)
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)


def tensor_nbytes(ggml_type: int, n_elements: int) -> int:
    """Byte size of a tensor, as ``GgufTensor::bytes`` (src/gguf.cpp:16)."""
    if ggml_type == F32:
        return 4 * n_elements
    if ggml_type == F16:
        return 2 * n_elements
    return (n_elements + 31) // 32 * BLOCK_BYTES[ggml_type]


@dataclass
class TensorInfo:
    name: str
    shape: Tuple[int, ...]  # ne0 first (ne0 = contiguous "in" dimension)
    ggml_type: int
    offset: int = 0
    data: Any = None  # bytes / np.ndarray view on read

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.shape:
            n *= int(d)
        return n

    @property
    def nbytes(self) -> int:
        return tensor_nbytes(self.ggml_type, self.n_elements)


class _Buf:
    def __init__(self) -> None:
        self.parts: List[bytes] = []
        self.n = 0

    def put(self, b: bytes) -> None:
        self.parts.append(b)
        self.n += len(b)

    def u32(self, v: int) -> None:
        self.put(struct.pack("<I", v))

    def u64(self, v: int) -> None:
        self.put(struct.pack("<Q", v))

    def string(self, s: str | bytes) -> None:
        b = s.encode("utf-8") if isinstance(s, str) else s
        self.u64(len(b))
        self.put(b)


def _put_value(buf: _Buf, v: Any) -> None:
    """Write one typed metadata value (type code first)."""
    if isinstance(v, bool):
        buf.u32(_BOOL); buf.put(struct.pack("<B", 1 if v else 0))
    elif isinstance(v, np.float32):
        buf.u32(_F32); buf.put(struct.pack("<f", float(v)))
    elif isinstance(v, float):
        buf.u32(_F32); buf.put(struct.pack("<f", v))
    elif isinstance(v, np.uint32) or (isinstance(v, int) and 0 <= v < 2**32):
        buf.u32(_U32); buf.u32(int(v))
    elif isinstance(v, int):
        buf.u32(_U64); buf.u64(v)
    elif isinstance(v, (str, bytes)):
        buf.u32(_STR); buf.string(v)
    elif isinstance(v, (list, tuple)):
        if all(isinstance(x, (str, bytes)) for x in v):
            buf.u32(_ARR); buf.u32(_STR); buf.u64(len(v))
            for x in v:
                buf.string(x)
        else:
            buf.u32(_ARR); buf.u32(_U32); buf.u64(len(v))
            buf.put(np.asarray(v, dtype="<u4").tobytes())
    else:
        raise TypeError(f"unsupported metadata value {type(v)}")


def write_gguf(path: str, metadata: Dict[str, Any], tensors: Sequence[Tuple[str, Tuple[int, ...], int, bytes]],
               alignment: int = 32) -> None:
    """Write a GGUF v3 file.

    ``tensors`` holds ``(name, shape_ne0_first, ggml_type, raw_bytes)``;
    the raw bytes are the block-encoded payload.
    """
    md = dict(metadata)
    md.setdefault("general.alignment", alignment)
    head = _Buf()
    head.u32(GGUF_MAGIC)
    head.u32(3)
    head.u64(len(tensors))
    head.u64(len(md))
    for k, v in md.items():
        head.string(k)
        _put_value(head, v)
    off = 0
    offsets = []
    for name, shape, gt, raw in tensors:
        n = 1
        for d in shape:
            n *= int(d)
        if len(raw) != tensor_nbytes(gt, n):
            raise ValueError(f"{name}: {len(raw)} bytes, expected {tensor_nbytes(gt, n)}")
        head.string(name)
        head.u32(len(shape))
        for d in shape:
            head.u64(int(d))
        head.u32(gt)
        head.u64(off)
        offsets.append(off)
        off = (off + len(raw) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        for p in head.parts:
            f.write(p)
        pad = (-head.n) % alignment
        f.write(b"\0" * pad)
        pos = 0
        for (name, shape, gt, raw), o in zip(tensors, offsets):
            if o > pos:
                f.write(b"\0" * (o - pos))
                pos = o
            f.write(raw)
            pos += len(raw)
        tail = (-pos) % alignment
        f.write(b"\0" * tail)


class GgufFile:
    """Read-only GGUF view (metadata dict + tensor infos over a memory map)."""

    def __init__(self, path: str) -> None:
        self.path = path
        self.raw = np.memmap(path, dtype=np.uint8, mode="r")
        self.metadata: Dict[str, Any] = {}
        self.tensors: Dict[str, TensorInfo] = {}
        self._p = 0
        self._parse()

    # -- little-endian field readers -------------------------------------------------
    def _take(self, n: int) -> bytes:
        if self._p + n > len(self.raw):
            raise ValueError("invalid/truncated GGUF")
        b = bytes(self.raw[self._p:self._p + n])
        self._p += n
        return b

    def _u32(self) -> int:
        return struct.unpack("<I", self._take(4))[0]

    def _u64(self) -> int:
        return struct.unpack("<Q", self._take(8))[0]

    def _str(self) -> str:
        n = self._u64()
        return self._take(n).decode("utf-8", errors="surrogateescape")

    def _value(self, t: int) -> Any:
        fmt = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i",
               _F32: "<f", _U64: "<Q", _I64: "<q", _F64: "<d"}
        if t in fmt:
            size = struct.calcsize(fmt[t])
            return struct.unpack(fmt[t], self._take(size))[0]
        if t == _BOOL:
            return self._take(1)[0] != 0
        if t == _STR:
            return self._str()
        if t == _ARR:
            et = self._u32()
            n = self._u64()
            return [self._value(et) for _ in range(n)]
        raise ValueError("unsupported GGUF metadata type")

    def _parse(self) -> None:
        if self._u32() != GGUF_MAGIC:
            raise ValueError("bad GGUF magic")
        ver = self._u32()
        if ver < 2 or ver > 3:
            raise ValueError("unsupported GGUF version")
        nt, nm = self._u64(), self._u64()
        for _ in range(nm):
            k = self._str()
            t = self._u32()
            self.metadata[k] = self._value(t)
        infos = []
        for _ in range(nt):
            name = self._str()
            nd = self._u32()
            shape = tuple(self._u64() for _ in range(nd))
            gt = self._u32()
            off = self._u64()
            infos.append(TensorInfo(name, shape, gt, off))
        align = int(self.metadata.get("general.alignment", 32)) or 32
        start = (self._p + align - 1) // align * align
        for ti in infos:
            base = start + ti.offset
            ti.data = self.raw[base:base + ti.nbytes]
            if len(ti.data) != ti.nbytes:
                raise ValueError("tensor data out of range")
            self.tensors[ti.name] = ti

    def u64(self, key: str, fallback: int = 0) -> int:
        v = self.metadata.get(key)
        return int(v) if isinstance(v, (int, bool)) else fallback

    def f64(self, key: str, fallback: float = 0.0) -> float:
        v = self.metadata.get(key)
        return float(v) if isinstance(v, (int, float)) and not isinstance(v, bool) else fallback
