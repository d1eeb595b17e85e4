"""Streaming GGUF inspection: metadata key/values and the tensor inventory.

Reads the header sequentially (never the tensor data): magic ``GGUF``,
version, tensor and key/value counts, typed key/values (arrays included),
then each tensor's name, dimensions, ggml type and data offset; the data
section starts at the next ``general.alignment`` boundary (default 32).

Reference: si/model/gguf.py:153-243.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import BinaryIO

GGUF_MAGIC = b"GGUF"
# value type -> struct format (scalars); 8 = string, 9 = array
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q",
           11: "<q", 12: "<d"}
# ggml tensor types: (name, block elements, block bytes)
GGML_TYPES = {0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20),
              6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 36),
              10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144),
              13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 15: ("Q8_K", 256, 292),
              24: ("I8", 1, 1), 25: ("I16", 1, 2), 26: ("I32", 1, 4), 27: ("I64", 1, 8),
              28: ("F64", 1, 8), 30: ("BF16", 1, 2)}
MAX_STRING = 1 << 24
MAX_ARRAY = 1 << 24


class GGUFError(ValueError):
    pass


@dataclass(frozen=True)
class GGUFTensor:
    name: str
    shape: tuple[int, ...]
    ggml_type: int
    offset: int

    @property
    def type_name(self) -> str:
        return GGML_TYPES.get(self.ggml_type, (f"type{self.ggml_type}", 1, 0))[0]

    @property
    def nbytes(self) -> int:
        _, blk, bb = GGML_TYPES.get(self.ggml_type, ("?", 1, 0))
        n = 1
        for d in self.shape:
            n *= d
        return (n // blk) * bb


@dataclass
class GGUFDescription:
    version: int
    metadata: dict = field(default_factory=dict)
    tensors: list[GGUFTensor] = field(default_factory=list)
    data_offset: int = 0

    @property
    def architecture(self) -> str | None:
        return self.metadata.get("general.architecture")


def _read(f: BinaryIO, fmt: str):
    n = struct.calcsize(fmt)
    b = f.read(n)
    if len(b) != n:
        raise GGUFError("truncated GGUF header")
    return struct.unpack(fmt, b)[0]


def _string(f: BinaryIO) -> str:
    n = _read(f, "<Q")
    if n > MAX_STRING:
        raise GGUFError("string too long")
    b = f.read(n)
    if len(b) != n:
        raise GGUFError("truncated string")
    return b.decode("utf-8", errors="replace")


def _value(f: BinaryIO, t: int):
    if t in _SCALAR:
        return _read(f, _SCALAR[t])
    if t == 8:
        return _string(f)
    if t == 9:
        et = _read(f, "<I")
        n = _read(f, "<Q")
        if n > MAX_ARRAY:
            raise GGUFError("array too long")
        return [_value(f, et) for _ in range(n)]
    raise GGUFError(f"unknown GGUF value type {t}")


def inspect_gguf(path) -> GGUFDescription:
    with open(path, "rb") as f:
        if f.read(4) != GGUF_MAGIC:
            raise GGUFError("not a GGUF file")
        version = _read(f, "<I")
        if version not in (2, 3):
            raise GGUFError(f"unsupported GGUF version {version}")
        n_tensors = _read(f, "<Q")
        n_kv = _read(f, "<Q")
        desc = GGUFDescription(version)
        for _ in range(n_kv):
            key = _string(f)
            desc.metadata[key] = _value(f, _read(f, "<I"))
        for _ in range(n_tensors):
            name = _string(f)
            nd = _read(f, "<I")
            if nd > 8:
                raise GGUFError("too many dimensions")
            dims = tuple(_read(f, "<Q") for _ in range(nd))
            t = _read(f, "<I")
            off = _read(f, "<Q")
            desc.tensors.append(GGUFTensor(name, dims, t, off))
        align = int(desc.metadata.get("general.alignment", 32))
        pos = f.tell()
        desc.data_offset = (pos + align - 1) // align * align
        return desc


def write_gguf(path, metadata: dict, tensors: list[tuple[str, tuple[int, ...], int, bytes]]) -> None:
    """Minimal writer (tests, fixtures): scalars int/float/bool/str and lists of them."""

    def wstr(f, s):
        b = s.encode()
        f.write(struct.pack("<Q", len(b)))
        f.write(b)

    def wval(f, v):
        if isinstance(v, bool):
            f.write(struct.pack("<I?", 7, v))
        elif isinstance(v, int):
            f.write(struct.pack("<Iq", 11, v))
        elif isinstance(v, float):
            f.write(struct.pack("<Id", 12, v))
        elif isinstance(v, str):
            f.write(struct.pack("<I", 8))
            wstr(f, v)
        elif isinstance(v, list):
            f.write(struct.pack("<II", 9, 8 if v and isinstance(v[0], str) else 11))
            f.write(struct.pack("<Q", len(v)))
            for x in v:
                if isinstance(x, str):
                    wstr(f, x)
                else:
                    f.write(struct.pack("<q", x))
        else:
            raise TypeError(type(v))

    with open(path, "wb") as f:
        f.write(GGUF_MAGIC)
        f.write(struct.pack("<IQQ", 3, len(tensors), len(metadata)))
        for k, v in metadata.items():
            wstr(f, k)
            wval(f, v)
        off = 0
        for name, shape, t, data in tensors:
            wstr(f, name)
            f.write(struct.pack("<I", len(shape)))
            for d in shape:
                f.write(struct.pack("<Q", d))
            f.write(struct.pack("<IQ", t, off))
            off += (len(data) + 31) // 32 * 32
        pos = f.tell()
        f.write(b"\0" * ((pos + 31) // 32 * 32 - pos))
        for _, _, _, data in tensors:
            f.write(data)
            f.write(b"\0" * ((len(data) + 31) // 32 * 32 - len(data)))
