"""Header-only safetensors inspection, sharded-index validation and tensor loading.

A safetensors file is ``u64 header_len | JSON header | raw data``; the header
maps tensor names to ``{"dtype", "shape", "data_offsets": [begin, end]}``
(offsets relative to the data section) plus an optional ``__metadata__``.
Inspection reads only the header, so multi-GB checkpoints are described
without touching their data; loading memory-maps the file and copies each
tensor once.

Reference: si/model/safetensors.py:67-267 (inventory, index validation).
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

DTYPE_BYTES = {"F64": 8, "F32": 4, "F16": 2, "BF16": 2, "I64": 8, "I32": 4, "I16": 2, "I8": 1,
               "U8": 1, "BOOL": 1, "F8_E4M3": 1, "F8_E5M2": 1, "U16": 2, "U32": 4, "U64": 8}
TORCH_DTYPES = {"F64": torch.float64, "F32": torch.float32, "F16": torch.float16,
                "BF16": torch.bfloat16, "I64": torch.int64, "I32": torch.int32, "I16": torch.int16,
                "I8": torch.int8, "U8": torch.uint8, "BOOL": torch.bool,
                "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2}
MAX_HEADER = 100 * 1024 * 1024


class SafetensorsError(ValueError):
    pass


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dtype: str
    shape: tuple[int, ...]
    begin: int
    end: int
    file: str

    @property
    def nbytes(self) -> int:
        return self.end - self.begin


def read_header(path: str | os.PathLike) -> tuple[dict, int]:
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise SafetensorsError(f"{path}: truncated header length")
        (n,) = struct.unpack("<Q", raw)
        if n > MAX_HEADER:
            raise SafetensorsError(f"{path}: header of {n} bytes exceeds the limit")
        hdr = f.read(n)
        if len(hdr) != n:
            raise SafetensorsError(f"{path}: truncated header")
    try:
        return json.loads(hdr), 8 + n
    except json.JSONDecodeError as exc:
        raise SafetensorsError(f"{path}: header is not JSON: {exc}") from None


def inspect_file(path: str | os.PathLike) -> list[TensorInfo]:
    header, data_start = read_header(path)
    size = os.path.getsize(path) - data_start
    out = []
    spans = []
    for name, v in header.items():
        if name == "__metadata__":
            continue
        dt = v.get("dtype")
        if dt not in DTYPE_BYTES:
            raise SafetensorsError(f"{name}: unsupported dtype {dt}")
        shape = tuple(int(x) for x in v["shape"])
        b, e = (int(x) for x in v["data_offsets"])
        n = int(np.prod(shape)) if shape else 1
        if e - b != n * DTYPE_BYTES[dt] or b < 0 or e > size:
            raise SafetensorsError(f"{name}: offsets do not match shape/dtype or file size")
        spans.append((b, e, name))
        out.append(TensorInfo(name, dt, shape, b, e, str(path)))
    spans.sort()
    for (b0, e0, n0), (b1, e1, n1) in zip(spans, spans[1:]):
        if b1 < e0:
            raise SafetensorsError(f"tensors {n0} and {n1} overlap")
    return out


def inspect_checkpoint(root: str | os.PathLike) -> dict[str, TensorInfo]:
    """Inventory of a checkpoint directory (single file or index-sharded)."""
    root = Path(root)
    index = root / "model.safetensors.index.json"
    files: list[Path]
    if index.exists():
        idx = json.loads(index.read_text())
        wm = idx.get("weight_map")
        if not isinstance(wm, dict) or not wm:
            raise SafetensorsError("index has no weight_map")
        files = sorted({root / f for f in wm.values()})
        inv = {}
        for f in files:
            for t in inspect_file(f):
                inv[t.name] = t
        missing = set(wm) - set(inv)
        extra = set(inv) - set(wm)
        if missing:
            raise SafetensorsError(f"index names tensors missing from shards: {sorted(missing)[:5]}")
        if extra:
            raise SafetensorsError(f"shards hold tensors absent from the index: {sorted(extra)[:5]}")
        for name, f in wm.items():
            if Path(inv[name].file).name != f:
                raise SafetensorsError(f"{name} is in {inv[name].file}, index says {f}")
        return inv
    files = sorted(root.glob("*.safetensors"))
    if not files:
        raise SafetensorsError(f"no safetensors files in {root}")
    inv = {}
    for f in files:
        for t in inspect_file(f):
            if t.name in inv:
                raise SafetensorsError(f"duplicate tensor {t.name}")
            inv[t.name] = t
    return inv


class CheckpointReader:
    """Memory-mapped tensor access: ``reader.get(name, shape)`` matches the
    ``get`` callable the model builders take."""

    def __init__(self, root: str | os.PathLike):
        self.inventory = inspect_checkpoint(root)
        self._maps: dict[str, tuple[mmap.mmap, int]] = {}

    def _map(self, file: str):
        m = self._maps.get(file)
        if m is None:
            _, start = read_header(file)
            f = open(file, "rb")
            mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
            f.close()
            m = (mm, start)
            self._maps[file] = m
        return m

    def tensor(self, name: str) -> torch.Tensor:
        t = self.inventory.get(name)
        if t is None:
            raise KeyError(name)
        mm, start = self._map(t.file)
        buf = mm[start + t.begin:start + t.end]
        dt = TORCH_DTYPES[t.dtype]
        out = torch.frombuffer(bytearray(buf), dtype=torch.uint8).view(dt)
        return out.reshape(t.shape)

    def get(self, name: str, shape=None) -> torch.Tensor:
        x = self.tensor(name)
        if shape is not None and tuple(x.shape) != tuple(shape):
            raise SafetensorsError(f"{name}: shape {tuple(x.shape)} != expected {tuple(shape)}")
        return x.float() if x.dtype not in (torch.float8_e4m3fn, torch.float8_e5m2) else x

    def close(self):
        for mm, _ in self._maps.values():
            mm.close()
        self._maps.clear()


def save_safetensors(path: str | os.PathLike, tensors: dict[str, torch.Tensor], metadata=None) -> None:
    """Minimal writer (used by tests and the stage artifact builder)."""
    rev = {v: k for k, v in TORCH_DTYPES.items()}
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": rev[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
