"""Canonical tensor payloads for stage-ring frames (cross-host / CPU plumbing).

A tensor becomes row-major little-endian raw bytes regardless of strides or
device; the dtype, shape, byte order, raw and encoded lengths, SHA-256 and
codec name travel as frame attributes.  Compression is opt-in: the
``shuffle+zlib`` codec groups the bytes of each element position together
(so the exponent bytes of bf16 activations compress well) and is only used
when it shrinks the payload by the configured ratio.

Inside one box activations never take this path: stage boundaries use NCCL
p2p on device buffers (``parallel/pipeline.py``).

Reference: si/transport/stage_tensor.py:50-271 and
si/transport/compression.py:14-218 (same attribute contract, own codec).
"""
from __future__ import annotations

import hashlib
import sys
import zlib
from dataclasses import dataclass

import numpy as np
import torch

DTYPES = {
    "float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16,
    "int64": torch.int64, "int32": torch.int32, "int8": torch.int8, "uint8": torch.uint8,
    "bool": torch.bool, "float64": torch.float64,
}
NAMES = {v: k for k, v in DTYPES.items()}


class CodecError(ValueError):
    pass


@dataclass(frozen=True)
class PackedTensor:
    payload: bytes
    attributes: dict

    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(self.attributes["shape"])


def _raw_bytes(t: torch.Tensor) -> bytes:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        arr = t.view(torch.int16).numpy()
    else:
        arr = t.numpy()
    if sys.byteorder == "big":  # pragma: no cover
        arr = arr.byteswap()
    return arr.tobytes(order="C")


def _shuffle(raw: bytes, elem: int) -> bytes:
    if elem == 1:
        return raw
    a = np.frombuffer(raw, dtype=np.uint8).reshape(-1, elem)
    return a.T.copy().tobytes()


def _unshuffle(data: bytes, elem: int) -> bytes:
    if elem == 1:
        return data
    a = np.frombuffer(data, dtype=np.uint8).reshape(elem, -1)
    return a.T.copy().tobytes()


def pack_tensor(t: torch.Tensor, *, compression: str = "none", min_ratio: float = 0.9) -> PackedTensor:
    if t.dtype not in NAMES:
        raise CodecError(f"unsupported dtype {t.dtype}")
    raw = _raw_bytes(t)
    elem = t.element_size()
    codec = "raw"
    payload = raw
    if compression in ("shuffle+zlib", "adaptive") and raw:
        comp = zlib.compress(_shuffle(raw, elem), 1)
        if len(comp) <= min_ratio * len(raw):
            codec, payload = "shuffle+zlib", comp
    attrs = {
        "dtype": NAMES[t.dtype], "shape": list(t.shape), "byte_order": "little",
        "raw_length": len(raw), "encoded_length": len(payload), "codec": codec,
        "sha256": hashlib.sha256(raw).hexdigest(),
    }
    return PackedTensor(payload, attrs)


def unpack_tensor(payload: bytes, attrs: dict, device="cpu") -> torch.Tensor:
    try:
        dtype = DTYPES[attrs["dtype"]]
        shape = [int(x) for x in attrs["shape"]]
        codec = attrs["codec"]
    except KeyError as exc:
        raise CodecError(f"missing tensor attribute {exc}") from None
    if attrs.get("byte_order", "little") != "little":
        raise CodecError("only little-endian payloads are defined")
    if len(payload) != attrs["encoded_length"]:
        raise CodecError("encoded length mismatch")
    elem = torch.empty((), dtype=dtype).element_size()
    if codec == "raw":
        raw = payload
    elif codec == "shuffle+zlib":
        raw = _unshuffle(zlib.decompress(payload), elem)
    else:
        raise CodecError(f"unknown codec {codec}")
    if len(raw) != attrs["raw_length"]:
        raise CodecError("raw length mismatch")
    if hashlib.sha256(raw).hexdigest() != attrs["sha256"]:
        raise CodecError("tensor checksum mismatch")
    n = int(np.prod(shape)) if shape else 1
    if n * elem != len(raw):
        raise CodecError("shape does not match payload")
    if dtype == torch.bfloat16:
        arr = np.frombuffer(raw, dtype=np.int16).copy()
        t = torch.from_numpy(arr).view(torch.bfloat16)
    else:
        np_dtype = torch.empty((), dtype=dtype).numpy().dtype
        t = torch.from_numpy(np.frombuffer(raw, dtype=np_dtype).copy())
    return t.reshape(shape).to(device)
