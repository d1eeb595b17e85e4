"""SWARMEX1 expert packets and tensor codecs (cross-host expert offload).

Packet layout (all integers big-endian):

    b"SWARMEX1" | u32 header_len | u32 lengths_len | header (JSON, UTF-8)
               | lengths (u64 per blob) | blob_0 | blob_1 | ...

On a TCP stream every packet is preceded by its u64 length.  Tensor blobs are
described in the header (``tensors``: name, shape, codec, blob index[, scale blob]).

Codecs:
    raw_fp32          little-endian fp32
    raw_fp16          little-endian fp16
    raw_bf16          little-endian bf16 (2 bytes per value)
    int8_per_vector   int8 values plus one fp32 absmax/127 scale per row (lossy)

The packet structure and codec names match the reference's so peers interoperate
at the framing level (si/transport/expert.py:26-240; codec names
si/protocol/expert.py:67-72).
"""
from __future__ import annotations

import asyncio
import json
import struct
from dataclasses import dataclass, field

import numpy as np
import torch

MAGIC = b"SWARMEX1"
_HDR = struct.Struct(">II")
_LEN = struct.Struct(">Q")
MAX_PACKET = 1 << 31


class ExpertWireError(ValueError):
    pass


@dataclass
class ExpertPacket:
    header: dict
    blobs: list[bytes] = field(default_factory=list)


def encode_packet(p: ExpertPacket) -> bytes:
    h = json.dumps(p.header, sort_keys=True, separators=(",", ":")).encode()
    lengths = b"".join(_LEN.pack(len(b)) for b in p.blobs)
    return MAGIC + _HDR.pack(len(h), len(lengths)) + h + lengths + b"".join(p.blobs)


def decode_packet(buf: bytes | memoryview) -> ExpertPacket:
    buf = memoryview(buf)
    n0 = len(MAGIC) + _HDR.size
    if len(buf) < n0 or bytes(buf[: len(MAGIC)]) != MAGIC:
        raise ExpertWireError("not a SWARMEX1 packet")
    hl, ll = _HDR.unpack_from(buf, len(MAGIC))
    if ll % _LEN.size or n0 + hl + ll > len(buf):
        raise ExpertWireError("truncated packet header")
    try:
        header = json.loads(bytes(buf[n0:n0 + hl]))
    except ValueError as exc:
        raise ExpertWireError(f"bad header JSON: {exc}") from None
    off = n0 + hl
    lens = [_LEN.unpack_from(buf, off + i * _LEN.size)[0] for i in range(ll // _LEN.size)]
    off += ll
    blobs = []
    for n in lens:
        if off + n > len(buf):
            raise ExpertWireError("truncated blob")
        blobs.append(bytes(buf[off:off + n]))
        off += n
    if off != len(buf):
        raise ExpertWireError("trailing bytes after the last blob")
    return ExpertPacket(header, blobs)


# ------------------------------------------------------------------ codecs
def encode_tensor(p: ExpertPacket, name: str, t: torch.Tensor, codec: str = "raw_fp32") -> None:
    t = t.detach().cpu()
    meta = {"name": name, "shape": list(t.shape), "codec": codec, "blob": len(p.blobs)}
    if codec == "raw_fp32":
        p.blobs.append(t.float().contiguous().numpy().astype("<f4").tobytes())
    elif codec == "raw_fp16":
        p.blobs.append(t.half().contiguous().numpy().astype("<f2").tobytes())
    elif codec == "raw_bf16":
        p.blobs.append(t.bfloat16().contiguous().view(torch.int16).numpy().astype("<i2").tobytes())
    elif codec == "int8_per_vector":
        f = t.float().reshape(-1, t.shape[-1]) if t.dim() else t.float().reshape(1, 1)
        scale = f.abs().amax(dim=1).clamp_min(1e-30) / 127.0
        q = torch.round(f / scale[:, None]).clamp(-127, 127).to(torch.int8)
        p.blobs.append(q.numpy().tobytes())
        meta["scale_blob"] = len(p.blobs)
        p.blobs.append(scale.numpy().astype("<f4").tobytes())
    else:
        raise ExpertWireError(f"unknown codec {codec}")
    p.header.setdefault("tensors", []).append(meta)


def decode_tensor(p: ExpertPacket, name: str) -> torch.Tensor:
    for meta in p.header.get("tensors", []):
        if meta["name"] != name:
            continue
        shape = tuple(meta["shape"])
        blob = p.blobs[meta["blob"]]
        n = int(np.prod(shape)) if shape else 1
        c = meta["codec"]
        if c == "raw_fp32":
            a = np.frombuffer(blob, dtype="<f4", count=n)
            return torch.from_numpy(a.copy()).reshape(shape)
        if c == "raw_fp16":
            return torch.from_numpy(np.frombuffer(blob, dtype="<f2", count=n).copy()).float().reshape(shape)
        if c == "raw_bf16":
            a = np.frombuffer(blob, dtype="<i2", count=n).copy()
            return torch.from_numpy(a).view(torch.bfloat16).float().reshape(shape)
        if c == "int8_per_vector":
            q = torch.from_numpy(np.frombuffer(blob, dtype=np.int8, count=n).copy()).float()
            scale = torch.from_numpy(np.frombuffer(p.blobs[meta["scale_blob"]], dtype="<f4").copy())
            rows = scale.numel()
            return (q.reshape(rows, -1) * scale[:, None]).reshape(shape)
        raise ExpertWireError(f"unknown codec {c}")
    raise ExpertWireError(f"no tensor {name!r} in packet")


# ------------------------------------------------------------------ stream framing
async def write_packet(writer: asyncio.StreamWriter, p: ExpertPacket) -> int:
    data = encode_packet(p)
    writer.write(_LEN.pack(len(data)) + data)
    await writer.drain()
    return len(data)


async def read_packet(reader: asyncio.StreamReader, timeout: float | None = 30.0) -> ExpertPacket:
    n = _LEN.unpack(await asyncio.wait_for(reader.readexactly(_LEN.size), timeout))[0]
    if n > MAX_PACKET:
        raise ExpertWireError(f"packet of {n} bytes exceeds the limit")
    return decode_packet(await asyncio.wait_for(reader.readexactly(n), timeout))
