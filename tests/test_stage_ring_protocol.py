"""SWRING01 frame codec, limits and validators (CPU)."""
import hashlib
import struct

import pytest

from swarm_inference_lab_b200.protocol import stage_ring as sr


def _msg(**kw):
    base = dict(operation=sr.Operation.DECODE, model_revision="rev", tokenizer_revision="tok",
                topology_id="topo", stage_id=1, layer_start=2, layer_end=4, session_id="s1",
                request_id="r1", sequence_number=7, token_position=33, source_stage=0,
                destination_stage=1, tensor_shape=(1, 256), tensor_dtype="float32",
                payload=b"\x01\x02\x03", attributes={"k": 1})
    base.update(kw)
    return sr.StageMessage(**base)


def test_header_layout_and_roundtrip():
    m = _msg()
    f = sr.encode(m)
    assert sr.HEADER_SIZE == 76
    magic, ver, op, flags, mlen, plen, seq, pos, src, dst, digest = struct.unpack_from("<8sHHIIQQihh32s", f)
    assert magic == b"SWRING01" and ver == 1 and op == 6 and seq == 7 and pos == 33
    assert src == 0 and dst == 1 and plen == 3
    assert digest == hashlib.sha256(f[76:]).digest()
    back = sr.decode(f)
    assert back == m


def test_golden_metadata_is_canonical():
    m = _msg(payload=b"", tensor_shape=(), tensor_dtype="none", attributes={})
    f = sr.encode(m)
    meta = f[76:]
    assert meta.startswith(b'{"attributes":{},"compression_mode":"none","destination_stage":1,')
    assert b" " not in meta


@pytest.mark.parametrize("mutate", ["checksum", "magic", "version", "length", "op"])
def test_tamper_rejected(mutate):
    f = bytearray(sr.encode(_msg()))
    if mutate == "checksum":
        f[-1] ^= 1
    elif mutate == "magic":
        f[0] = ord("X")
    elif mutate == "version":
        f[8] = 9
    elif mutate == "length":
        f = f[:-1]
    elif mutate == "op":
        f[10] = 99
    with pytest.raises(sr.FrameError):
        sr.decode(bytes(f))


def test_header_metadata_disagreement_rejected():
    m = _msg()
    f = bytearray(sr.encode(m))
    # change header token position only: checksum still fine, metadata disagrees
    struct.pack_into("<i", f, 36, 34)
    with pytest.raises(sr.FrameError):
        sr.decode(bytes(f))


def test_limits():
    with pytest.raises(sr.FrameError):
        sr.encode(_msg(source_stage=40000))
    with pytest.raises(sr.FrameError):
        sr.encode(_msg(token_position=-2))


def test_sequence_validator():
    v = sr.SequenceValidator()
    v.check(_msg(sequence_number=0))
    v.check(_msg(sequence_number=1))
    with pytest.raises(sr.SequenceError, match="duplicate"):
        v.check(_msg(sequence_number=1))
    with pytest.raises(sr.SequenceError, match="stale"):
        v.check(_msg(sequence_number=0))
    with pytest.raises(sr.SequenceError, match="gap"):
        v.check(_msg(sequence_number=5))
    v.reset_session("s1")
    v.check(_msg(sequence_number=9))


def test_session_validator_pins():
    v = sr.SessionValidator(sr.SessionPin("rev", "topo", stage_id=1, layer_range=(2, 4)))
    v.check(_msg(operation=sr.Operation.OPEN_SESSION))
    v.check(_msg())
    with pytest.raises(sr.SessionError):
        v.check(_msg(operation=sr.Operation.OPEN_SESSION))  # opened twice
    with pytest.raises(sr.SessionError):
        v.check(_msg(model_revision="other"))
    with pytest.raises(sr.SessionError):
        v.check(_msg(layer_start=0))
    v.check(_msg(operation=sr.Operation.CLOSE_SESSION))
    with pytest.raises(sr.SessionError):
        v.check(_msg())


def test_tensor_codec_roundtrip_and_compression():
    import torch
    from swarm_inference_lab_b200.transport.tensor_codec import CodecError, pack_tensor, unpack_tensor
    t = torch.randn(4, 64).to(torch.bfloat16)[:, ::2]  # strided view
    for comp in ("none", "shuffle+zlib"):
        pk = pack_tensor(t, compression=comp, min_ratio=1.5)
        back = unpack_tensor(pk.payload, pk.attributes)
        assert torch.equal(back, t.contiguous())
    pk = pack_tensor(torch.zeros(1000))
    bad = dict(pk.attributes, sha256="0" * 64)
    with pytest.raises(CodecError):
        unpack_tensor(pk.payload, bad)
