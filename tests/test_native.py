"""Host-side C++ runtime: CPU SwiGLU / fp8 oracle, SWRING01 codec, page allocator."""
import pytest
import torch

native = pytest.importorskip("swarm_inference_lab_b200._native")

from swarm_inference_lab_b200.protocol import stage_ring as sr


def _ref_swiglu(x, g, u, d):
    return (torch.nn.functional.silu(x @ g.T) * (x @ u.T)) @ d.T


def test_swiglu_f32_and_bf16():
    torch.manual_seed(0)
    x, g, u, d = torch.randn(3, 64), torch.randn(96, 64) * .1, torch.randn(96, 64) * .1, torch.randn(64, 96) * .1
    assert torch.allclose(native.swiglu_f32(x, g, u, d), _ref_swiglu(x, g, u, d), atol=1e-4)
    gb, ub, db = g.bfloat16(), u.bfloat16(), d.bfloat16()
    ref = _ref_swiglu(x, gb.float(), ub.float(), db.float())
    assert torch.allclose(native.swiglu_bf16(x, gb, ub, db), ref, atol=1e-4)


def _pack_int4(q):
    q = q.to(torch.uint8)
    return (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()


def test_swiglu_int4_g32():
    torch.manual_seed(1)
    H, I = 64, 64
    def mk(rows, cols):
        q = torch.randint(0, 16, (rows, cols))
        s = (torch.rand(rows, cols // 32) * 0.1).bfloat16()
        deq = (q - 8).float() * s.float().repeat_interleave(32, dim=1)
        return _pack_int4(q), s, deq
    gq, gs, g = mk(I, H)
    uq, us, u = mk(I, H)
    dq, ds, d = mk(H, I)
    x = torch.randn(2, H)
    out = native.swiglu_int4_g32(x, gq, gs, uq, us, dq, ds)
    assert torch.allclose(out, _ref_swiglu(x, g, u, d), atol=1e-3, rtol=1e-4)


def test_fp8_block_gemm_and_e4m3():
    torch.manual_seed(2)
    codes = torch.arange(256, dtype=torch.uint8)
    dec = native.e4m3_decode(codes)
    ref = codes.view(torch.float8_e4m3fn).float()
    ok = ~torch.isnan(ref)
    assert torch.equal(dec[ok], ref[ok])
    x = torch.randn(3, 256)
    xq, xs = native.quant_fp8_1x128(x)
    wf = torch.randn(128, 256)
    wq = wf.to(torch.float8_e4m3fn).view(torch.uint8)
    ws = torch.ones(1, 2)
    y = native.fp8_block_gemm(xq, xs, wq, ws)
    xd = native.e4m3_decode(xq) * xs.repeat_interleave(128, dim=1)
    ref = xd @ native.e4m3_decode(wq).T
    assert torch.allclose(y, ref, atol=1e-3, rtol=1e-4)


def test_ring_codec_matches_python():
    m = sr.StageMessage(sr.Operation.DECODE, "rev", "tok", "topo", 1, 2, 4, "s", "r", 7, 33, 0, 1,
                        (1, 8), "float32", payload=b"abc", attributes={"x": 1})
    py = sr.encode(m)
    meta = sr.canonical_json(m.metadata())
    cc = native.ring_encode(6, 0, 7, 33, 0, 1, meta, b"abc")
    assert cc == py
    op, flags, seq, pos, src, dst, meta2, payload = native.ring_decode(py)
    assert (op, seq, pos, src, dst, payload) == (6, 7, 33, 0, 1, b"abc") and meta2 == meta
    bad = bytearray(py)
    bad[-1] ^= 1
    with pytest.raises(ValueError, match="checksum"):
        native.ring_decode(bytes(bad))


def test_page_allocator():
    a = native.PageAllocator(4)
    p = a.alloc(3)
    assert a.free == 1 and sorted(p) == [0, 1, 2]
    a.retain([p[0]])
    a.release([p[0]])
    assert a.refcount(p[0]) == 1
    a.release(p)
    assert a.free == 4
    with pytest.raises(RuntimeError):
        a.release([p[0]])
    with pytest.raises(RuntimeError, match="out of KV pages"):
        a.alloc(5)
