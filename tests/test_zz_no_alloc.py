"""The allocation-free decode-attention entry point, called through its exported C symbol.

Some embedders cannot allocate device memory while they run (their allocator
belongs to a host runtime, or they decode inside a capture that forbids
allocations); ``sil_paged_decode_noalloc`` serves them by keeping its split-K
scratch in a static device array.  This file is collected last so that a
failure here never hides the results of the other tests; it must pass both in
a fresh process and after the rest of the suite.

The GPU cases compare against an fp32 softmax(QK^T)V oracle and against the
torch entry point (same kernel, so bit-equal for the same split count); the
argument checks run on the host only and need no GPU.
"""
import ctypes
import math

import pytest
import torch


def _lib():
    try:
        import swarm_inference_lab_b200._C as C  # noqa: F401  (loads libtorch deps first)
    except ImportError as exc:  # pragma: no cover - the build step has not run
        pytest.skip(f"kernel library not built: {exc}")
    lib = ctypes.CDLL(C.__file__)
    f = lib.sil_paged_decode_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                  ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    lib.sil_noalloc_last_error.restype = ctypes.c_char_p
    lib.sil_noalloc_status.restype = ctypes.c_int
    lib.sil_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    return lib


def _case(seed, lens, hq=8, hkv=2, pages=64):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(pages, hkv, 64, 128, device="cuda", generator=g).bfloat16()
    vc = torch.randn(pages, hkv, 64, 128, device="cuda", generator=g).bfloat16()
    maxp = max((L + 63) // 64 for L in lens)
    perm = torch.randperm(pages, generator=torch.Generator().manual_seed(seed))
    bt = torch.zeros(len(lens), maxp, dtype=torch.int32)
    used = 0
    for b, L in enumerate(lens):
        n = (L + 63) // 64
        bt[b, :n] = perm[used:used + n].int()
        used += n
    q = torch.randn(len(lens), hq, 128, device="cuda", generator=g).bfloat16()
    return q, kc, vc, bt.cuda(), torch.tensor(lens, dtype=torch.int32, device="cuda")


def _oracle(q, kc, vc, bt, sl):
    """fp32 softmax(q k^T / sqrt(128)) v over each sequence's pages -> [B, Hq*128]."""
    from swarm_inference_lab_b200.ops.attention import attention_reference
    outs = []
    for b in range(q.shape[0]):
        L = int(sl[b])
        pages = bt[b, :(L + 63) // 64].long()
        k = kc[pages].permute(0, 2, 1, 3).reshape(-1, kc.shape[1], 128)[:L]
        v = vc[pages].permute(0, 2, 1, 3).reshape(-1, vc.shape[1], 128)[:L]
        outs.append(attention_reference(q[b:b + 1], k, v, causal_offset=L - 1).reshape(-1))
    return torch.stack(outs)


def _call(lib, q, kc, vc, bt, sl, splits):
    B, hq, _ = q.shape
    out = torch.empty(B, hq * 128, dtype=torch.bfloat16, device="cuda")
    rc = lib.sil_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.shape[0], kc.shape[1],
        bt.data_ptr(), bt.stride(0), sl.data_ptr(), out.data_ptr(), out.stride(0), B, hq,
        1.0 / math.sqrt(128), splits, torch.cuda.current_stream().cuda_stream)
    return rc, out


def _status(lib):
    v = ctypes.c_int(-1)
    rc = lib.sil_noalloc_status(ctypes.byref(v), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sil_noalloc_last_error()
    return v.value


@pytest.mark.gpu
def test_noalloc_matches_existing_entry_point_twice():
    from swarm_inference_lab_b200.ops import attention as A
    lib = _lib()
    # splits 4 and 3 (split-K through the static scratch), 1 (direct store, no
    # counters), and 8 splits of a 5-token sequence (splits with no pages at all).
    cases = ((1, [300, 70, 1000], 4), (2, [64, 2049, 5, 640], 3), (4, [300, 70, 1000], 1),
             (5, [5, 129, 64], 8))
    for seed, lens, splits in cases:
        q, kc, vc, bt, sl = _case(seed, lens)
        ref32 = _oracle(q, kc, vc, bt, sl)
        prev = None
        for _ in range(2):  # two calls in a row share (and reuse) the static scratch
            rc, out = _call(lib, q, kc, vc, bt, sl, splits)
            assert rc == 0, lib.sil_noalloc_last_error()
            assert _status(lib) == 0
            torch.cuda.synchronize()
            err = (out.float() - ref32).abs().max().item()
            assert err <= 1e-2 * ref32.abs().max().item() + 2e-3, (splits, err)
            if prev is not None:
                assert torch.equal(out, prev)
            prev = out
        ref = A.paged_decode(q, kc, vc, bt, sl, num_splits=splits)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), (splits, (out.float() - ref.float()).abs().max().item())


@pytest.mark.gpu
def test_noalloc_reports_a_bad_page_through_its_status():
    lib = _lib()
    q, kc, vc, bt, sl = _case(6, [300, 200], pages=16)
    bad = bt.clone()
    bad[1, 1] = 16  # one past the last page: not loaded, reported as status 5
    rc, _ = _call(lib, q, kc, vc, bad, sl, 2)
    assert rc == 0, lib.sil_noalloc_last_error()
    assert _status(lib) == 5
    # The next call clears the status and runs clean.
    rc, out = _call(lib, q, kc, vc, bt, sl, 2)
    assert rc == 0 and _status(lib) == 0
    ref32 = _oracle(q, kc, vc, bt, sl)
    assert (out.float() - ref32).abs().max().item() <= 1e-2 * ref32.abs().max().item() + 2e-3


@pytest.mark.gpu
def test_noalloc_rejects_oversized_requests():
    lib = _lib()
    q, kc, vc, bt, sl = _case(3, [64] * 8, hq=32, hkv=8)
    rc, _ = _call(lib, q, kc, vc, bt, sl, 10_000)
    assert rc == -2
    assert b"allocation-free" in lib.sil_noalloc_last_error()
    # One split needs no scratch, so batch * kv_heads above the counter count is fine...
    n = lib.sil_noalloc_max_counters() // 8 + 1
    q2, kc2, vc2, bt2, sl2 = _case(7, [64] * n, hq=16, hkv=8, pages=n)
    rc, out = _call(lib, q2, kc2, vc2, bt2, sl2, 1)
    assert rc == 0, lib.sil_noalloc_last_error()
    assert _status(lib) == 0
    # ...but two splits need a counter per (sequence, kv-head).
    rc, _ = _call(lib, q2, kc2, vc2, bt2, sl2, 2)
    assert rc == -2


def test_noalloc_rejects_bad_arguments_on_the_host():
    """Argument checks return SIL_NOALLOC_EINVAL before any CUDA call (no GPU needed)."""
    lib = _lib()
    A16 = 1 << 20  # a 16-byte aligned stand-in address; never dereferenced on these paths

    def call(q=A16, q_stride=1024, k=A16, v=A16, pages=4, hkv=2, bt=A16, bt_stride=4, sl=A16,
             out=A16, out_stride=1024, batch=1, hq=8, splits=1):
        return lib.sil_paged_decode_noalloc(q, q_stride, k, v, pages, hkv, bt, bt_stride, sl, out,
                                            out_stride, batch, hq, 0.088, splits, None)

    cases = {
        "null q": dict(q=0), "null out": dict(out=0), "null block table": dict(bt=0),
        "odd q stride": dict(q_stride=1025), "short q stride": dict(q_stride=1022),
        "short out stride": dict(out_stride=1000), "zero bt stride": dict(bt_stride=0),
        "negative bt stride": dict(bt_stride=-4), "misaligned cache": dict(k=A16 + 8),
        "misaligned q": dict(q=A16 + 2), "odd out": dict(out=A16 + 1),
        "group of 32": dict(hq=64, q_stride=8192, out_stride=8192),
        "heads not a multiple": dict(hq=7, q_stride=896, out_stride=896),
        "zero batch": dict(batch=0), "zero splits": dict(splits=0),
    }
    for name, kw in cases.items():
        assert call(**kw) == -1, name
        assert lib.sil_noalloc_last_error(), name
