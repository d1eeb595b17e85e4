"""The allocation-free decode-attention entry point, called through its exported C symbol.

Some embedders cannot allocate device memory while they run (their allocator
belongs to a host runtime, or they decode inside a capture that forbids
allocations); ``sil_paged_decode_noalloc`` serves them by keeping its split-K
scratch in a static device array.  This file is collected last so that a
failure here never hides the results of the other tests; it must pass both in
a fresh process and after the rest of the suite.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import swarm_inference_lab_b200._C as C  # noqa: F401  (loads libtorch deps first)
    lib = ctypes.CDLL(C.__file__)
    f = lib.sil_paged_decode_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                  ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    lib.sil_noalloc_last_error.restype = ctypes.c_char_p
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


def _call(lib, q, kc, vc, bt, sl, splits):
    B, hq, _ = q.shape
    out = torch.empty(B, hq * 128, dtype=torch.bfloat16, device="cuda")
    rc = lib.sil_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.shape[0], kc.shape[1],
        bt.data_ptr(), bt.stride(0), sl.data_ptr(), out.data_ptr(), out.stride(0), B, hq,
        1.0 / math.sqrt(128), splits, torch.cuda.current_stream().cuda_stream)
    return rc, out


def test_noalloc_matches_existing_entry_point_twice():
    from swarm_inference_lab_b200.ops import attention as A
    lib = _lib()
    for seed, lens, splits in ((1, [300, 70, 1000], 4), (2, [64, 2049, 5, 640], 3)):
        q, kc, vc, bt, sl = _case(seed, lens)
        rc, out = _call(lib, q, kc, vc, bt, sl, splits)
        assert rc == 0, lib.sil_noalloc_last_error()
        ref = A.paged_decode(q, kc, vc, bt, sl, num_splits=splits)
        torch.cuda.synchronize()
        assert (out.float() - ref.float()).abs().max().item() < 2e-2


def test_noalloc_rejects_oversized_requests():
    lib = _lib()
    q, kc, vc, bt, sl = _case(3, [64] * 8, hq=32, hkv=8)
    rc, _ = _call(lib, q, kc, vc, bt, sl, 10_000)
    assert rc == -2
    assert b"allocation-free" in lib.sil_noalloc_last_error()
