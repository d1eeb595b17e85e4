"""Device-side failure detection without a GPU fault.

The one-shot all-reduce waits for a flag from every peer.  Here its group has two
"ranks" whose buffers both live on this GPU, and nothing plays rank 1, so rank 1's
flag is never raised: with a 1 ms wait limit the kernel must give up, record
kStatusTimeoutPeer (4) in the status block, leave the residual untouched and
return; the host turns that code into a TransportError.  The next call (a group
of one, the limit back at its default) must run clean.  A single kernel on one
GPU waits on a flag that nothing sets; no two kernels wait on each other.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _geometry(T, H):
    flags_off = 256
    partial_off = ((flags_off + 8 * 256 * 4 + 255) // 256) * 256
    max_elems = T * H
    recv_off = ((partial_off + max_elems * 2 + 255) // 256) * 256
    return flags_off, partial_off, recv_off, max_elems, recv_off + 2 * 8 * max_elems * 2


def test_peer_wait_times_out_and_the_next_call_runs_clean():
    from swarm_inference_lab_b200.ops._ext import ext
    from swarm_inference_lab_b200.ops.workspace import (KernelStatusError, PeerTimeoutError,
                                                        get_workspace)
    from swarm_inference_lab_b200.transport.stage_ring_net import TransportError

    e = ext()
    dev = torch.cuda.current_device()
    T, H = 4, 512
    flags_off, partial_off, recv_off, max_elems, nbytes = _geometry(T, H)
    mine = e.symm_alloc(nbytes, dev)
    silent_peer = e.symm_alloc(nbytes, dev)  # "rank 1": nobody raises its flags
    try:
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
        e.symm_tensor(mine, partial_off, T, H, dev).copy_(x)
        h = torch.zeros(T, H, dtype=torch.bfloat16, device="cuda")
        ws = get_workspace()
        ws.reset()
        ws.set_wait_limit_ns(1_000_000)  # 1 ms
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e.oneshot_allreduce(h, [mine, silent_peer], 0, flags_off, recv_off, partial_off,
                            max_elems, ws.status)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert ws.code() == 4
        assert elapsed < 1.0, elapsed  # the 1 ms limit, not the 2 s default
        with pytest.raises(TransportError) as info:
            ws.check()
        assert isinstance(info.value, PeerTimeoutError)
        assert isinstance(info.value, KernelStatusError) and info.value.code == 4
        assert torch.count_nonzero(h).item() == 0  # gave up before touching the residual
        # Recover: clear the code, restore the default limit, run a clean call.
        ws.clear_status()
        ws.set_wait_limit_ns(0)
        e.oneshot_allreduce(h, [mine], 0, flags_off, recv_off, partial_off, max_elems,
                            ws.status)
        torch.cuda.synchronize()
        assert ws.code() == 0
        ws.check()
        assert torch.equal(h, x)
    finally:
        torch.cuda.synchronize()
        e.symm_free(mine)
        e.symm_free(silent_peer)
        get_workspace().reset()


def test_wait_limit_lives_in_the_status_block():
    from swarm_inference_lab_b200.ops.workspace import get_workspace
    ws = get_workspace()
    ws.set_wait_limit_ns(123_456_789)
    assert int(ws.status.view(torch.int64)[1].item()) == 123_456_789
    assert ws.code() == 0
    ws.set_wait_limit_ns(0)
    assert int(ws.status.view(torch.int64)[1].item()) == 0
