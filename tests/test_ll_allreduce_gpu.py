"""The low-latency all-reduce kernel (one-shot and two-shot exchanges) on one GPU.

A group of two "ranks" whose buffers both live on this GPU; only rank 0 runs.  Rank 1's
words are written into rank 0's buffer before the call, exactly as rank 1's kernel would
send them (payload and epoch in every 8-byte word), so the single kernel finds every word it
waits for and no kernel waits on another.  Checked: rank 0's new residual row equals the
fp32 rank-ordered sum rounded once (the same bits as deterministic NCCL), the words rank 0
sent into rank 1's buffer (for two-shot: its partial for rank 1's slice, and its finished
slice), the epoch, and the fused RMSNorm output.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

T, H = 4, 512
LL_OFF = 256
MAX_ELEMS = T * H
PARTIAL_OFF = LL_OFF + 2 * 8 * MAX_ELEMS * 4
NBYTES = PARTIAL_OFF + MAX_ELEMS * 2


def _slot(buf, par, src, dev):
    """int32 view [T, H / 2, 2] of slot [par][src]: (bf16 pair, epoch) per 8-byte word."""
    from swarm_inference_lab_b200.ops._ext import ext
    words = MAX_ELEMS // 2  # 8-byte words per slot
    off = LL_OFF + (par * 8 + src) * words * 8
    return ext().symm_tensor(buf, off, T, H * 2, dev).view(torch.int32).view(T, H // 2, 2)


def _pairs(x):
    """bf16 [T, H] -> int32 [T, H / 2] (element 2k in the low half)."""
    return x.contiguous().view(torch.int32)


@pytest.mark.parametrize("two_shot", [False, True])
def test_ll_exchange_against_emulated_peer(two_shot):
    from swarm_inference_lab_b200.ops._ext import ext
    from swarm_inference_lab_b200.ops.workspace import get_workspace

    e = ext()
    dev = torch.cuda.current_device()
    mine = e.symm_alloc(NBYTES, dev)
    peer = e.symm_alloc(NBYTES, dev)
    try:
        for b in (mine, peer):
            e.symm_tensor(b, 0, 1, NBYTES // 2, dev).zero_()
        g = torch.Generator(device="cuda").manual_seed(7)
        p0 = (torch.randn(T, H, device="cuda", generator=g) * 0.5).bfloat16()
        p1 = (torch.randn(T, H, device="cuda", generator=g) * 0.5).bfloat16()
        h0 = torch.randn(T, H, device="cuda", generator=g).bfloat16()
        hn = (h0.float() + (p0.float() + p1.float())).bfloat16()
        e.symm_tensor(mine, PARTIAL_OFF, T, H, dev).copy_(p0)
        epoch, par = 1, 1  # the state word starts at 0
        inbox = _slot(mine, par, 1, dev)  # what rank 1 sends to rank 0
        half = H // 4  # int32 words per half row: slice 0 = elements 0..255
        if two_shot:
            inbox[:, :half, 0] = _pairs(p1)[:, :half]   # reduce-scatter: rank 1's partial, slice 0
            inbox[:, half:, 0] = _pairs(hn)[:, half:]   # all-gather: rank 1's finished slice 1
        else:
            inbox[:, :, 0] = _pairs(p1)
        inbox[:, :, 1] = epoch
        h = h0.clone()
        ws = get_workspace()
        ws.reset()
        e.ll_allreduce_norm(h, [mine, peer], 0, LL_OFF, PARTIAL_OFF, MAX_ELEMS, None, 0.0, None,
                            ws.status, two_shot)
        torch.cuda.synchronize()
        assert ws.code() == 0
        assert torch.equal(h, hn)
        sent = _slot(peer, par, 0, dev)  # what rank 0 sent to rank 1
        assert torch.all(sent[:, :, 1] == epoch)
        if two_shot:
            assert torch.equal(sent[:, half:, 0], _pairs(p0)[:, half:])
            assert torch.equal(sent[:, :half, 0], _pairs(hn)[:, :half])
        else:
            assert torch.equal(sent[:, :, 0], _pairs(p0))
        assert e.symm_tensor(mine, 0, 1, 2, dev).view(torch.int32).item() == epoch

        # Second call (epoch 2, parity 0) with the RMSNorm fused.
        epoch, par = 2, 0
        p1b = (torch.randn(T, H, device="cuda", generator=g) * 0.5).bfloat16()
        hn2 = (hn.float() + (p0.float() + p1b.float())).bfloat16()
        inbox = _slot(mine, par, 1, dev)
        if two_shot:
            inbox[:, :half, 0] = _pairs(p1b)[:, :half]
            inbox[:, half:, 0] = _pairs(hn2)[:, half:]
        else:
            inbox[:, :, 0] = _pairs(p1b)
        inbox[:, :, 1] = epoch
        w = (torch.rand(H, device="cuda", generator=g) + 0.5).bfloat16()
        x = torch.empty_like(h)
        e.ll_allreduce_norm(h, [mine, peer], 0, LL_OFF, PARTIAL_OFF, MAX_ELEMS, w, 1e-5, x,
                            ws.status, two_shot)
        torch.cuda.synchronize()
        assert ws.code() == 0
        assert torch.equal(h, hn2)
        ref = hn2.float() * torch.rsqrt(hn2.float().pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
        assert (x.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()
    finally:
        torch.cuda.synchronize()
        e.symm_free(mine)
        e.symm_free(peer)
        get_workspace().reset()


def test_set_up_timing_picks_a_mode_in_a_group_of_one():
    """The set-up timing that chooses between the exchanges (run at construction in groups of
    more than two ranks) runs both kernels, sums the timings over the group and leaves the
    communicator usable; here in a one-rank NCCL group."""
    import socket

    import torch.distributed as dist

    from swarm_inference_lab_b200.parallel.comm import NcclComm
    from swarm_inference_lab_b200.parallel.ll_tp import LLTPComm
    from swarm_inference_lab_b200.ops.workspace import get_workspace

    created = not dist.is_initialized()
    if created:
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0,
                                world_size=1, device_id=torch.device("cuda", torch.cuda.current_device()))
    comm = None
    try:
        comm = LLTPComm(NcclComm(), torch.device("cuda", torch.cuda.current_device()),
                        max_tokens=32, hidden=512)
        assert comm.two_shot is False and comm.tuning is None  # a group of one: one-shot
        pick = comm._pick_two_shot(tokens=32, iters=5)
        assert isinstance(pick, bool)
        assert comm.tuning["oneshot_ms_sum"] > 0 and comm.tuning["twoshot_ms_sum"] > 0
        get_workspace().check()
        # still usable: h += partial with the group's own (single) contribution
        g = torch.Generator(device="cuda").manual_seed(3)
        part = comm.partial_buffer(8, 512)
        part.copy_(torch.randn(8, 512, device="cuda", generator=g).bfloat16())
        h = torch.randn(8, 512, device="cuda", generator=g).bfloat16()
        expect = (h.float() + part.float()).bfloat16()
        comm.allreduce_partial_residual(h)
        torch.cuda.synchronize()
        assert torch.equal(h, expect)
    finally:
        if comm is not None:
            comm.close()
        if created:
            dist.destroy_process_group()


def test_set_up_timing_skips_an_exchange_that_reports_an_error():
    """If one exchange leaves an error code while it is timed (here a fake of the two-shot
    call that writes a peer-timeout code after the real call; no device fault), set-up counts
    it as infinitely slow, keeps the other one and clears the status word."""
    import socket

    import torch.distributed as dist

    from swarm_inference_lab_b200.ops.workspace import get_workspace
    from swarm_inference_lab_b200.parallel.comm import NcclComm
    from swarm_inference_lab_b200.parallel.ll_tp import LLTPComm

    created = not dist.is_initialized()
    if created:
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0,
                                world_size=1, device_id=torch.device("cuda", torch.cuda.current_device()))
    comm = None
    try:
        comm = LLTPComm(NcclComm(), torch.device("cuda", torch.cuda.current_device()),
                        max_tokens=32, hidden=512)
        real = comm._exchange

        def failing(h, norm_w, eps, x_out, status, two_shot=None):
            real(h, norm_w, eps, x_out, status, two_shot)
            if two_shot:
                status[0].fill_(4)  # what a peer wait that ran out records
        comm._exchange = failing
        with pytest.warns(RuntimeWarning, match="two-shot"):
            pick = comm._pick_two_shot(tokens=32, iters=3)
        assert pick is False
        assert comm.tuning["twoshot_ms_sum"] == float("inf") and comm.tuning["oneshot_ms_sum"] > 0
        assert get_workspace().code() == 0
    finally:
        if comm is not None:
            comm.__dict__.pop("_exchange", None)
            comm.close()
        if created:
            dist.destroy_process_group()
        get_workspace().reset()
