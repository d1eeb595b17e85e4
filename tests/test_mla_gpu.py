"""MLA kernels (latent KV write, query split, absorbed paged attention) against fp32 references."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _latent_cache(ctxs, pages_total=96, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    cache = (torch.randn(pages_total, 64, 576, device="cuda", generator=g) * 0.5).bfloat16()
    perm = torch.randperm(pages_total, device="cuda", generator=g).to(torch.int32)
    maxp = max((c + 63) // 64 for c in ctxs)
    bt = torch.zeros(len(ctxs), maxp, dtype=torch.int32, device="cuda")
    off = 0
    for b, c in enumerate(ctxs):
        n = (c + 63) // 64
        bt[b, :n] = perm[off:off + n]
        off += n
    assert off <= pages_total
    return cache, bt


def _rows(cache, bt_row, n):
    idx = torch.arange(n, device="cuda")
    return cache[bt_row.long()[idx // 64], idx % 64]


def test_mla_kv_write_and_q_prep():
    from swarm_inference_lab_b200.ops import mla, rope
    T, H = 37, 8
    cs = rope.rope_cos_sin_table(4096, 64, 10000.0, device="cuda")
    kv = torch.randn(T, 640, device="cuda").bfloat16()          # padded row (576 used)
    w = torch.rand(512, device="cuda") + 0.5
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device="cuda")
    slots = torch.randperm(20 * 64, device="cuda")[:T].to(torch.int32)
    slots[3] = -1
    cache = torch.zeros(20, 64, 576, dtype=torch.bfloat16, device="cuda")
    mla.kv_write(kv, w, 1e-6, pos, slots, cs, cache)
    flat = cache.view(-1, 576)
    c = kv[:, :512].float()
    c_ref = c * torch.rsqrt(c.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    pe_ref = mla.rope_interleaved_reference(kv[:, 512:576], pos, cs)
    for t in range(T):
        if t == 3:
            continue
        row = flat[int(slots[t])].float()
        assert (row[:512] - c_ref[t]).abs().max().item() < 3e-2
        assert (row[512:] - pe_ref[t]).abs().max().item() < 3e-2
    q = torch.randn(T, H * 192, device="cuda").bfloat16()
    qn, qp = mla.q_prep(q, pos, cs, H)
    q3 = q.view(T, H, 192)
    assert torch.equal(qn, q3[:, :, :128].transpose(0, 1).contiguous())
    ref = mla.rope_interleaved_reference(q3[:, :, 128:], pos, cs)
    assert (qp.float() - ref).abs().max().item() < 3e-2
    src = torch.randn(H, T, 128, device="cuda").bfloat16()
    assert torch.equal(mla.heads_to_tokens(src, T, H), src.transpose(0, 1).reshape(T, H * 128))


@pytest.mark.parametrize("ctxs,splits", [([1, 100, 1000], 1), ([1, 100, 1000], 4),
                                         ([64, 2049], 7), ([33], 1)])
@pytest.mark.parametrize("H", [64, 16])
def test_mla_decode(ctxs, splits, H):
    from swarm_inference_lab_b200.ops import mla
    cache, bt = _latent_cache(ctxs, seed=len(ctxs) + splits)
    B = len(ctxs)
    g = torch.Generator(device="cuda").manual_seed(H)
    q_lat_hm = torch.randn(H, B, 512, device="cuda", generator=g).bfloat16() * 0.1
    q_lat = q_lat_hm.transpose(0, 1)                       # [B, H, 512] head-major storage
    q_pe = torch.randn(B, H, 64, device="cuda", generator=g).bfloat16() * 0.1
    sl = torch.tensor(ctxs, dtype=torch.int32, device="cuda")
    scale = 192 ** -0.5
    out = mla.attention(q_lat, q_pe, cache, bt, sl, scale=scale, num_splits=splits)
    for b, c in enumerate(ctxs):
        ref = mla.attention_reference(q_lat[b:b + 1], q_pe[b:b + 1], _rows(cache, bt[b], c), c - 1,
                                      scale)
        err = (out[b:b + 1].float() - ref).abs().max().item()
        assert err < 2e-2, (b, err)


@pytest.mark.parametrize("qlens,ctxs,H", [([70], [130], 64), ([5, 64], [5, 300], 16),
                                          ([1, 3], [1, 67], 64)])
def test_mla_prefill(qlens, ctxs, H):
    from swarm_inference_lab_b200.ops import mla
    cache, bt = _latent_cache(ctxs, seed=3)
    T = sum(qlens)
    q_lat = torch.randn(T, H, 512, device="cuda").bfloat16() * 0.1
    q_pe = torch.randn(T, H, 64, device="cuda").bfloat16() * 0.1
    cu = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0)), dtype=torch.int32, device="cuda")
    sl = torch.tensor(ctxs, dtype=torch.int32, device="cuda")
    scale = 192 ** -0.5
    out = mla.attention(q_lat, q_pe, cache, bt, sl, cu_q=cu, max_q_len=max(qlens), scale=scale)
    for b in range(len(qlens)):
        s, e = int(cu[b]), int(cu[b + 1])
        ref = mla.attention_reference(q_lat[s:e], q_pe[s:e], _rows(cache, bt[b], ctxs[b]),
                                      ctxs[b] - qlens[b], scale)
        err = (out[s:e].float() - ref).abs().max().item()
        assert err < 2e-2, (b, err)


def test_mla_status_clean():
    from swarm_inference_lab_b200.ops.workspace import get_workspace
    get_workspace().check()
