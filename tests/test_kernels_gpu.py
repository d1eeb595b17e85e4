"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref_linear(x, w):
    return x.float() @ w.float().T


@pytest.mark.parametrize("T", [1, 7, 32, 100, 128, 129, 300])
@pytest.mark.parametrize("shape", [(512, 1024), (6144, 4096), (384, 1792)])
def test_gemm_plain(T, shape):
    from swarm_inference_lab_b200.ops import gemm
    N, K = shape
    g = torch.Generator(device="cuda").manual_seed(T * 7 + N)
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    y = gemm.linear(x, w)
    ref = _ref_linear(x, w)
    torch.cuda.synchronize()
    err = (y.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-2, err


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("splits", [0, 1, 3])
def test_gemm_modes_and_splits(mode, splits):
    from swarm_inference_lab_b200.ops import gemm
    T, N, K = 64, 1024, 2048
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    y = gemm.linear(x, w, force_mode=mode, force_splits=splits)
    ref = _ref_linear(x, w)
    torch.cuda.synchronize()
    assert (y.float() - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("T", [1, 16, 32, 64, 128])
@pytest.mark.parametrize("splits", [2, 5, 8, 13, 24])
@pytest.mark.parametrize("epi", ["plain", "residual", "swiglu", "fp32"])
def test_gemm_tile_aligned_splits(T, splits, epi):
    """Decode GEMMs with every tile split into equal K ranges (up to 8 per tile as one
    thread-block cluster reducing through shared memory, more through the global-memory
    fix-up): the partials are summed in K-range order, so the result matches the fp32
    reference and is bitwise identical from launch to launch."""
    from swarm_inference_lab_b200.ops import gemm
    N, K = (768, 1536) if epi == "swiglu" else (640, 1536)   # 3 / 5 tiles of 128 rows, 24 K blocks
    g = torch.Generator(device="cuda").manual_seed(T * 31 + splits)
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).bfloat16()
    h = torch.randn(T, N, device="cuda", generator=g).bfloat16()

    def run():
        if epi == "plain":
            return gemm.linear(x, w, force_mode=1, force_splits=splits)
        if epi == "fp32":
            return gemm.linear(x, w, fp32_out=True, force_mode=1, force_splits=splits)
        if epi == "swiglu":
            return gemm.linear(x, w, swiglu=True, force_mode=1, force_splits=splits)
        out = torch.empty_like(h)
        return gemm.linear(x, w, out=out, residual=h, force_mode=1, force_splits=splits)
    ys = [run() for _ in range(3)]
    torch.cuda.synchronize()
    ref = _ref_linear(x, w)
    if epi == "swiglu":
        ref = torch.nn.functional.silu(ref[:, :N // 2]) * ref[:, N // 2:]
    elif epi == "residual":
        ref = ref + h.float()
    err = (ys[0].float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-2, err
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])


def test_gemm_splits_beyond_resident_ctas():
    """More split CTAs than SMs (32 tiles x 8 K ranges): the tiles' clusters run in waves."""
    from swarm_inference_lab_b200.ops import gemm
    from swarm_inference_lab_b200.ops.workspace import get_workspace
    T, N, K = 32, 4096, 2048                       # 32 tiles x 8 splits = 256 CTAs
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    y = gemm.linear(x, w, force_mode=1, force_splits=8)
    y2 = gemm.linear(x, w, force_mode=1, force_splits=8)
    ref = _ref_linear(x, w)
    torch.cuda.synchronize()
    assert (y.float() - ref).abs().max().item() < 2e-2
    assert torch.equal(y, y2)
    get_workspace().check()


@pytest.mark.parametrize("T", [3, 32, 200])
def test_gemm_residual_inplace(T):
    from swarm_inference_lab_b200.ops import gemm
    N, K = 1024, 512
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    h = torch.randn(T, N, device="cuda").bfloat16()
    ref = _ref_linear(x, w) + h.float()
    gemm.linear(x, w, out=h, residual=h)
    torch.cuda.synchronize()
    assert (h.float() - ref).abs().max().item() < 5e-2


@pytest.mark.parametrize("T", [1, 32, 128, 257])
def test_gemm_swiglu(T):
    from swarm_inference_lab_b200.ops import gemm
    I, K = 768, 1024
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(2 * I, K, device="cuda") * 0.05).bfloat16()
    y = gemm.linear(x, w, swiglu=True)
    gu = _ref_linear(x, w)
    ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    torch.cuda.synchronize()
    assert (y.float() - ref).abs().max().item() < 3e-2 * ref.abs().max().item() + 1e-2


@pytest.mark.parametrize("T", [2, 32, 160])
def test_gemm_fp32_logits(T):
    from swarm_inference_lab_b200.ops import gemm
    V, K = 4000, 512  # V not a multiple of the tile
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(V, K, device="cuda") * 0.05).bfloat16()
    y = gemm.linear(x, w, fp32_out=True)
    ref = _ref_linear(x, w)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32
    assert (y - ref).abs().max().item() < 1e-3 * ref.abs().max().item() + 1e-3


def test_rmsnorm_and_residual():
    from swarm_inference_lab_b200.ops import norm
    T, H = 37, 4096
    x = torch.randn(T, H, device="cuda").bfloat16()
    r = torch.randn(T, H, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    y = norm.rmsnorm(x, w, 1e-5)
    ref = norm.rmsnorm_reference(x, w, 1e-5)
    assert (y.float() - ref.float()).abs().max().item() < 2e-2
    r2 = r.clone()
    y2 = norm.rmsnorm(x, w, 1e-5, residual=r2)
    s = (x.float() + r.float()).bfloat16()
    assert torch.equal(r2, s)
    ref2 = norm.rmsnorm_reference(s, w, 1e-5)
    assert (y2.float() - ref2.float()).abs().max().item() < 2e-2


def _make_cache(pages, hkv):
    k = torch.zeros(pages, hkv, 64, 128, device="cuda", dtype=torch.bfloat16)
    return k, torch.zeros_like(k)


@pytest.mark.parametrize("qk_norm", [False, True])
def test_rope_kv_write(qk_norm):
    from swarm_inference_lab_b200.ops import rope
    from swarm_inference_lab_b200.models.reference import _rms
    T, Hq, Hkv = 5, 4, 2
    qkv = torch.randn(T, (Hq + 2 * Hkv) * 128, device="cuda").bfloat16()
    orig = qkv.clone()
    pos = torch.tensor([0, 1, 63, 64, 200], dtype=torch.int32, device="cuda")
    slots = torch.tensor([3 * 64 + 0, 3 * 64 + 1, 3 * 64 + 63, 5 * 64 + 0, -1], dtype=torch.int32, device="cuda")
    cs = rope.rope_cos_sin_table(512, 128, 10000.0, device="cuda")
    kc, vc = _make_cache(8, Hkv)
    qn = (1 + 0.1 * torch.randn(128, device="cuda")).bfloat16() if qk_norm else None
    kn = (1 + 0.1 * torch.randn(128, device="cuda")).bfloat16() if qk_norm else None
    rope.rope_kv_write(qkv, pos, slots, cs, kc, vc, Hq, Hkv, qn, kn, 1e-6)
    q = orig[:, : Hq * 128].view(T, Hq, 128)
    k = orig[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128)
    v = orig[:, (Hq + Hkv) * 128:].view(T, Hkv, 128)
    if qk_norm:
        q, k = _rms(q, qn, 1e-6), _rms(k, kn, 1e-6)
    qr = rope.apply_rope_reference(q, pos, cs)
    kr = rope.apply_rope_reference(k, pos, cs)
    assert (qkv[:, : Hq * 128].view(T, Hq, 128).float() - qr.float()).abs().max() < 3e-2
    for i in range(4):
        s = int(slots[i])
        assert (kc[s // 64, :, s % 64].float() - kr[i].float()).abs().max() < 3e-2
        assert torch.equal(vc[s // 64, :, s % 64], v[i])


def _fill_paged(lens, hkv, pages_total=64, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(pages_total, hkv, 64, 128, device="cuda", generator=g).bfloat16()
    vc = torch.randn(pages_total, hkv, 64, 128, device="cuda", generator=g).bfloat16()
    perm = torch.randperm(pages_total, generator=torch.Generator().manual_seed(seed)).tolist()
    maxp = max((L + 63) // 64 for L in lens)
    bt = torch.zeros(len(lens), maxp, dtype=torch.int32)
    used = 0
    for b, L in enumerate(lens):
        n = (L + 63) // 64
        bt[b, :n] = torch.tensor(perm[used:used + n])
        used += n
    return kc, vc, bt.cuda()


def _gather(kc, bt_row, L):
    n = (L + 63) // 64
    pages = kc[bt_row[:n].long()]              # [n, Hkv, 64, D]
    return pages.permute(0, 2, 1, 3).reshape(n * 64, kc.shape[1], 128)[:L]


@pytest.mark.parametrize("lens,hq,hkv,splits", [([1], 4, 2, 1), ([70, 5, 130], 8, 2, 1),
                                                ([300, 1000, 64], 32, 8, 4), ([2049], 16, 1, 7)])
def test_paged_decode(lens, hq, hkv, splits):
    from swarm_inference_lab_b200.ops import attention as A
    kc, vc, bt = _fill_paged(lens, hkv, pages_total=96)
    B = len(lens)
    q = torch.randn(B, hq, 128, device="cuda").bfloat16()
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = A.paged_decode(q, kc, vc, bt, sl, num_splits=splits)
    for b, L in enumerate(lens):
        k = _gather(kc, bt[b], L)
        v = _gather(vc, bt[b], L)
        ref = A.attention_reference(q[b:b + 1], k, v, causal_offset=L - 1)
        got = out[b].view(hq, 128).float()
        assert (got - ref[0]).abs().max().item() < 2e-2, (b, L)


@pytest.mark.parametrize("qlens,ctx,hq,hkv", [([5], [5], 4, 2), ([100, 64, 1], [100, 64, 1], 8, 2),
                                             ([130, 10], [200, 400], 32, 8), ([257], [257], 4, 4)])
def test_paged_prefill(qlens, ctx, hq, hkv):
    from swarm_inference_lab_b200.ops import attention as A
    kc, vc, bt = _fill_paged(ctx, hkv, pages_total=64, seed=1)
    T = sum(qlens)
    q = torch.randn(T, hq, 128, device="cuda").bfloat16()
    cu = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0)), dtype=torch.int32, device="cuda")
    sl = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    out = A.paged_prefill(q, kc, vc, bt, sl, cu, max(qlens))
    for b in range(len(qlens)):
        k = _gather(kc, bt[b], ctx[b])
        v = _gather(vc, bt[b], ctx[b])
        qs = q[int(cu[b]):int(cu[b + 1])]
        ref = A.attention_reference(qs, k, v, causal_offset=ctx[b] - qlens[b])
        got = out[int(cu[b]):int(cu[b + 1])].view(-1, hq, 128).float()
        assert (got - ref).abs().max().item() < 2e-2, b


def test_argmax_ties_lowest():
    from swarm_inference_lab_b200.ops import sampling
    x = torch.randn(6, 50001, device="cuda")
    x[2, 17] = 100.0
    x[2, 40000] = 100.0
    out = sampling.argmax(x)
    ref = torch.argmax(x, dim=1)
    assert out[2].item() == 17
    assert torch.equal(out, ref)


@pytest.mark.parametrize("V", [128256, 4096, 1000, 163840])
def test_argmax_split_rows(V):
    """Rows split over a cluster of CTAs (V >= 4096) or one CTA (short rows): the maximum
    in any quarter of the row, ties across quarters resolved to the lowest index."""
    from swarm_inference_lab_b200.ops import sampling
    g = torch.Generator(device="cuda").manual_seed(V)
    x = torch.randn(33, V, device="cuda", generator=g)
    x[0, V - 1] = 50.0                       # in the last quarter
    x[1, 3] = 50.0
    x[1, V - 2] = 50.0                       # tie across the first and last quarter
    x[2, V // 2] = 50.0
    x[2, V // 2 + 1] = 50.0                  # tie inside one quarter
    out = sampling.argmax(x)
    assert out[0].item() == V - 1 and out[1].item() == 3 and out[2].item() == V // 2
    assert torch.equal(out, torch.argmax(x, dim=1))


def test_status_word_clean():
    from swarm_inference_lab_b200.ops.workspace import get_workspace
    get_workspace().check()


def test_sampling_distribution_matches_reference():
    from swarm_inference_lab_b200.ops import sampling
    torch.manual_seed(0)
    V, N = 64, 4000
    base = torch.randn(1, V, device="cuda") * 2
    for temp, k, p in [(1.0, 0, 1.0), (0.7, 10, 1.0), (1.3, 0, 0.8), (1.0, 20, 0.9)]:
        logits = base.repeat(N, 1).contiguous()
        toks = sampling.sample(logits, temperature=temp, top_k=k, top_p=p,
                               seeds=torch.arange(N, device="cuda"), offsets=0)
        emp = torch.bincount(toks, minlength=V).float() / N
        ref = sampling.sample_reference_probs(base, temp, k, p)[0]
        assert (emp[ref == 0] == 0).all(), (temp, k, p)        # truncation is exact
        assert (emp - ref).abs().max().item() < 0.04, (temp, k, p)


def test_sampling_greedy_and_penalty():
    from swarm_inference_lab_b200.ops import sampling
    logits = torch.tensor([[1.0, 5.0, 4.9, -1.0]], device="cuda")
    assert sampling.sample(logits.clone(), temperature=0.0).item() == 1
    hist = torch.tensor([[1]], dtype=torch.int64, device="cuda")
    out = sampling.sample(logits.clone(), temperature=0.0, repetition_penalty=2.0, history=hist,
                          history_len=torch.tensor([1], dtype=torch.int32, device="cuda"))
    assert out.item() == 2
