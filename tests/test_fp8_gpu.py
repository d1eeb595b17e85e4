"""Block-scaled fp8 GEMM (tcgen05 kind::f8f6f4) vs. fp32 dequantised references."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _mk(T, N, K, seed=0):
    from swarm_inference_lab_b200.ops import fp8
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g) * 0.05
    xq, xs = fp8.quantize(x)
    wq, ws = fp8.quantize_weight(w)
    return x, xq, xs, wq, ws


def test_quantize_matches_oracle():
    from swarm_inference_lab_b200.ops import fp8
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(5, 512, device="cuda", generator=g) * 3).bfloat16()
    q, s = fp8.quantize(x)
    deq = fp8.dequantize(q, s, 1)
    assert torch.allclose(s, x.float().abs().reshape(5, 4, 128).amax(-1) / 448.0, rtol=1e-6)
    # e4m3 rounding: half an ulp of 3 mantissa bits for normal values (2^-4 relative),
    # half the subnormal step 2^-9 (scaled back by the block scale) below 2^-6.
    step = s.repeat_interleave(128, dim=1) * 2.0 ** -10
    assert ((deq - x.float()).abs() <= x.float().abs() * 0.0625 + step + 1e-12).all()


@pytest.mark.parametrize("T", [1, 16, 33, 64, 130, 400])
@pytest.mark.parametrize("N,K", [(512, 1024), (1536, 7168)])
def test_fp8_linear(T, N, K):
    from swarm_inference_lab_b200.ops import fp8
    _, xq, xs, wq, ws = _mk(T, N, K)
    y = fp8.linear(xq, xs, wq, ws)
    ref = fp8.linear_reference(xq, xs, wq, ws)
    torch.cuda.synchronize()
    err = (y.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-2, err


@pytest.mark.parametrize("T", [8, 200])
def test_fp8_swiglu_and_residual(T):
    from swarm_inference_lab_b200.ops import fp8
    I, K = 256, 512
    _, xq, xs, wq, ws = _mk(T, 2 * I, K, seed=1)
    y = fp8.linear(xq, xs, wq, ws, epi=fp8.EPI_SWIGLU)
    gu = fp8.linear_reference(xq, xs, wq, ws)
    ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    assert (y.float() - ref).abs().max().item() < 2e-2 * ref.abs().max().item() + 1e-2
    _, xq2, xs2, wq2, ws2 = _mk(T, K, K, seed=2)
    r = torch.randn(T, K, device="cuda").bfloat16()
    out = fp8.linear(xq2, xs2, wq2, ws2, epi=fp8.EPI_RESADD, residual=r)
    ref2 = fp8.linear_reference(xq2, xs2, wq2, ws2) + r.float()
    assert (out.float() - ref2).abs().max().item() < 5e-2


@pytest.mark.parametrize("hint", [4, 100])
def test_fp8_grouped(hint):
    from swarm_inference_lab_b200.ops import fp8
    E, K, N = 5, 512, 256
    counts = torch.tensor([3, 0, 40, 1, 130])
    offs = torch.zeros(E + 1, dtype=torch.int32)
    offs[1:] = counts.cumsum(0)
    R = int(offs[-1])
    _, xq, xs, _, _ = _mk(R, N, K, seed=3)
    w = torch.randn(E * 2 * N, K, device="cuda") * 0.05
    wq, wsc = fp8.quantize_weight(w)
    out = fp8.grouped_linear(xq, xs, wq, wsc, offs.cuda(), E, swiglu=True, rows_hint=hint)
    torch.cuda.synchronize()
    wd = fp8.dequantize(wq, wsc, 128)
    xd = fp8.dequantize(xq, xs, 1)
    for g in range(E):
        a, b = int(offs[g]), int(offs[g + 1])
        if a == b:
            continue
        gu = xd[a:b] @ wd[g * 2 * N:(g + 1) * 2 * N].T
        ref = torch.nn.functional.silu(gu[:, :N]) * gu[:, N:]
        assert (out[a:b].float() - ref).abs().max().item() < 2e-2 * ref.abs().max().item() + 1e-2, g


@pytest.mark.parametrize("T,H", [(1, 7168), (37, 1536), (5, 2048), (3, 640)])
def test_rmsnorm_fp8_matches_rmsnorm_then_quantize(T, H):
    from swarm_inference_lab_b200.ops import fp8, norm
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = (torch.rand(H, device="cuda") + 0.5).bfloat16()
    y, q, s = norm.rmsnorm_fp8(x, w, 1e-6)
    y_ref = norm.rmsnorm(x, w, 1e-6)
    q_ref, s_ref = fp8.quantize(y_ref)
    assert torch.equal(y, y_ref)
    assert torch.equal(q, q_ref) and torch.equal(s, s_ref)
