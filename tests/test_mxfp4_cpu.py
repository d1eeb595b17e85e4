"""MXFP4 (OCP microscaling FP4: E2M1 codes, one E8M0 scale per 32 elements) and SiTU-GLU
oracle on CPU, against float64 arithmetic."""
import pytest
import torch

from swarm_inference_lab_b200.ops.mxfp4 import (E2M1_VALUES, mxfp4_dequantize, mxfp4_matmul,
                                                mxfp4_quantize, situ_glu)


def test_representable_values_round_trip_exactly():
    vals = torch.cat([E2M1_VALUES, -E2M1_VALUES[1:]])
    w = torch.zeros(3, 64)
    w[0, :15] = vals                        # block max 6 -> scale 2^0
    w[1, :15] = vals * 0.25                 # block max 1.5 -> scale 2^-2
    w[2, 32:47] = vals * 1024               # a second block with scale 2^10
    p, s = mxfp4_quantize(w)
    assert p.shape == (3, 32) and s.shape == (3, 2) and p.dtype == torch.uint8
    assert torch.equal(mxfp4_dequantize(p, s), w)
    assert int(s[0, 0]) == 127 and int(s[1, 0]) == 125 and int(s[2, 1]) == 137


def test_quantisation_error_bounds():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(16, 256, generator=g) * torch.rand(16, 1, generator=g) * 10
    p, s = mxfp4_quantize(w)
    deq = mxfp4_dequantize(p, s)
    blocks = w.reshape(16, 8, 32)
    scale = torch.exp2(s.float() - 127).unsqueeze(-1)
    # The block max maps into [4, 8) * scale; values up to 6 * scale round to the nearest
    # code (largest step 2: error <= 1 * scale), larger ones saturate at 6 * scale (error < 2 *
    # scale), and nothing exceeds 6 * scale.
    err = (deq.reshape(16, 8, 32) - blocks).abs()
    inside = blocks.abs() <= 6 * scale
    assert torch.all(err[inside] <= (1.0 * scale.expand_as(err))[inside] + 1e-6)
    assert torch.all(err <= 2.0 * scale + 1e-6)
    assert torch.all(deq.reshape(16, 8, 32).abs() <= 6 * scale + 1e-6)


def test_matmul_equals_dequantised_product():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(24, 96, generator=g)
    x = torch.randn(5, 96, generator=g)
    p, s = mxfp4_quantize(w)
    ref = x.double() @ mxfp4_dequantize(p, s).double().T
    assert (mxfp4_matmul(x, p, s).double() - ref).abs().max().item() < 1e-4


def test_ties_round_to_the_even_code():
    # 2.5 lies between 2 (code 4) and 3 (code 5): the even code wins; 5 between 4 and 6 -> 6
    w = torch.zeros(1, 32)
    w[0, 0], w[0, 1], w[0, 2], w[0, 3] = 6.0, 2.5, 5.0, 0.25
    p, s = mxfp4_quantize(w)
    d = mxfp4_dequantize(p, s)[0]
    assert d[1].item() == 2.0 and d[2].item() == 4.0 and d[3].item() == 0.0


def test_situ_glu_matches_float64_and_is_stable():
    g = torch.linspace(-80, 80, 401)
    u = torch.linspace(-5, 5, 401).flip(0)
    b1, b2 = 3.0, 2.0
    gd, ud = g.double(), u.double()
    ref = b1 * torch.tanh(gd / b1) * torch.sigmoid(gd) * b2 * torch.tanh(ud / b2)
    out = situ_glu(g, u, b1, b2)
    assert torch.isfinite(out).all()
    assert (out.double() - ref).abs().max().item() < 1e-5
    with pytest.raises(ValueError):
        situ_glu(g, u, 0.0, 1.0)
