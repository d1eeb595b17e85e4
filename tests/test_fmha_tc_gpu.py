"""Causal paged prefill attention on tcgen05 (S and O accumulators in TMEM) against the fp32
reference softmax(QK^T / sqrt(d)) V, over odd lengths, several 128-query tiles, chunked
prefill (queries at the end of a longer context), GQA groups and scattered pages; also
against the ``mma.sync`` prefill kernel."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(seed, qlens, ctxs, hq=8, hkv=2, pages=96):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(pages, hkv, 64, 128, device="cuda", generator=g).bfloat16()
    vc = torch.randn(pages, hkv, 64, 128, device="cuda", generator=g).bfloat16()
    maxp = max((c + 63) // 64 for c in ctxs)
    perm = torch.randperm(pages, generator=torch.Generator().manual_seed(seed))
    bt = torch.zeros(len(ctxs), maxp, dtype=torch.int32)
    used = 0
    for b, c in enumerate(ctxs):
        n = (c + 63) // 64
        bt[b, :n] = perm[used:used + n].int()
        used += n
    T = sum(qlens)
    # q as a strided view of a fused qkv row, like the model passes it
    qkv = torch.randn(T, (hq + 2 * hkv) * 128, device="cuda", generator=g).bfloat16()
    q = qkv.as_strided((T, hq, 128), (qkv.stride(0), 128, 1))
    cu = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0)), dtype=torch.int32, device="cuda")
    return q, kc, vc, bt.cuda(), torch.tensor(ctxs, dtype=torch.int32, device="cuda"), cu


def _oracle(q, kc, vc, bt, sl, cu):
    from swarm_inference_lab_b200.ops.attention import attention_reference
    outs = []
    for b in range(sl.shape[0]):
        L = int(sl[b])
        q0, q1 = int(cu[b]), int(cu[b + 1])
        pages = bt[b, :(L + 63) // 64].long()
        k = kc[pages].permute(0, 2, 1, 3).reshape(-1, kc.shape[1], 128)[:L]
        v = vc[pages].permute(0, 2, 1, 3).reshape(-1, vc.shape[1], 128)[:L]
        outs.append(attention_reference(q[q0:q1], k, v, causal_offset=L - (q1 - q0)).reshape(q1 - q0, -1))
    return torch.cat(outs)


@pytest.mark.parametrize("qlens,ctxs", [
    ([300], [300]),                       # three query tiles, the last partial
    ([17, 129, 256], [17, 129, 256]),     # odd lengths, exact multiples
    ([200, 64], [700, 64]),               # chunked prefill: queries at the end of the context
    ([1000], [1000]),
])
def test_fmha_tc_matches_fp32_reference(qlens, ctxs):
    from swarm_inference_lab_b200.ops import attention as A
    from swarm_inference_lab_b200.ops.workspace import get_workspace
    q, kc, vc, bt, sl, cu = _case(1, qlens, ctxs)
    out = A.paged_prefill(q, kc, vc, bt, sl, cu, max(qlens), kernel="tc")
    torch.cuda.synchronize()
    get_workspace().check()
    ref = _oracle(q, kc, vc, bt, sl, cu)
    err = (out.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 4e-3, err
    mma = A.paged_prefill(q, kc, vc, bt, sl, cu, max(qlens), kernel="mma")
    torch.cuda.synchronize()
    assert (out.float() - mma.float()).abs().max().item() <= 2e-2


def test_fmha_tc_gqa_group_of_four():
    from swarm_inference_lab_b200.ops import attention as A
    q, kc, vc, bt, sl, cu = _case(2, [190, 333], [190, 400], hq=16, hkv=4)
    out = A.paged_prefill(q, kc, vc, bt, sl, cu, 333, kernel="tc")
    ref = _oracle(q, kc, vc, bt, sl, cu)
    torch.cuda.synchronize()
    assert (out.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 4e-3
