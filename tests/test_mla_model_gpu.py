"""DeepSeek-V3 / Kimi-K2 architecture (MLA + fp8 experts) on the sm_100a kernels against the
fp32 non-absorbed oracle."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(num_layers=None):
    from swarm_inference_lab_b200.models.config import TINY_MLA_GPU
    from swarm_inference_lab_b200.models.deepseek import MLAModel, MLAReference, MLAWeights
    from swarm_inference_lab_b200.models.dense import TPInfo
    w = MLAWeights.random(TINY_MLA_GPU, TPInfo(), "cuda", seed=3, num_layers=num_layers)
    return w, MLAModel(w, "cuda", max_positions=512), MLAReference(w)


@pytest.mark.parametrize("num_layers", [1, 3])
def test_mla_prefill_logits_match_oracle(num_layers):
    """One layer (MLA + dense fp8 MLP, no routing): every row within a few percent.  Three
    layers add routed experts, where a near-tie in top-k can send a token to another expert
    than the fp32 oracle does; those rows are allowed to differ, the rest must agree."""
    from swarm_inference_lab_b200.engine.kv_cache import PagedKVCache
    from swarm_inference_lab_b200.models.dense import ForwardBatch
    w, model, ref = _model(num_layers)
    kv = PagedKVCache(model.num_layers, 1, 8, "cuda", latent_dim=576)
    g = torch.Generator().manual_seed(0)
    lens = [37, 70]
    seqs = [torch.randint(0, 1024, (n,), generator=g) for n in lens]
    pages = [[0], [2, 5]]
    ids = torch.cat(seqs).cuda()
    pos = torch.cat([torch.arange(n) for n in lens]).to(torch.int32).cuda()
    slots = torch.cat([torch.tensor([pages[b][p // 64] * 64 + p % 64 for p in range(n)])
                       for b, n in enumerate(lens)]).to(torch.int32).cuda()
    bt = torch.tensor([[0, 0], [2, 5]], dtype=torch.int32, device="cuda")
    cu = torch.tensor([0, lens[0], sum(lens)], dtype=torch.int32, device="cuda")
    T = sum(lens)
    fb = ForwardBatch(ids=ids, positions=pos, slots=slots,
                      seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"), block_table=bt,
                      last_idx=torch.arange(T, device="cuda"), is_decode=False, cu_q=cu,
                      max_q_len=max(lens))
    logits = model.logits(model.forward_hidden(fb, kv), fb)
    off = 0
    for b, s in enumerate(seqs):
        r = ref.forward_logits(s.cuda())
        got = logits[off:off + lens[b]]
        off += lens[b]
        row_err = ((got - r).norm(dim=1) / r.norm(dim=1)).cpu()
        # e4m3 activations re-quantised from slightly different bf16 / fp32 inputs flip
        # codes near rounding boundaries: a few percent of relative error per row.
        if num_layers == 1:
            assert row_err.max().item() < 0.06, (b, row_err.max().item())
        else:
            assert row_err.median().item() < 0.06, (b, row_err.tolist())
            assert (row_err < 0.1).float().mean().item() >= 0.8, (b, row_err.tolist())


def test_mla_engine_greedy_decode_matches_oracle():
    from swarm_inference_lab_b200.engine.engine import LLMEngine, SamplingParams
    from swarm_inference_lab_b200.models.config import TINY_MLA_GPU
    w, _, ref = _model()
    eng = LLMEngine(TINY_MLA_GPU, device="cuda", weights=w, max_batch=4, max_seq_len=256)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (5, 40, 66)]
    outs, _ = eng.generate(prompts, SamplingParams(max_new_tokens=6))
    exact = total = 0
    for p, o in zip(prompts, outs):
        seq = list(p)
        for tok in o.token_ids:
            r = ref.forward_logits(torch.tensor(seq, device="cuda"))[-1]
            top = torch.topk(r, 5).indices.tolist()
            # Teacher-forced: every engine token is among the oracle's top 5 (a broken decode
            # path lands there with probability 5/1024), and most are its argmax (bf16/fp8
            # rounding and routing near-ties flip close calls).
            assert tok in top, (tok, top)
            exact += tok == top[0]
            total += 1
            seq.append(tok)
    assert exact >= 0.7 * total, (exact, total)
    from swarm_inference_lab_b200.ops.workspace import get_workspace
    get_workspace().check()
