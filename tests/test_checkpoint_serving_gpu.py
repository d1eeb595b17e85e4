"""``swarm run <checkpoint dir>`` on the GPU: a tiny random Hugging Face Qwen3 (and
Qwen3-MoE) checkpoint written by ``transformers`` together with a word-level tokenizer built
offline.  The CLI tokenizes the prompt, serves the checkpoint's own weights on the sm_100a
kernels (bf16) and detokenizes the output; its 32 greedy tokens are checked against HF's
fp32 model teacher-forced on them: each token is within the bf16 error bound of the fp32
maximum, and wherever the fp32 top-2 margin exceeds that bound it is the fp32 argmax.
"""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORDS = [f"w{i}" for i in range(1000)]


def _tokenizer(path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab = {"[UNK]": 0, "[BOS]": 1, "[EOS]": 2}
    for w in WORDS:
        vocab[w] = len(vocab)
    tok = Tokenizer(models.WordLevel(vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="[UNK]", bos_token="[BOS]",
                                   eos_token="[EOS]")
    fast.save_pretrained(path)
    return fast


def _model(kind):
    common = dict(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                  max_position_embeddings=1024, rms_norm_eps=1e-6, rope_theta=10000.0,
                  tie_word_embeddings=False, initializer_range=0.05, bos_token_id=1,
                  eos_token_id=2)
    if kind == "qwen3":
        from transformers import Qwen3Config, Qwen3ForCausalLM
        return Qwen3ForCausalLM(Qwen3Config(**common))
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM
    return Qwen3MoeForCausalLM(Qwen3MoeConfig(**common, num_local_experts=8, num_experts_per_tok=2,
                                              moe_intermediate_size=256, norm_topk_prob=True))


@pytest.mark.parametrize("kind", ["qwen3", "qwen3_moe"])
def test_swarm_run_serves_a_checkpoint_with_its_tokenizer(tmp_path, kind):
    torch.manual_seed(0)
    hf = _model(kind).float().eval()
    hf.save_pretrained(tmp_path, safe_serialization=True)
    tok = _tokenizer(tmp_path)
    prompt = " ".join(WORDS[i] for i in (5, 77, 300, 12, 999, 41, 8, 650, 123, 7))
    env = dict(os.environ, PYTHONPATH=ROOT)
    out = subprocess.run([sys.executable, "-m", "swarm_inference_lab_b200.cli", "run", str(tmp_path),
                          "--prompt", prompt, "--max-tokens", "32", "--ignore-eos", "--json"],
                         capture_output=True, text=True, env=env, cwd=ROOT, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert res["prompt_tokenization"] == "tokenizer"
    ids = tok.encode(prompt)
    assert res["prompt_tokens"] == len(ids)
    toks = res["tokens"]
    assert len(toks) == 32
    assert res["text"] == tok.decode(toks)
    with torch.no_grad():
        lg = hf(torch.tensor([ids + toks])).logits[0, len(ids) - 1:len(ids) - 1 + 32].float()
    tol = 0.02 * lg.abs().max().item() + 1e-3
    top2 = lg.topk(2, dim=-1).values
    # MoE: a near-tie in the router can send a token to another expert in bf16 than in fp32,
    # which moves that position's logits beyond the dense error bound; allow up to 3 such
    # positions of 32 there (dense: none).
    allowed = 3 if kind == "qwen3_moe" else 0
    decisive = bad = 0
    for i, t in enumerate(toks):
        ok = lg[i, t].item() >= top2[i, 0].item() - tol
        if (top2[i, 0] - top2[i, 1]).item() > tol:
            decisive += 1
            ok = ok and t == int(lg[i].argmax())
        bad += not ok
    assert bad <= allowed, (bad, toks, lg.argmax(-1).tolist())
    assert decisive >= 8, decisive
