"""Checkpoint loading on CPU: tiny random Hugging Face checkpoints written by
``transformers`` (Llama, Qwen3, Qwen3-MoE, Mixtral) are read through the loader's
canonical-name source and run by the fp32 reference decoder; logits must match HF's own
fp32 forward pass.  This pins the tensor-name mapping of every dense and MoE family."""
import pytest
import torch

transformers = pytest.importorskip("transformers")


def _tiny(model_type):
    common = dict(vocab_size=320, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                  max_position_embeddings=256, rms_norm_eps=1e-6, rope_theta=10000.0,
                  tie_word_embeddings=False, initializer_range=0.2)
    if model_type == "llama":
        from transformers import LlamaConfig, LlamaForCausalLM
        return LlamaForCausalLM(LlamaConfig(**common, attention_bias=False, mlp_bias=False))
    if model_type == "qwen3":
        from transformers import Qwen3Config, Qwen3ForCausalLM
        return Qwen3ForCausalLM(Qwen3Config(**common))
    if model_type == "qwen3_moe":
        from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM
        return Qwen3MoeForCausalLM(Qwen3MoeConfig(**common, num_experts=4, num_experts_per_tok=2,
                                                  moe_intermediate_size=32, norm_topk_prob=True,
                                                  decoder_sparse_step=1, mlp_only_layers=[]))
    if model_type == "mixtral":
        from transformers import MixtralConfig, MixtralForCausalLM
        c = dict(common)
        c.pop("head_dim")
        return MixtralForCausalLM(MixtralConfig(**c, num_local_experts=4, num_experts_per_tok=2))
    raise ValueError(model_type)


@pytest.mark.parametrize("model_type", ["llama", "qwen3", "qwen3_moe", "mixtral"])
def test_hf_checkpoint_loads_and_matches_hf_forward(tmp_path, model_type):
    from swarm_inference_lab_b200.model_io.loader import checkpoint_config, safetensors_source
    from swarm_inference_lab_b200.models.reference import ReferenceDecoder

    torch.manual_seed(0)
    hf = _tiny(model_type).float().eval()
    hf.save_pretrained(tmp_path, safe_serialization=True)
    cfg = checkpoint_config(tmp_path)
    assert cfg.family == model_type
    get = safetensors_source(tmp_path)
    ours = ReferenceDecoder(cfg, get, device="cpu", dtype=torch.float32)
    ids = torch.randint(0, cfg.vocab_size, (1, 12), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = hf(ids).logits[0].float()
        got = ours.forward(ids[0], ours.new_cache()).float()
    assert got.shape == ref.shape
    err = (got - ref).abs().max().item()
    assert err <= 1e-4 * max(1.0, ref.abs().max().item()), err


def test_name_mapping_and_fp8_dequantisation():
    from swarm_inference_lab_b200.model_io.loader import checkpoint_name, dequantize_block_fp8
    assert checkpoint_name("mixtral", "model.layers.3.mlp.experts.5.gate_proj.weight") == \
        "model.layers.3.block_sparse_moe.experts.5.w1.weight"
    assert checkpoint_name("mixtral", "model.layers.3.mlp.experts.5.up_proj.weight") == \
        "model.layers.3.block_sparse_moe.experts.5.w3.weight"
    assert checkpoint_name("mixtral", "model.layers.3.mlp.experts.5.down_proj.weight") == \
        "model.layers.3.block_sparse_moe.experts.5.w2.weight"
    assert checkpoint_name("mixtral", "model.layers.0.mlp.gate.weight") == \
        "model.layers.0.block_sparse_moe.gate.weight"
    assert checkpoint_name("qwen3_moe", "model.layers.0.mlp.gate.weight") == \
        "model.layers.0.mlp.gate.weight"
    # 130 x 200 weight, 128x128 blocks: scale rows / cols are ceil-divided.
    w = torch.randn(130, 200) * 0.1
    s = torch.rand(2, 2) + 0.5
    codes = (w / s.repeat_interleave(128, 0)[:130].repeat_interleave(128, 1)[:, :200]).to(
        torch.float8_e4m3fn)
    deq = dequantize_block_fp8(codes, s)
    expect = codes.float() * s.repeat_interleave(128, 0)[:130].repeat_interleave(128, 1)[:, :200]
    assert torch.equal(deq, expect)


def test_tokenizer_absent_is_none(tmp_path):
    from swarm_inference_lab_b200.model_io.loader import load_tokenizer
    assert load_tokenizer(tmp_path) is None


def test_deepseek_v3_checkpoint_builds_mla_weights(tmp_path):
    """A tiny HF DeepSeek-V3 checkpoint maps onto the MLA model's weights (names, shapes,
    the padded fused q_a / kv_a projection, fp8 128x128 quantisation of bf16 tensors)."""
    from transformers import DeepseekV3Config, DeepseekV3ForCausalLM

    from swarm_inference_lab_b200.model_io.loader import (checkpoint_config, fp8_source,
                                                          safetensors_source)
    from swarm_inference_lab_b200.models.deepseek import MLAWeights
    from swarm_inference_lab_b200.models.dense import TPInfo
    c = DeepseekV3Config(vocab_size=512, hidden_size=256, intermediate_size=384,
                         moe_intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                         num_key_value_heads=4, n_shared_experts=1, n_routed_experts=8,
                         num_experts_per_tok=2, n_group=2, topk_group=1, first_k_dense_replace=1,
                         q_lora_rank=256, kv_lora_rank=512, qk_nope_head_dim=128,
                         qk_rope_head_dim=64, v_head_dim=128, max_position_embeddings=1024,
                         tie_word_embeddings=False)
    torch.manual_seed(0)
    DeepseekV3ForCausalLM(c).save_pretrained(tmp_path, safe_serialization=True)
    cfg = checkpoint_config(tmp_path)
    assert cfg.mla and cfg.num_experts == 8 and cfg.first_k_dense == 1
    get = safetensors_source(tmp_path)

    def getd(name, shape, dt=torch.bfloat16):
        return get(name, shape).to(dt)

    w = MLAWeights.from_source(cfg, TPInfo(0, 2), getd, fp8_source(get), "cpu")
    L0, L1 = w.layers
    assert L0.dense and not L1.dense
    assert L0.w_qkv_a[0].shape == (896, 256)            # pad128(256 + 512 + 64) rows
    assert L1.experts_gate_up[0].shape == (4 * 2 * 128, 256)   # 4 local experts (EP 2)
    assert L1.router_bias.dtype == torch.float32 and L1.router_bias.shape == (8,)
    ref = get("model.layers.1.mlp.experts.0.gate_proj.weight", (128, 256))  # rank 0 owns 0..3
    q, s = L1.experts_gate_up
    deq = (q[:128].view(torch.float8_e4m3fn).float() * s[0].repeat_interleave(128)[None, :256])
    assert (deq - ref).abs().max().item() <= ref.abs().max().item() * 0.07


@pytest.mark.parametrize("model_type", ["llama", "qwen3_moe"])
def test_validate_checkpoint_headers_only(tmp_path, model_type):
    """``swarm model validate``: a complete checkpoint passes with every tensor used; a
    dropped tensor and a resized one are both reported, and the command exits 1."""
    import json

    from safetensors.torch import load_file, save_file
    from typer.testing import CliRunner

    from swarm_inference_lab_b200.cli import app
    torch.manual_seed(0)
    _tiny(model_type).save_pretrained(tmp_path, safe_serialization=True)
    r = CliRunner().invoke(app, ["model", "validate", str(tmp_path)])
    rep = json.loads(r.output)
    assert r.exit_code == 0 and rep["ok"] and rep["unused"] == [] and rep["tensors_checked"] > 10
    f = tmp_path / "model.safetensors"
    t = load_file(str(f))
    t.pop("model.layers.1.mlp.gate.weight" if model_type == "qwen3_moe"
          else "model.layers.1.mlp.down_proj.weight")
    t["model.layers.0.self_attn.o_proj.weight"] = t["model.layers.0.self_attn.o_proj.weight"][:, :8].contiguous()
    save_file(t, str(f), metadata={"format": "pt"})
    r = CliRunner().invoke(app, ["model", "validate", str(tmp_path)])
    rep = json.loads(r.output)
    assert r.exit_code == 1 and not rep["ok"]
    assert any(p.startswith("missing model.layers.1.mlp") for p in rep["problems"])
    assert any("o_proj.weight: shape" in p for p in rep["problems"])
