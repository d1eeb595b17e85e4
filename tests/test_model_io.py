"""Checkpoint inspection, architecture profiles, resolver and partitioning (CPU)."""
import json

import pytest
import torch
from hypothesis import given, settings, strategies as st

from swarm_inference_lab_b200.model_io import gguf, partition
from swarm_inference_lab_b200.model_io.architecture import TensorRole, classify_tensor, default_registry
from swarm_inference_lab_b200.model_io.resolver import ModelSourceResolver, ResolutionError
from swarm_inference_lab_b200.model_io.safetensors_io import (CheckpointReader, SafetensorsError,
                                                               inspect_checkpoint, save_safetensors)


def _tiny_ckpt(tmp_path, shards=2):
    cfg = {"model_type": "qwen3", "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 2,
           "num_key_value_heads": 1, "head_dim": 32, "intermediate_size": 128, "vocab_size": 100,
           "rms_norm_eps": 1e-6, "rope_theta": 10000.0}
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    tensors = {"model.embed_tokens.weight": torch.randn(100, 64), "model.norm.weight": torch.ones(64),
               "lm_head.weight": torch.randn(100, 64)}
    for i in range(2):
        p = f"model.layers.{i}."
        tensors.update({p + "self_attn.q_proj.weight": torch.randn(64, 64),
                        p + "self_attn.o_proj.weight": torch.randn(64, 64),
                        p + "mlp.down_proj.weight": torch.randn(64, 128),
                        p + "input_layernorm.weight": torch.ones(64)})
    names = sorted(tensors)
    wm = {}
    for s in range(shards):
        part = {n: tensors[n] for n in names[s::shards]}
        fn = f"model-{s:05d}.safetensors"
        save_safetensors(tmp_path / fn, part)
        wm.update({n: fn for n in part})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    return tensors


def test_safetensors_roundtrip_and_index(tmp_path):
    tensors = _tiny_ckpt(tmp_path)
    inv = inspect_checkpoint(tmp_path)
    assert set(inv) == set(tensors)
    r = CheckpointReader(tmp_path)
    for n, t in tensors.items():
        assert torch.equal(r.tensor(n), t)
    with pytest.raises(SafetensorsError):
        r.get("lm_head.weight", (1, 2))
    r.close()
    idx = json.loads((tmp_path / "model.safetensors.index.json").read_text())
    idx["weight_map"]["ghost"] = "model-00000.safetensors"
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(idx))
    with pytest.raises(SafetensorsError, match="missing"):
        inspect_checkpoint(tmp_path)


def test_resolver_profile_and_revision(tmp_path):
    _tiny_ckpt(tmp_path)
    res = ModelSourceResolver().inspect(str(tmp_path))
    assert res.profile.family == "qwen3" and res.profile.kind == "dense"
    assert res.revision.startswith("sha256:")
    assert res.profile.tensors["lm_head.weight"].role == TensorRole.OUTPUT_HEAD
    files0 = res.select_files(0, 1, embed=True, head=False)
    assert files0 and res.stage_bytes(0, 2, embed=True, head=True) == sum(res.tensor_bytes.values())
    rev = res.revision
    (tmp_path / "config.json").write_text((tmp_path / "config.json").read_text().replace("1e-06", "1e-05"))
    assert ModelSourceResolver().inspect(str(tmp_path)).revision != rev  # content-addressed


def test_resolver_rejects_unknown(tmp_path):
    with pytest.raises(ResolutionError):
        ModelSourceResolver().inspect(str(tmp_path / "nope"))
    with pytest.raises(ResolutionError, match="pin a revision"):
        ModelSourceResolver().inspect("hf://org/model")


def test_gguf_roundtrip(tmp_path):
    p = tmp_path / "m.gguf"
    gguf.write_gguf(p, {"general.architecture": "llama", "llama.block_count": 2,
                        "llama.embedding_length": 64, "tokenizer.ggml.tokens": ["a", "b"]},
                    [("token_embd.weight", (64, 10), 0, b"\0" * 2560),
                     ("blk.0.ffn_down.weight", (64, 64), 1, b"\0" * 8192)])
    d = gguf.inspect_gguf(p)
    assert d.architecture == "llama" and len(d.tensors) == 2
    assert d.tensors[1].type_name == "F16" and d.tensors[1].nbytes == 8192
    res = ModelSourceResolver().inspect(str(p))
    assert res.format == "gguf" and res.profile.num_layers == 2


def test_family_registry_covers_configs():
    reg = default_registry()
    for mt in ("llama", "mistral", "qwen3", "qwen3_moe", "mixtral", "deepseek_v3", "kimi_k2"):
        assert mt in reg.by_type
    cfg = {"model_type": "deepseek_v3", "hidden_size": 7168, "num_hidden_layers": 61,
           "num_attention_heads": 128, "num_key_value_heads": 128, "vocab_size": 129280,
           "n_routed_experts": 256, "num_experts_per_tok": 8, "moe_intermediate_size": 2048,
           "kv_lora_rank": 512, "q_lora_rank": 1536, "qk_nope_head_dim": 128, "qk_rope_head_dim": 64,
           "v_head_dim": 128, "intermediate_size": 18432, "n_shared_experts": 1,
           "first_k_dense_replace": 3, "n_group": 8, "topk_group": 4,
           "quantization_config": {"quant_method": "fp8", "weight_block_size": [128, 128]}}
    prof = reg.resolve_config(cfg)
    assert prof.attention == "mla" and prof.routing == "sigmoid_group"
    assert prof.quantization == "fp8_block128" and prof.config.first_k_dense == 3


@pytest.mark.parametrize("name,role", [
    ("model.layers.3.mlp.experts.7.down_proj.weight", TensorRole.ROUTED_EXPERT),
    ("model.layers.3.mlp.gate.weight", TensorRole.ROUTER),
    ("model.layers.3.mlp.shared_experts.up_proj.weight", TensorRole.SHARED_EXPERT),
    ("model.layers.0.self_attn.o_proj.weight", TensorRole.ATTENTION),
    ("model.norm.weight", TensorRole.FINAL_NORM),
])
def test_classify(name, role):
    d = classify_tensor(name)
    assert d.role == role


@settings(max_examples=60, deadline=None)
@given(st.integers(1, 40), st.integers(1, 8))
def test_equal_ranges_cover_each_layer_once(n, s):
    if n < s:
        with pytest.raises(partition.PartitionError):
            partition.equal_ranges(n, s)
        return
    r = partition.equal_ranges(n, s)
    assert r[0][0] == 0 and r[-1][1] == n
    assert all(a < b for a, b in r) and all(r[i][1] == r[i + 1][0] for i in range(s - 1))
    sizes = [b - a for a, b in r]
    assert max(sizes) - min(sizes) <= 1


@settings(max_examples=40, deadline=None)
@given(st.lists(st.floats(0.1, 10.0), min_size=2, max_size=16), st.integers(1, 4))
def test_balanced_ranges_is_optimal(costs, s):
    if len(costs) < s:
        return
    r = partition.balanced_ranges(costs, s)
    assert r[0][0] == 0 and r[-1][1] == len(costs)
    best = max(sum(costs[a:b]) for a, b in r)
    # no single-boundary move improves the bottleneck
    eq = partition.equal_ranges(len(costs), s)
    assert best <= max(sum(costs[a:b]) for a, b in eq) + 1e-9


def test_balanced_ranges_memory_cap():
    costs = [1.0] * 8
    mem = [1.0, 1.0, 5.0, 1.0, 1.0, 1.0, 1.0, 1.0]
    r = partition.balanced_ranges(costs, 3, mem=mem, mem_cap=6.0)
    assert all(sum(mem[a:b]) <= 6.0 for a, b in r)
    with pytest.raises(partition.PartitionError):
        partition.balanced_ranges(costs, 2, mem=mem, mem_cap=4.0)


def test_heterogeneous_capacities():
    r = partition.ranges_for_capacities([1.0] * 12, [2.0, 1.0], [100, 100], [1.0] * 12)
    assert r[0][1] - r[0][0] == 8  # the 2x faster stage takes twice the layers


def test_stage_artifact_build_transfer_resume_and_evict(tmp_path):
    from swarm_inference_lab_b200.cluster.artifacts import (ArtifactError, ArtifactStore,
                                                           build_stage_artifact, transfer)
    ck = tmp_path / "ck"
    ck.mkdir()
    tensors = _tiny_ckpt(ck)
    res = ModelSourceResolver().inspect(str(ck))
    src = ArtifactStore(tmp_path / "a")
    man = build_stage_artifact(res, src.root, 1, 2, embed=False, head=True)
    assert "lm_head.weight" in man.tensors and "model.embed_tokens.weight" not in man.tensors
    assert all(not n.startswith("model.layers.0.") for n in man.tensors)
    assert build_stage_artifact(res, src.root, 1, 2, embed=False, head=True).artifact_id == man.artifact_id
    assert src.verify(man.artifact_id)
    dst = ArtifactStore(tmp_path / "b")
    with pytest.raises(ArtifactError, match="interrupted"):
        transfer(src, dst, man.artifact_id, chunk=4096, fail_after_chunks=2)
    n = transfer(src, dst, man.artifact_id, chunk=4096)       # resumes after the 2 verified chunks
    total = -(-man.bytes // 4096)
    assert n == total - 2 and dst.verify(man.artifact_id)
    r = CheckpointReader(dst.path(man.artifact_id))
    assert torch.equal(r.tensor("lm_head.weight"), tensors["lm_head.weight"])
    r.close()
    other = build_stage_artifact(res, src.root, 0, 1, embed=True, head=False)
    src.lease(other.artifact_id)
    src.budget = 1
    gone = src.evict()
    assert man.artifact_id in gone and other.artifact_id not in gone


def test_cli_model_partition_and_shard(tmp_path):
    """``swarm model partition`` / ``shard`` on a tiny HF Llama checkpoint: contiguous
    intervals covering every layer, one artifact per stage holding exactly its tensors (the
    embedding on stage 0, norm and head on the last), each with a verified SHA-256."""
    import json

    import pytest
    transformers = pytest.importorskip("transformers")
    from typer.testing import CliRunner

    from swarm_inference_lab_b200.cli import app
    from swarm_inference_lab_b200.cluster.artifacts import ArtifactStore
    cfg = transformers.LlamaConfig(vocab_size=256, hidden_size=64, intermediate_size=96,
                                   num_hidden_layers=5, num_attention_heads=4,
                                   num_key_value_heads=2, tie_word_embeddings=False)
    ck = tmp_path / "ck"
    transformers.LlamaForCausalLM(cfg).save_pretrained(ck, safe_serialization=True)
    r = CliRunner().invoke(app, ["model", "partition", str(ck), "--stages", "2"])
    assert r.exit_code == 0, r.output
    st = json.loads(r.output)["stages"]
    assert [s["layers"] for s in st] in ([[0, 3], [3, 5]], [[0, 2], [2, 5]])
    out = tmp_path / "arts"
    r = CliRunner().invoke(app, ["model", "shard", str(ck), "--stages", "2", "--out", str(out)])
    assert r.exit_code == 0, r.output
    mans = json.loads(r.output)
    assert len(mans) == 2 and mans[0]["embed"] and mans[1]["head"]
    assert [m["layer_start"] for m in mans] == [s["layers"][0] for s in st]
    assert any("embed_tokens" in n for n in mans[0]["tensors"])
    assert any("lm_head" in n for n in mans[1]["tensors"])
    assert not any("embed_tokens" in n for n in mans[1]["tensors"])
    store = ArtifactStore(out)
    assert all(store.verify(m["artifact_id"]) for m in mans)
