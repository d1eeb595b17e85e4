"""Metadata-only model facts: quantization names, GGUF variants, B200 feasibility,
bounded discovery and the model manifest (CPU)."""
import json

import pytest

from swarm_inference_lab_b200.config.models import ConfigError
from swarm_inference_lab_b200.model_io import facts
from swarm_inference_lab_b200.model_io.resolver import ModelSourceResolver

from test_model_io import _tiny_ckpt


@pytest.mark.parametrize("cfg,want", [
    ({}, None),
    ({"quantization_config": {"quant_method": "fp8", "fmt": "e4m3",
                              "weight_block_size": [128, 128]}}, "fp8-e4m3-b128"),
    ({"quantization_config": {"quant_method": "fp8"}}, "fp8-e4m3"),
    ({"quantization_config": {"quant_method": "awq", "bits": 4}}, "awq-int4"),
    ({"quantization_config": {"quant_method": "mxfp4"}}, "mxfp4"),
    ({"text_config": {"quantization_config": {"quant_method": "compressed-tensors", "config_groups": {
        "g0": {"weights": {"num_bits": 4, "type": "int", "strategy": "group", "group_size": 32}}}}}},
     "int4-g32"),
    ({"quantization_config": {"quant_method": "compressed-tensors", "config_groups": {
        "a": {"weights": {"num_bits": 4, "type": "int"}},
        "b": {"weights": {"num_bits": 8, "type": "float"}}}}}, "mixed:int4+fp8-e4m3"),
])
def test_quantization_scheme(cfg, want):
    assert facts.quantization_scheme(cfg) == want


def test_quant_names_and_kernels():
    assert facts.normalize_quant_name("float8_e4m3fn") == "fp8-e4m3"
    assert facts.normalize_quant_name("BFloat16") == "bf16"
    assert facts.normalize_quant_name("  ") is None
    assert facts.weight_dtype({"torch_dtype": "float16"}) == "f16"
    assert facts.canonical_scheme("fp8_block128") == "fp8-e4m3-b128"
    k, note = facts.b200_kernel_for("fp8-e4m3-b128")
    assert "f8f6f4" in k and note == "native"
    assert facts.b200_kernel_for(None)[0].startswith("tcgen05 bf16")
    assert facts.b200_kernel_for("fp8-e4m3")[0] is None
    assert facts.b200_kernel_for("mxfp4")[0] is None


def _gguf_listing():
    gb = 10**9
    return {
        "Q4_K_M/model-Q4_K_M-00001-of-00002.gguf": 20 * gb,
        "Q4_K_M/model-Q4_K_M-00002-of-00002.gguf": 18 * gb,
        "model-Q8_0.gguf": 70 * gb,
        "model-BF16-00001-of-00003.gguf": 50 * gb,       # incomplete split: dropped
        "model-BF16-00003-of-00003.gguf": 50 * gb,
        "model-IQ2_XXS.gguf": 17 * gb,
        "mmproj-model-f16.gguf": 1 * gb,                  # auxiliary: dropped
        "README.md": 100,
    }


def test_gguf_variants_grouping():
    vs = {v.variant_id: v for v in facts.discover_gguf_variants(_gguf_listing())}
    assert set(vs) == {"Q4_K_M", "Q8_0", "IQ2_XXS"}
    q4 = vs["Q4_K_M"]
    assert q4.total_bytes == 38 * 10**9 and len(q4.files) == 2 and q4.files[0].endswith("00001-of-00002.gguf")
    assert vs["Q8_0"].bits_per_weight == 8.5
    assert 4.5 < q4.bits_per_weight < 5.0
    assert vs["IQ2_XXS"].bits_per_weight < 2.5


def test_gguf_variant_selection():
    vs = facts.discover_gguf_variants(_gguf_listing())
    gb = 10**9
    assert facts.select_variant(vs, memory_bytes=180 * gb, objective="capacity").selected.quant == "Q8_0"
    # speed: fewest bytes among variants with >= 4 bits per weight
    assert facts.select_variant(vs, memory_bytes=180 * gb, objective="speed").selected.quant == "Q4_K_M"
    # balanced keeps 35% for the cache: Q8_0 (70 GB) does not leave it in 100 GB
    assert facts.select_variant(vs, memory_bytes=100 * gb).selected.quant == "Q4_K_M"
    with pytest.raises(ValueError):
        facts.select_variant(vs, memory_bytes=10 * gb)
    sel = facts.select_variant(vs, memory_bytes=40 * gb, request="Q8_0")
    assert sel.selected.quant == "Q8_0" and not sel.feasible
    with pytest.raises(ValueError):
        facts.select_variant(vs, memory_bytes=40 * gb, objective="fast")


def test_b200_feasibility(tmp_path):
    _tiny_ckpt(tmp_path)
    r = ModelSourceResolver().inspect(str(tmp_path))
    out = facts.b200_feasibility(r, batch=4, context=128)
    assert out["total_weight_bytes"] == sum(r.tensor_bytes.values())
    assert out["expert_bytes"] == 0 and out["layout"] == "tp1" and out["executable"]
    assert set(out["layer_bytes"]) == {"0", "1"}
    # GQA: 2 (k, v) x 1 kv head x 32 dims x 2 bytes x 2 layers
    assert out["kv_bytes_per_token"] == 2 * 1 * 32 * 2 * 2
    small = facts.b200_feasibility(r, gpu_bytes=out["total_weight_bytes"] // 3, usable_fraction=1.0,
                                   batch=1, context=1)
    assert small["gpus_for_target"] == 4 and small["layout"] == "tp4"


def test_kv_bytes_mla():
    from swarm_inference_lab_b200.models.config import KIMI_K2
    assert facts.kv_bytes_per_token(KIMI_K2) == (512 + 64) * 2 * KIMI_K2.num_layers


def test_discovery_bounded(tmp_path):
    _tiny_ckpt(tmp_path)
    rep = facts.discover_models([str(tmp_path), str(tmp_path), str(tmp_path / "missing")])
    assert rep["inspected"] == 2
    assert rep["records"][0]["status"] == "PROFILED" and rep["records"][0]["family"] == "qwen3"
    assert rep["records"][1]["status"] == "FAILED"
    with pytest.raises(ValueError):
        facts.discover_models([])
    with pytest.raises(ValueError):
        facts.discover_models([f"m{i}" for i in range(5)], limit=4)


def test_manifest_roundtrip_and_verify(tmp_path):
    ck = tmp_path / "ck"
    ck.mkdir()
    _tiny_ckpt(ck)
    r = ModelSourceResolver().inspect(str(ck))
    m = facts.build_manifest(r, [(0, 1), (1, 2)], workers=["w0", "w1"])
    assert [s.embed for s in m.stages] == [True, False] and [s.head for s in m.stages] == [False, True]
    assert sum(s.weight_bytes for s in m.stages) == sum(r.tensor_bytes.values())
    assert set(m.shard_hashes) == set(r.files)
    p = facts.save_manifest(m, tmp_path / "out" / "manifest.json")
    m2 = facts.load_manifest(p)
    assert m2 == m
    facts.verify_manifest_shards(m2, ck)
    summ = facts.manifest_summary(m2)
    assert summ["stage_layers"] == [[0, 1], [1, 2]] and summ["stages"] == 2
    f = sorted(r.files)[0]
    (ck / f).write_bytes((ck / f).read_bytes() + b"x")
    with pytest.raises(ConfigError, match="sha256"):
        facts.verify_manifest_shards(m2, ck)
    (ck / f).unlink()
    with pytest.raises(ConfigError, match="missing"):
        facts.verify_manifest_shards(m2, ck)
    (tmp_path / "bad.json").write_text(json.dumps({"model_id": "x"}))
    with pytest.raises(ConfigError):
        facts.load_manifest(tmp_path / "bad.json")
    with pytest.raises(ConfigError):
        facts.build_manifest(r, [(0, 1)])


def test_directory_hash_is_order_and_name_sensitive(tmp_path):
    a = tmp_path / "a"
    a.mkdir()
    (a / "x").write_bytes(b"1")
    (a / "y").write_bytes(b"2")
    h = facts.hash_directory(a)
    (a / "y").rename(a / "z")
    assert facts.hash_directory(a) != h


def test_cli_feasibility_and_variants(tmp_path):
    from typer.testing import CliRunner
    from swarm_inference_lab_b200.cli import app
    ck = tmp_path / "ck"
    ck.mkdir()
    _tiny_ckpt(ck)
    r = CliRunner().invoke(app, ["model", "feasibility", str(ck), "--batch", "2", "--ctx", "64"])
    assert r.exit_code == 0, r.output
    assert json.loads(r.output)["layout"] == "tp1"
    g = tmp_path / "g"
    g.mkdir()
    (g / "m-Q4_K_M.gguf").write_bytes(b"\0" * 400)
    (g / "m-Q8_0.gguf").write_bytes(b"\0" * 800)
    r = CliRunner().invoke(app, ["model", "variants", str(g), "--memory-gb", "5e-7",
                                 "--objective", "capacity"])
    assert r.exit_code == 0, r.output
    assert json.loads(r.output)["selected"] == "Q4_K_M"


def test_weight_bytes_count_tensors_and_skip_flags():
    """``nbytes`` of MoE weights counts every tensor (also inside (codes, scales) pairs) and
    skips the per-layer flags that sit beside them."""
    import dataclasses

    import torch

    from swarm_inference_lab_b200.models import config as C
    from swarm_inference_lab_b200.models.dense import TPInfo
    from swarm_inference_lab_b200.models.moe import MoEWeights
    cfg = dataclasses.replace(C.preset("mixtral-8x7b-shape"), hidden_size=256,
                              intermediate_size=512, moe_intermediate_size=512, num_layers=2,
                              vocab_size=1024, num_heads=4, num_kv_heads=2, head_dim=64)
    w = MoEWeights.random(cfg, TPInfo(0, 2), "cpu")
    expect = 0
    for t in [w.embed, w.final_norm, w.lm_head]:
        expect += t.numel() * t.element_size() if t is not None else 0
    for L in w.layers:
        for v in vars(L).values():
            if isinstance(v, torch.Tensor):
                expect += v.numel() * v.element_size()
    assert any(isinstance(v, bool) for v in vars(w.layers[0]).values())
    assert w.nbytes() == expect > 0
