"""MoE execution backends on CPU (fp32): a tiny Qwen3-MoE decoder whose routed experts run
locally, on whole-expert remote workers, as microshards split over two workers, or in a
hybrid placement chosen by the expert planner -- logits must equal the all-local decoder's
to fp32 rounding, and the remote workers must actually have served the rows."""
import asyncio
import threading

import pytest
import torch

from swarm_inference_lab_b200.models.config import ModelConfig
from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
from swarm_inference_lab_b200.runtime.expert_service import (ExpertClient, ExpertService,
                                                             ExpertStore, split_microshards,
                                                             Microshard)
from swarm_inference_lab_b200.runtime.moe_backends import (HybridMoEBackend, LocalMoEBackend,
                                                           MicroshardRemoteBackend,
                                                           WholeExpertRemoteBackend)

CFG = ModelConfig(name="tiny-moe-cpu", family="qwen3_moe", vocab_size=512, hidden_size=64,
                  num_layers=2, num_heads=4, num_kv_heads=2, head_dim=16, intermediate_size=96,
                  qk_norm=True, num_experts=8, num_experts_per_tok=2, moe_intermediate_size=48,
                  rms_norm_eps=1e-6)
LEASE = "lease-hash-1"


def _expert(get, layer, e):
    p = f"model.layers.{layer}.mlp.experts.{e}."
    I, H = CFG.moe_intermediate_size, CFG.hidden_size
    return get(p + "gate_proj.weight", (I, H)), get(p + "up_proj.weight", (I, H)), \
        get(p + "down_proj.weight", (H, I))


class _Servers:
    """Expert services on a background event loop (the decoder calls them synchronously)."""

    def __init__(self, stores):
        self.loop = asyncio.new_event_loop()
        self.thread = threading.Thread(target=self.loop.run_forever, daemon=True)
        self.thread.start()
        self.services = [ExpertService(s) for s in stores]
        for sv in self.services:
            sv.accept_lease(LEASE)
        self.ports = [asyncio.run_coroutine_threadsafe(sv.start(), self.loop).result(10)
                      for sv in self.services]

    def close(self):
        for sv in self.services:
            asyncio.run_coroutine_threadsafe(sv.close(), self.loop).result(10)
        self.loop.call_soon_threadsafe(self.loop.stop)
        self.thread.join(5)


@pytest.fixture(scope="module")
def setup():
    torch.set_num_threads(2)
    get = random_source(7, std=0.1)
    ids = torch.randint(0, CFG.vocab_size, (20,), generator=torch.Generator().manual_seed(3))
    base = ReferenceDecoder(CFG, get)
    ref = base.forward(ids, base.new_cache())
    I = CFG.moe_intermediate_size
    local, a, b, c = ExpertStore(), ExpertStore(), ExpertStore(), ExpertStore()
    for layer in range(CFG.num_layers):
        for e in range(CFG.num_experts):
            g, u, d = _expert(get, layer, e)
            local.add(Microshard(layer, e, 0, I), g, u, d)
            if e in (2, 3, 6):                      # whole experts on worker a
                a.add(Microshard(layer, e, 0, I), g, u, d)
            sh = split_microshards(layer, e, I, 2)  # every expert split over b and c
            b.add(sh[0], g, u, d)
            c.add(sh[1], g, u, d)
    srv = _Servers([a, b, c])
    yield get, ids, ref, local, srv
    srv.close()


def _run(get, ids, backend):
    dec = ReferenceDecoder(CFG, get)
    dec.moe_backend = backend
    return dec.forward(ids, dec.new_cache())


def test_local_backend_matches(setup):
    get, ids, ref, local, _ = setup
    out = _run(get, ids, LocalMoEBackend(local))
    assert (out - ref).abs().max().item() <= 1e-5


def test_microshard_backend_matches(setup):
    get, ids, ref, _, srv = setup
    shards = {(l, e): [ExpertClient("127.0.0.1", srv.ports[1]), ExpertClient("127.0.0.1", srv.ports[2])]
              for l in range(CFG.num_layers) for e in range(CFG.num_experts)}
    be = MicroshardRemoteBackend(shards, LEASE)
    try:
        out = _run(get, ids, be)
    finally:
        be.close()
    assert (out - ref).abs().max().item() <= 1e-5
    assert be.requests > 0 and srv.services[1].stats["rows"] > 0 and srv.services[2].stats["rows"] > 0


def test_hybrid_placement_from_the_planner_matches(setup):
    from swarm_inference_lab_b200.planner.expert_planner import ExpertDecision
    get, ids, ref, local, srv = setup
    decisions = []
    for layer in range(CFG.num_layers):
        for e in range(CFG.num_experts):
            if e in (2, 3, 6):
                decisions.append(ExpertDecision(layer, e, "whole_remote", ("a",), 0.1))
            elif e in (0, 5):
                decisions.append(ExpertDecision(layer, e, "microshard", ("b", "c"), 0.1))
            else:
                decisions.append(ExpertDecision(layer, e, "local", (), 0.1))
    whole = WholeExpertRemoteBackend({(l, e): ExpertClient("127.0.0.1", srv.ports[0])
                                      for l in range(CFG.num_layers) for e in (2, 3, 6)}, LEASE)
    cl_b, cl_c = ExpertClient("127.0.0.1", srv.ports[1]), ExpertClient("127.0.0.1", srv.ports[2])
    micro = MicroshardRemoteBackend({(l, e): [cl_b, cl_c] for l in range(CFG.num_layers)
                                     for e in (0, 5)}, LEASE)
    be = HybridMoEBackend.from_decisions(decisions, local=LocalMoEBackend(local), whole=whole,
                                         micro=micro)
    rows_a = srv.services[0].stats["rows"]
    try:
        out = _run(get, ids, be)
    finally:
        whole.close()
        micro.close()
    assert (out - ref).abs().max().item() <= 1e-5
    assert srv.services[0].stats["rows"] > rows_a and whole.requests > 0 and micro.requests > 0


def test_unaccepted_lease_is_refused(setup):
    get, ids, _, _, srv = setup
    be = WholeExpertRemoteBackend({(l, e): ExpertClient("127.0.0.1", srv.ports[0])
                                   for l in range(CFG.num_layers) for e in range(CFG.num_experts)},
                                  "someone-else")
    try:
        with pytest.raises(RuntimeError, match="route lease not accepted"):
            _run(get, ids, be)
    finally:
        be.close()


def test_build_and_validate_microshards(tmp_path):
    """``model build-microshards`` / ``validate-microshards`` on a tiny HF Qwen3-MoE
    checkpoint: 3 microshards per expert reproduce each expert; a tampered file and a missing
    slice are both reported."""
    import json

    import pytest
    transformers = pytest.importorskip("transformers")
    from safetensors.torch import load_file, save_file
    from typer.testing import CliRunner

    from swarm_inference_lab_b200.cli import app
    cfg = transformers.Qwen3MoeConfig(vocab_size=256, hidden_size=64, intermediate_size=96,
                                      moe_intermediate_size=40, num_hidden_layers=2,
                                      num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                                      num_experts=4, num_experts_per_tok=2, decoder_sparse_step=1,
                                      mlp_only_layers=[])
    torch.manual_seed(0)
    ck, out = tmp_path / "ck", tmp_path / "ms"
    transformers.Qwen3MoeForCausalLM(cfg).save_pretrained(ck, safe_serialization=True)
    run = CliRunner().invoke
    r = run(app, ["model", "build-microshards", str(ck), "--out", str(out), "--layers", "0,1",
                  "--experts", "1,3", "--parts", "3"])
    assert r.exit_code == 0, r.output
    assert json.loads(r.output)["microshards"] == 12
    r = run(app, ["model", "validate-microshards", str(out), str(ck)])
    rep = json.loads(r.output)
    assert r.exit_code == 0 and rep["ok"] and rep["experts"] == 4 and rep["max_rel_err"] < 1e-5
    # 40 channels in 3 parts: 14 + 13 + 13
    m0 = json.loads((out / "l000_e0001_s00.json").read_text())
    assert (m0["i0"], m0["i1"]) == (0, 14)
    f = out / "l001_e0003_s01.safetensors"
    t = load_file(str(f))
    t["down"] = t["down"] * 1.01
    save_file(t, str(f))
    (out / "l000_e0001_s02.json").unlink()
    r = run(app, ["model", "validate-microshards", str(out), str(ck)])
    rep = json.loads(r.output)
    assert r.exit_code == 1
    assert any("SHA-256" in p for p in rep["problems"])
    assert any("do not tile" in p for p in rep["problems"])


def test_expert_backends_harness_is_exact():
    from swarm_inference_lab_b200.testing.expert_backends import run
    rows = {r["backend"]: r for r in run(tokens=8, repeats=1)}
    assert set(rows) == {"local", "whole_remote", "microshard_2", "microshard_4"}
    assert all(r["exact"] for r in rows.values())
    assert rows["local"]["remote_rows_served"] == 0
    # microshards: every routed row goes to every shard of its expert
    assert rows["microshard_4"]["remote_rows_served"] == 2 * rows["microshard_2"]["remote_rows_served"] \
        == 4 * rows["whole_remote"]["remote_rows_served"] > 0
