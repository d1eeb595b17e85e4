"""The cluster product end to end on CPU, one OS process per role.

1. ``swarm cluster create`` + ``swarm cluster start`` (coordinator process), two
   ``swarm node join`` + ``swarm node agent`` (worker processes that register and
   heartbeat over mutual-TLS gRPC), then ``swarm run tiny-llama-cpu
   --require-distributed --stages 2``: the coordinator deploys the 4-layer tiny Llama as
   2 pipeline stages (signed route leases, HELLO handshakes) and streams the request
   through the stage ring.  Tokens and every step's logits must match a single-process
   fp32 run to 1e-5.
2. A node killed mid-decode (SIGKILL between two tokens) is detected by the
   coordinator's probe, replaced by a spare node under route generation + 1, and the
   request is replayed and finished with the same tokens.

BASELINE config #1 (CPU plumbing): batch 1, 32 prompt ids uniform in [0, 32000) from
seed 0, greedy decode 64 tokens.
"""
import asyncio
import json
import os
import random
import signal
import socket
import subprocess
import sys
import time

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PROMPT = torch.randint(0, 32000, (32,), generator=torch.Generator().manual_seed(0)).tolist()
NEW = 64


def _free_pair() -> int:
    for _ in range(200):
        p = random.randint(20000, 60000)
        ok = True
        for q in (p, p + 1):
            with socket.socket() as s:
                try:
                    s.bind(("127.0.0.1", q))
                except OSError:
                    ok = False
        if ok:
            return p
    raise RuntimeError("no free port pair")


def _env():
    return dict(os.environ, PYTHONPATH=ROOT, OMP_NUM_THREADS="2", CUDA_VISIBLE_DEVICES="")


def _swarm(*args, timeout=120, check=True):
    out = subprocess.run([sys.executable, "-m", "swarm_inference_lab_b200.cli", *args],
                         capture_output=True, text=True, env=_env(), cwd=ROOT, timeout=timeout)
    if check and out.returncode != 0:
        raise AssertionError(f"swarm {' '.join(args)} failed:\n{out.stdout}\n{out.stderr[-3000:]}")
    return out


def _start_agent(state, ready):
    return subprocess.Popen([sys.executable, "-m", "swarm_inference_lab_b200.cli", "node", "agent",
                             "--state-dir", str(state), "--ready-file", str(ready)],
                            env=_env(), cwd=ROOT, stdout=subprocess.DEVNULL,
                            stderr=subprocess.PIPE, start_new_session=True)


def _wait_file(path, proc=None, timeout=90):
    t0 = time.time()
    while not os.path.exists(path):
        if proc is not None and proc.poll() is not None:
            raise AssertionError(f"process exited: {proc.stderr.read().decode()[-3000:]}")
        if time.time() - t0 > timeout:
            raise AssertionError(f"timed out waiting for {path}")
        time.sleep(0.1)
    time.sleep(0.05)
    return json.loads(open(path).read())


def _stop(procs):
    for p in procs:
        if p.poll() is None:
            try:
                os.killpg(p.pid, signal.SIGTERM)
            except ProcessLookupError:
                pass
    for p in procs:
        try:
            p.wait(timeout=20)
        except subprocess.TimeoutExpired:
            os.killpg(p.pid, signal.SIGKILL)
            p.wait(timeout=10)


@pytest.fixture(scope="module")
def single_process():
    from swarm_inference_lab_b200.models.config import preset
    from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
    torch.set_num_threads(2)
    dec = ReferenceDecoder(preset("tiny-llama-cpu"), random_source(0), device="cpu",
                           dtype=torch.float32)
    return dec.greedy_generate(PROMPT, NEW)


def test_cluster_create_join_and_run_distributed(tmp_path, single_process):
    toks_ref, logits_ref = single_process
    port = _free_pair()
    coord, n1, n2 = tmp_path / "coord", tmp_path / "n1", tmp_path / "n2"
    _swarm("cluster", "create", "demo", "--host", "127.0.0.1", "--port", str(port),
           "--state-dir", str(coord), "--json")
    agents = []
    try:
        _swarm("cluster", "start", "--state-dir", str(coord))
        for name, st in (("n1", n1), ("n2", n2)):
            uri = _swarm("cluster", "pair", "--state-dir", str(coord)).stdout.strip().splitlines()[-1]
            _swarm("node", "join", uri, "--name", name, "--state-dir", str(st))
        for st in (n1, n2):
            ready = tmp_path / f"{st.name}.ready"
            agents.append(_start_agent(st, ready))
            _wait_file(ready, agents[-1])
        out = _swarm("run", "tiny-llama-cpu", "--require-distributed", "--stages", "2",
                     "--prompt-ids", ",".join(map(str, PROMPT)), "--max-tokens", str(NEW),
                     "--return-logits", "--json", "--state-dir", str(coord), timeout=300)
        res = json.loads(out.stdout.strip().splitlines()[-1])
        assert res["distributed"] is True
        assert len(res["deployment"]["stages"]) == 2
        assert {s["worker_id"] for s in res["deployment"]["stages"]} == {"n1", "n2"}
        assert res["tokens"] == toks_ref
        got = torch.tensor(res["logits"], dtype=torch.float32)
        ref = torch.stack([x.float().reshape(-1) for x in logits_ref])
        assert got.shape == ref.shape
        assert (got - ref).abs().max().item() <= 1e-5
        # The coordinator saw both workers register and heartbeat.
        status = _swarm("cluster", "status", "--state-dir", str(coord), "--json").stdout
        assert json.loads(status.strip().splitlines()[-1])["members"] == 2
        # The running coordinator's own view: workers, generated tokens, finished sessions.
        st = json.loads(_swarm("status", "--state-dir", str(coord), "--json").stdout)
        assert st["healthy_workers"] == 2 and st["generated_tokens"] >= NEW
        assert st["uptime_s"] > 0 and st["recoveries"] == 0 and st["last_error"] is None
        sess = json.loads(_swarm("sessions", "--include-terminal", "--state-dir", str(coord),
                                 "--json").stdout)
        assert any(r["state"] == "COMPLETED" and r["tokens"] == NEW and
                   r["prompt_tokens"] == len(PROMPT) for r in sess.values())
        ws = json.loads(_swarm("workers", "--state-dir", str(coord), "--json").stdout)
        assert {w["worker_id"] for w in ws} == {"n1", "n2"}
        name = res["deployment"]["model"]
        _swarm("model", "unload", name, "--state-dir", str(coord))
        st = json.loads(_swarm("status", "--state-dir", str(coord), "--json").stdout)
        assert name not in st["models"]
        # with the workers free again, the coordinator places a new 2-stage plan on them
        plan = json.loads(_swarm("model", "plan", "tiny-llama-cpu", "--stages", "2",
                                 "--state-dir", str(coord)).stdout)
        assert len(plan) == 2 and {p["worker_id"] for p in plan} == {"n1", "n2"}
        # n2 leaves: the coordinator forgets it and drops its membership, its agent stops
        # and its local state is gone; the topology view no longer lists it
        r = _swarm("node", "leave", "--yes", "--state-dir", str(n2))
        assert json.loads(r.stdout.strip().splitlines()[0])["ok"]
        agents[1].wait(timeout=30)
        assert not (n2 / "cluster.json").exists()
        status = _swarm("cluster", "status", "--state-dir", str(coord), "--json").stdout
        assert json.loads(status.strip().splitlines()[-1])["members"] == 1
        topo = json.loads(_swarm("cluster", "topology", "--state-dir", str(coord)).stdout)
        assert [w["worker_id"] for w in topo["workers"]] == ["n1"] and topo["departed"] == ["n2"]
        # revoking n1 on the coordinator removes it from the running registry at once
        r = _swarm("cluster", "revoke", "n1", "--state-dir", str(coord))
        assert json.loads(r.stdout.strip().splitlines()[-1])["ok"]
        topo = json.loads(_swarm("cluster", "topology", "--state-dir", str(coord)).stdout)
        assert topo["workers"] == [] and topo["departed"] == ["n1", "n2"]
    finally:
        _stop(agents)
        _swarm("cluster", "stop", "--state-dir", str(coord), check=False)


def test_coordinator_restart_restores_the_deployment(tmp_path, single_process):
    """``cluster stop`` / ``cluster start`` with a model deployed: the restarted coordinator
    finds its deployment in the durable state, the agents re-register over mutual TLS, the
    model comes back under its name (``cluster topology --wait``) and a request through
    ``submit`` returns the single-process tokens."""
    toks_ref, _ = single_process
    port = _free_pair()
    coord, n1, n2 = tmp_path / "coord", tmp_path / "n1", tmp_path / "n2"
    _swarm("cluster", "create", "restart", "--host", "127.0.0.1", "--port", str(port),
           "--state-dir", str(coord), "--json")
    agents = []
    try:
        _swarm("cluster", "start", "--state-dir", str(coord))
        for name, st in (("n1", n1), ("n2", n2)):
            uri = _swarm("cluster", "pair", "--state-dir", str(coord)).stdout.strip().splitlines()[-1]
            _swarm("node", "join", uri, "--name", name, "--state-dir", str(st))
        for st in (n1, n2):
            ready = tmp_path / f"{st.name}.ready"
            agents.append(_start_agent(st, ready))
            _wait_file(ready, agents[-1])
        dep = json.loads(_swarm("model", "deploy", "tiny-llama-cpu", "--stages", "2", "--name", "tiny",
                                "--state-dir", str(coord)).stdout)
        assert dep["model"] == "tiny"
        _swarm("cluster", "stop", "--state-dir", str(coord))
        _swarm("cluster", "start", "--state-dir", str(coord))
        topo = json.loads(_swarm("cluster", "topology", "--wait", "60", "--model", "tiny",
                                 "--state-dir", str(coord), timeout=120).stdout)
        assert topo["models"]["tiny"]["complete"]
        rep = next(iter(topo["models"]["tiny"]["replicas"].values()))
        assert rep["generation"] > dep["generation"]
        out = _swarm("submit", "tiny", "--prompt-ids", ",".join(map(str, PROMPT)),
                     "--max-tokens", str(NEW), "--state-dir", str(coord), timeout=300).stdout
        events = [json.loads(l) for l in out.strip().splitlines()]
        assert events[-1]["event"] == "completed" and events[-1]["tokens"] == toks_ref
    finally:
        _stop(agents)
        _swarm("cluster", "stop", "--state-dir", str(coord), check=False)


def test_worker_killed_mid_decode_recovers_on_a_spare(tmp_path, single_process):
    """The coordinator runs in this process so the test can pause the stream between two
    tokens; the three nodes are separate processes."""
    from swarm_inference_lab_b200.cluster.control import (channel_credentials, coordinator_tls,
                                                          server_credentials)
    from swarm_inference_lab_b200.cluster.pairing import PairingManager
    from swarm_inference_lab_b200.cluster.state import ClusterStateStore
    from swarm_inference_lab_b200.coordinator.service import CoordinatorCore, CoordinatorRpcServer

    toks_ref, _ = single_process
    port = _free_pair()
    coord = tmp_path / "coord"
    _swarm("cluster", "create", "demo", "--host", "127.0.0.1", "--port", str(port),
           "--state-dir", str(coord), "--json")
    store = ClusterStateStore(coord)

    async def go():
        ca, crt, key = coordinator_tls(store)
        core = CoordinatorCore(store.identity("coordinator"), state_dir=coord, cluster_store=store,
                               heartbeat_timeout_s=5.0, heartbeat_s=0.5,
                               worker_credentials=channel_credentials(ca, crt, key))
        pm = PairingManager(store, f"127.0.0.1:{port}")
        await pm.start("127.0.0.1", port)
        rpc = CoordinatorRpcServer(core, host="127.0.0.1", port=port + 1,
                                   credentials=server_credentials(ca, crt, key))
        await rpc.start()
        agents = {}
        try:
            for name in ("n1", "n2", "n3"):
                st = tmp_path / name
                proc = await asyncio.create_subprocess_exec(
                    sys.executable, "-m", "swarm_inference_lab_b200.cli", "node", "join",
                    pm.invite().uri(), "--name", name, "--state-dir", str(st), env=_env(), cwd=ROOT,
                    stdout=asyncio.subprocess.DEVNULL, stderr=asyncio.subprocess.PIPE)
                _, err = await asyncio.wait_for(proc.communicate(), 120)
                assert proc.returncode == 0, err.decode()[-2000:]
                ready = tmp_path / f"{name}.ready"
                agents[name] = _start_agent(st, ready)
                t0 = time.time()
                while not ready.exists():
                    assert agents[name].poll() is None, agents[name].stderr.read().decode()[-2000:]
                    assert time.time() - t0 < 90
                    await asyncio.sleep(0.1)
            while len(core.registry.healthy()) < 3:
                await asyncio.sleep(0.1)
            dep = await core.deploy({"model": {"preset": "tiny-llama-cpu", "seed": 0}, "stages": 2})
            gen0 = dep["generation"]
            victim = dep["stages"][1]["worker_id"]
            spare = ({"n1", "n2", "n3"} - {s["worker_id"] for s in dep["stages"]}).pop()
            tokens, recovered = [], []
            async for ev in core.submit_stream({"model": dep["model"], "prompt_ids": PROMPT,
                                                "max_tokens": NEW}):
                if ev["event"] == "token":
                    tokens.append(ev["token"])
                    if len(tokens) == 10:
                        agents[victim].kill()           # SIGKILL between two decode steps
                        agents[victim].wait(timeout=20)
                elif ev["event"] == "recovered":
                    recovered.append(ev)
                elif ev["event"] == "failed":
                    raise AssertionError(ev)
            m = core.models[dep["model"]]
            st = core.status()
            assert st["recoveries"] == 1 and st["generated_tokens"] == NEW
            req = next(iter(st["requests"].values()))
            assert req["state"] == "COMPLETED" and req["generations"] == [gen0, gen0 + 1]
            return tokens, recovered, gen0, m, victim, spare
        finally:
            _stop(list(agents.values()))
            await rpc.stop()
            await pm.close()

    tokens, recovered, gen0, m, victim, spare = asyncio.run(go())
    assert tokens == toks_ref
    assert len(recovered) == 1 and recovered[0]["generation"] == gen0 + 1
    assert recovered[0]["replayed"] == 10
    assert m.deployment.generation == gen0 + 1
    assert spare in {s.worker_id for s in m.deployment.stages}
    assert victim not in {s.worker_id for s in m.deployment.stages}


def test_replica_pipelines_share_concurrent_requests(tmp_path, single_process):
    """Two replicas of a 2-stage pipeline on four nodes; four concurrent requests are
    placed by the replica scheduler on both replicas and all return the reference tokens."""
    from swarm_inference_lab_b200.cluster.control import (channel_credentials, coordinator_tls,
                                                          server_credentials)
    from swarm_inference_lab_b200.cluster.pairing import PairingManager
    from swarm_inference_lab_b200.cluster.state import ClusterStateStore
    from swarm_inference_lab_b200.coordinator.service import CoordinatorCore, CoordinatorRpcServer

    toks_ref, _ = single_process
    n_new = 16
    port = _free_pair()
    coord = tmp_path / "coord"
    _swarm("cluster", "create", "demo", "--host", "127.0.0.1", "--port", str(port),
           "--state-dir", str(coord), "--json")
    store = ClusterStateStore(coord)

    async def go():
        ca, crt, key = coordinator_tls(store)
        core = CoordinatorCore(store.identity("coordinator"), state_dir=coord, cluster_store=store,
                               worker_credentials=channel_credentials(ca, crt, key))
        pm = PairingManager(store, f"127.0.0.1:{port}")
        await pm.start("127.0.0.1", port)
        rpc = CoordinatorRpcServer(core, host="127.0.0.1", port=port + 1,
                                   credentials=server_credentials(ca, crt, key))
        await rpc.start()
        agents = []
        try:
            names = ["r1", "r2", "r3", "r4"]
            for name in names:
                st = tmp_path / name
                proc = await asyncio.create_subprocess_exec(
                    sys.executable, "-m", "swarm_inference_lab_b200.cli", "node", "join",
                    pm.invite().uri(), "--name", name, "--state-dir", str(st), env=_env(), cwd=ROOT,
                    stdout=asyncio.subprocess.DEVNULL, stderr=asyncio.subprocess.PIPE)
                _, err = await asyncio.wait_for(proc.communicate(), 120)
                assert proc.returncode == 0, err.decode()[-2000:]
                agents.append(_start_agent(st, tmp_path / f"{name}.ready"))
            t0 = time.time()
            while len(core.registry.healthy()) < 4:
                assert time.time() - t0 < 120
                await asyncio.sleep(0.1)
            dep = await core.deploy({"model": {"preset": "tiny-llama-cpu", "seed": 0}, "stages": 2,
                                     "replicas": 2})
            assert len(dep["replicas"]) == 2

            async def one(i):
                toks, rep = [], None
                async for ev in core.submit_stream({"model": dep["model"], "prompt_ids": PROMPT,
                                                    "max_tokens": n_new, "request_id": f"q{i}"}):
                    if ev["event"] == "accepted":
                        rep = ev["replica"]
                    elif ev["event"] == "token":
                        toks.append(ev["token"])
                    elif ev["event"] == "failed":
                        raise AssertionError(ev)
                return rep, toks
            return await asyncio.gather(*[one(i) for i in range(4)])
        finally:
            _stop(agents)
            await rpc.stop()
            await pm.close()

    results = asyncio.run(go())
    assert {rep for rep, _ in results} == {"replica0", "replica1"}
    for _, toks in results:
        assert toks == toks_ref[:n_new]


def test_hf_qwen3_checkpoint_four_stages_matches_hf_generate(tmp_path):
    """A Hugging Face Qwen3 checkpoint (tiny, random, fp32) served as 4 process-isolated
    pipeline stages through the public commands (``testing/real_loopback.py``: cluster
    create / start / pair, node join / agent, ``swarm run --require-distributed``): greedy
    tokens equal HF's own ``generate``, both ending at the checkpoint's EOS token."""
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from swarm_inference_lab_b200.testing.real_loopback import run

    torch.manual_seed(0)
    hf = Qwen3ForCausalLM(Qwen3Config(vocab_size=320, hidden_size=64, intermediate_size=96,
                                      num_hidden_layers=4, num_attention_heads=4,
                                      num_key_value_heads=2, head_dim=16, initializer_range=0.2,
                                      max_position_embeddings=256, tie_word_embeddings=False)).eval()
    prompt = torch.randint(0, 320, (12,), generator=torch.Generator().manual_seed(2)).tolist()
    with torch.no_grad():
        free = hf.generate(torch.tensor([prompt]), max_new_tokens=24, do_sample=False)[0, 12:].tolist()
    # the checkpoint's EOS is a token greedy decoding reaches: both sides must stop after it
    eos = free[10]
    cut = free.index(eos) + 1
    hf.generation_config.eos_token_id = eos
    ckpt = tmp_path / "qwen3-tiny"
    hf.save_pretrained(ckpt, safe_serialization=True)
    rep = run(str(ckpt), stages=4, tokens=24, prompt=prompt, workdir=str(tmp_path / "run"))
    assert rep["reference"].startswith("transformers")
    assert [s["layers"] for s in rep["stages"]] == [[0, 1], [1, 2], [2, 3], [3, 4]]
    assert len({s["worker"] for s in rep["stages"]}) == 4
    assert rep["exact"], (rep["tokens"], rep["reference_tokens"])
    assert rep["tokens"] == free[:cut] and rep["stop_reason"] == "stop_token"
    from swarm_inference_lab_b200.testing.acceptance import check_contract, load_contract
    assert check_contract(load_contract("real_loopback"), rep)["ok"]
