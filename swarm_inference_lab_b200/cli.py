"""The ``swarm`` command line.

    swarm cluster create NAME            # this machine becomes coordinator; prints a pairing URI
    swarm cluster start | stop           # the coordinator process (pairing + gRPC control plane)
    swarm cluster pair                   # mint another single-use pairing URI
    swarm cluster status | nodes | revoke NODE | delete
    swarm node join URI                  # pair this machine with a cluster
    swarm node agent                     # this node's worker runtime (registers, heartbeats)
    swarm node configure | install-service | update | status | doctor | leave
    swarm coordinator                    # the coordinator in the foreground
    swarm submit MODEL --prompt-ids ...  # a request through the running coordinator
    swarm run MODEL [--prompt TEXT | --prompt-ids 1,2,3] [--max-tokens N] [--gpus N]
              [--mode speed|throughput|capacity|balanced] [--dry-run] [--explain-plan]
              [--json | --ndjson] [--require-distributed] [--engine native-stage]
    swarm model inspect PATH             # header-only checkpoint inspection
    swarm plan MODEL --gpus 8 --batch 32 --ctx 2304
    swarm worker --stage I --stages N ...  # one stage owner (SWRING01 server)
    swarm probe nvlink                   # measure the intra-box links
    swarm identity show

MODEL is a preset name (``llama-3-8b-shape``, ``qwen3-30b-a3b-shape``, ...), a
local checkpoint directory, a ``.gguf`` file or ``hf://org/name@revision``.
A safetensors checkpoint directory is served with its own weights and, when it
carries one, its tokenizer (``--prompt`` text is tokenized and the output detokenized);
without a tokenizer ``--prompt`` text is mapped to ids byte-wise (deterministic;
documented as such in the output).  ``--require-distributed`` serves through the
cluster's coordinator across the joined nodes instead of this box's GPUs.

Reference: si/cli.py:129-2372 and si/commands/{run,cluster,node}.py.
"""
from __future__ import annotations

import asyncio
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import typer

app = typer.Typer(add_completion=False, help="Blackwell-native distributed inference runtime")
cluster_app = typer.Typer(help="cluster lifecycle")
node_app = typer.Typer(help="this node")
model_app = typer.Typer(help="model inspection and deployment")
identity_app = typer.Typer(help="node identity")
probe_app = typer.Typer(help="measurements")
experiment_app = typer.Typer(help="research harnesses on the real control plane (CPU)")
app.add_typer(cluster_app, name="cluster")
app.add_typer(node_app, name="node")
app.add_typer(model_app, name="model")
app.add_typer(experiment_app, name="experiment")
app.add_typer(identity_app, name="identity")
app.add_typer(probe_app, name="probe")

STATE = os.environ.get("SWARM_STATE_DIR", "~/.swarm-b200")
EXIT_USAGE, EXIT_STATE, EXIT_RUNTIME = 2, 3, 4


def _store(state: str):
    from .cluster.state import ClusterStateStore
    return ClusterStateStore(Path(state))


def _out(obj, as_json: bool):
    if as_json:
        typer.echo(json.dumps(obj, default=str))
    else:
        for k, v in obj.items():
            typer.echo(f"{k}: {v}")


def _resolve_model(model: str):
    from .models.config import PRESETS
    if model in PRESETS:
        return PRESETS[model], None
    from .model_io.resolver import ModelSourceResolver
    res = ModelSourceResolver().inspect(model)
    if res.profile.config is None:
        raise typer.BadParameter(f"{model}: no runnable configuration ({res.profile.notes})")
    return res.profile.config, res


def _gpu_caps(gpus: int | None):
    from .engines import ClusterCapabilities
    from .planner.box_planner import BoxMeasurements
    n = gpus
    name = "NVIDIA B200"
    try:
        import torch
        if torch.cuda.is_available():
            n = n or torch.cuda.device_count()
            name = torch.cuda.get_device_name(0)
    except Exception:  # noqa: BLE001
        pass
    root = Path(__file__).resolve().parent.parent
    m = BoxMeasurements.from_files(str(root / "MEASURED_PEAKS.json"),
                                   os.environ.get("SWARM_NVLINK_PROBE"))
    return ClusterCapabilities(nodes={"local": {"gpus": n or 1, "gpu_name": name}}, measurements=m)


def _prompt_ids(prompt: str | None, prompt_ids: str | None, vocab: int,
                tokenizer=None) -> tuple[list[int], str]:
    if prompt_ids:
        return [int(x) for x in prompt_ids.split(",") if x.strip()], "ids"
    text = prompt or "Hello"
    if tokenizer is not None:
        return list(tokenizer.encode(text)), "tokenizer"
    return [b % vocab for b in text.encode("utf-8")], "bytes"


# ------------------------------------------------------------------ run
@app.command("run")
def run_command(model: str, prompt: str = typer.Option(None, "--prompt"),
                prompt_ids: str = typer.Option(None, "--prompt-ids"),
                max_tokens: int = typer.Option(32, "--max-tokens"),
                gpus: int = typer.Option(None, "--gpus"),
                mode: str = typer.Option("balanced", "--mode"),
                engine: str = typer.Option("native-stage", "--engine"),
                dry_run: bool = typer.Option(False, "--dry-run"),
                explain_plan: bool = typer.Option(False, "--explain-plan"),
                require_distributed: bool = typer.Option(False, "--require-distributed"),
                as_json: bool = typer.Option(False, "--json"),
                ndjson: bool = typer.Option(False, "--ndjson"),
                seed: int = typer.Option(0, "--seed"),
                temperature: float = typer.Option(0.0, "--temperature"),
                top_k: int = typer.Option(0, "--top-k"),
                top_p: float = typer.Option(1.0, "--top-p"),
                repetition_penalty: float = typer.Option(1.0, "--repetition-penalty"),
                stages: int = typer.Option(None, "--stages"),
                replicas: int = typer.Option(1, "--replicas"),
                return_logits: bool = typer.Option(False, "--return-logits"),
                ignore_eos: bool = typer.Option(False, "--ignore-eos",
                                                help="generate MAX_TOKENS even past the model's EOS"),
                state: str = typer.Option(STATE, "--state-dir")):
    """Resolve, plan and run MODEL (on this box, or across the cluster), streaming tokens;
    generation ends after MAX_TOKENS or after the checkpoint's EOS token (which is emitted)."""
    from .engines import EngineRegistry, RequestShape
    if mode not in ("speed", "throughput", "capacity", "balanced"):
        raise typer.BadParameter("mode must be speed|throughput|capacity|balanced")
    cfg, res = _resolve_model(model)
    ckpt = _checkpoint_dir(model, res)
    tokenizer = None
    if ckpt is not None:
        from .model_io.loader import load_tokenizer
        tokenizer = load_tokenizer(ckpt)
    ids, tok_kind = _prompt_ids(prompt, prompt_ids, cfg.vocab_size, tokenizer)
    if require_distributed:
        _run_distributed(model, cfg, ckpt, ids, tok_kind, max_tokens, stages, seed, tokenizer,
                         as_json, ndjson, return_logits, state, replicas, ignore_eos)
        return
    caps = _gpu_caps(gpus)
    comp = EngineRegistry().compete(cfg, caps, RequestShape(
        batch=1, prompt_tokens=len(ids), output_tokens=max_tokens, mode=mode,
        require_distributed=require_distributed))
    plan = comp.winner
    if plan is None or plan.engine != engine:
        _out({"error": "no admissible plan", "rejected": comp.rejected}, as_json or ndjson)
        raise typer.Exit(EXIT_RUNTIME)
    explanation = {"model": cfg.name, "revision": res.revision if res else "preset",
                   "plan": plan.description, "predicted_tok_s": round(plan.predicted_tok_s, 1),
                   "predicted_ttft_ms": round(plan.predicted_ttft_ms, 2),
                   "mechanisms": plan.mechanisms, "confidence": plan.confidence,
                   "terms": plan.explain, "alternatives": [p.description for p in comp.ranked[1:4]],
                   "rejected": comp.rejected, "prompt_tokenization": tok_kind,
                   "weights": "checkpoint" if ckpt is not None else f"random (seed {seed})"}
    if explain_plan or dry_run:
        _out(explanation, as_json or ndjson)
        if dry_run:
            return
    if plan.parallelism.get("tp", 1) * plan.parallelism.get("pp", 1) > 1:
        typer.echo("multi-GPU plans run under torchrun (see bench.py); serving this request on one GPU",
                   err=True)
    from .engine.engine import LLMEngine, SamplingParams
    t0 = time.perf_counter()
    weights = None
    if ckpt is not None:
        from .model_io.loader import load_weights
        weights = load_weights(cfg, ckpt, device="cuda")
    eng = LLMEngine(cfg, device="cuda", seed=seed, max_batch=1,
                    max_seq_len=len(ids) + max_tokens + 64, weights=weights)
    params = SamplingParams(max_new_tokens=max_tokens, temperature=temperature, top_k=top_k,
                            top_p=top_p, repetition_penalty=repetition_penalty, seed=seed,
                            stop_token_ids=() if ignore_eos else tuple(cfg.eos_token_ids))
    eng.add_request(ids, params, request_id="cli")
    out = []
    while eng.scheduler.has_work():
        for rid, tok in eng.step():
            out.append(tok)
            if ndjson:
                typer.echo(json.dumps({"event": "TOKEN_GENERATED", "token": tok, "index": len(out) - 1}))
    dt = time.perf_counter() - t0
    result = {"tokens": out, "output_tokens": len(out), "seconds": round(dt, 3),
              "prompt_tokens": len(ids), "prompt_tokenization": tok_kind}
    if tokenizer is not None:
        result["text"] = tokenizer.decode(out)
    if ndjson:
        typer.echo(json.dumps({"event": "REQUEST_COMPLETED", **result}))
    else:
        _out(result, as_json)


def _checkpoint_dir(model: str, res) -> str | None:
    """The local safetensors directory behind MODEL, when it is one."""
    if res is None:
        return None
    p = Path(model).expanduser()
    if p.is_dir() and any(p.glob("*.safetensors")) and (p / "config.json").is_file():
        return str(p)
    src = getattr(res, "local_path", None)
    if src and Path(src).is_dir() and any(Path(src).glob("*.safetensors")):
        return str(src)
    return None


def _model_desc(model: str, cfg, ckpt: str | None, seed: int) -> dict:
    if ckpt is not None:
        return {"checkpoint": str(Path(ckpt).resolve())}
    return {"preset": cfg.name, "seed": seed}


def _run_distributed(model, cfg, ckpt, ids, tok_kind, max_tokens, stages, seed, tokenizer,
                     as_json, ndjson, return_logits, state, replicas=1, ignore_eos=False):
    """Deploy MODEL across the cluster's joined nodes through the coordinator and stream
    the request's tokens (the coordinator replays the request on a replacement node if a
    node fails mid-request)."""
    from .cluster.control import coordinator_client
    st = _store(state)
    if not st.has_cluster():
        typer.echo("--require-distributed needs a cluster: `swarm cluster create` + `swarm node join`",
                   err=True)
        raise typer.Exit(EXIT_STATE)

    async def go():
        cli = coordinator_client(st)
        try:
            desc = _model_desc(model, cfg, ckpt, seed)
            dep = await cli.deploy(desc, stages=stages, replicas=replicas)
            name = dep["model"]
            events, tokens, logits = [], [], []
            async for ev in cli.submit_stream(name, ids, max_tokens, return_logits=return_logits,
                                              ignore_eos=ignore_eos):
                events.append(ev)
                if ev["event"] == "token":
                    tokens.append(ev["token"])
                    if return_logits:
                        logits.append(ev.get("logits"))
                if ndjson:
                    typer.echo(json.dumps(ev if not return_logits else
                                          {k: v for k, v in ev.items() if k != "logits"}))
            return dep, events, tokens, logits
        finally:
            await cli.close()
    dep, events, tokens, logits = asyncio.run(go())
    last = events[-1] if events else {"event": "failed", "error": "no events"}
    if last["event"] != "completed":
        _out({"error": last.get("error", "request failed")}, as_json or ndjson)
        raise typer.Exit(EXIT_RUNTIME)
    result = {"tokens": tokens, "output_tokens": len(tokens), "deployment": dep,
              "generations": last.get("generations"), "prompt_tokenization": tok_kind,
              "stop_reason": last.get("stop_reason"), "distributed": True}
    if return_logits:
        result["logits"] = logits
    if tokenizer is not None:
        result["text"] = tokenizer.decode(tokens)
    if ndjson:
        typer.echo(json.dumps({"event": "REQUEST_COMPLETED",
                               **{k: v for k, v in result.items() if k != "logits"}}))
    else:
        _out(result, as_json)


# ------------------------------------------------------------------ cluster
@cluster_app.command("create")
def cluster_create(name: str, host: str = "127.0.0.1", port: int = 7651,
                   state: str = typer.Option(STATE, "--state-dir"), as_json: bool = typer.Option(False, "--json")):
    """Bootstrap a cluster: identity, CA, state; print a single-use pairing URI."""
    from .cluster.pairing import PairingManager
    from .cluster.state import StateError
    from .security.tls import create_ca
    st = _store(state)
    ca = create_ca(name)
    try:
        st.create_cluster(name, f"{host}:{port}", ca.cert, ca.key)
    except StateError as exc:
        typer.echo(str(exc), err=True)
        raise typer.Exit(EXIT_STATE)
    inv = PairingManager(st, f"{host}:{port}").invite()
    _out({"cluster": name, "coordinator": f"{host}:{port}",
          "coordinator_fingerprint": st.identity().fingerprint, "pairing_uri": inv.uri()}, as_json)


@cluster_app.command("status")
def cluster_status(state: str = typer.Option(STATE, "--state-dir"), as_json: bool = typer.Option(False, "--json")):
    """This node's view of the cluster record: name, role, coordinator endpoint, member and
    revoked counts."""
    st = _store(state)
    doc = st.load_cluster()
    _out({"cluster": doc["name"], "role": doc["role"], "coordinator": doc["coordinator_endpoint"],
          "members": len(doc["members"]), "revoked": len(doc["revoked"])}, as_json)


@cluster_app.command("nodes")
def cluster_nodes(state: str = typer.Option(STATE, "--state-dir")):
    """Members of the cluster (name, fingerprint, endpoints, capabilities)."""
    doc = _store(state).load_cluster()
    typer.echo(json.dumps(doc["members"], indent=1, default=str))


@cluster_app.command("revoke")
def cluster_revoke(node: str, state: str = typer.Option(STATE, "--state-dir")):
    """Revoke NODE: its fingerprint is refused by the coordinator from now on; when the
    coordinator is running, NODE's stages move to spares at once (running requests resume
    on the new route by replay)."""
    st = _store(state)
    fp = st.revoke(node)
    typer.echo(f"revoked {node} ({fp})")
    if "coordinator" in st.runtime():
        rep = _with_coordinator(state, lambda c: c.remove_worker(node))
        typer.echo(json.dumps(rep))


@cluster_app.command("topology")
def cluster_topology(state: str = typer.Option(STATE, "--state-dir"),
                     wait: float = typer.Option(0.0, "--wait",
                                                help="seconds to wait for complete coverage"),
                     model: str = typer.Option(None, "--model",
                                               help="with --wait: a model that must be deployed")):
    """The running coordinator's view: workers (health, draining, reachability, link class)
    and, per deployed model and replica, which worker covers which layers and whether
    coverage is complete; exits 1 when a deployed model has a gap or a stage on a dead or
    unreachable worker.  --wait polls until coverage is complete (and --model is deployed)."""
    def complete(rep):
        return (all(m["complete"] for m in rep["models"].values())
                and (model is None or model in rep["models"]))

    async def poll(c):
        t0 = time.time()
        while True:
            rep = await c.topology()
            if complete(rep) or time.time() - t0 >= wait:
                return rep
            await asyncio.sleep(0.25)
    rep = _with_coordinator(state, poll)
    typer.echo(json.dumps(rep, indent=1))
    if not complete(rep):
        raise typer.Exit(1)


@cluster_app.command("delete")
def cluster_delete(state: str = typer.Option(STATE, "--state-dir"), yes: bool = typer.Option(False, "--yes")):
    """Delete this node's cluster state (needs --yes)."""
    if not yes:
        typer.echo("refusing to delete cluster state without --yes", err=True)
        raise typer.Exit(EXIT_USAGE)
    _store(state).delete()
    typer.echo("deleted")


@cluster_app.command("pair")
def cluster_pair(serve: bool = typer.Option(False, "--serve"), ttl: float = 600.0,
                 state: str = typer.Option(STATE, "--state-dir")):
    """Mint a pairing URI (from the running coordinator when ``cluster start`` runs; with
    --serve, answer pairing requests here until interrupted)."""
    from .cluster.pairing import PairingManager
    st = _store(state)
    doc = st.load_cluster()
    if not serve and st.runtime().get("coordinator"):
        from .cluster.control import coordinator_client

        async def mint():
            cli = coordinator_client(st, timeout=30.0)
            try:
                return await cli.pairing_uri(ttl)
            finally:
                await cli.close()
        typer.echo(asyncio.run(mint()))
        return
    pm = PairingManager(st, doc["coordinator_endpoint"])
    inv = pm.invite(ttl)
    typer.echo(inv.uri())
    if serve:
        host, port = doc["coordinator_endpoint"].rsplit(":", 1)

        async def go():
            await pm.start(host, int(port))
            while True:
                await asyncio.sleep(3600)
        asyncio.run(go())


@cluster_app.command("start")
def cluster_start(state: str = typer.Option(STATE, "--state-dir"),
                  foreground: bool = typer.Option(False, "--foreground"),
                  wait_s: float = typer.Option(60.0, "--wait")):
    """Start the coordinator process (pairing server + gRPC control plane)."""
    st = _store(state)
    doc = st.load_cluster()
    if doc["role"] != "coordinator":
        typer.echo("only the coordinator node starts the cluster", err=True)
        raise typer.Exit(EXIT_STATE)
    if foreground:
        from .cluster.control import serve_coordinator
        asyncio.run(serve_coordinator(st))
        return
    import subprocess
    import tempfile
    ready = Path(tempfile.mkdtemp()) / "ready.json"
    log = open(st.root / "coordinator.log", "ab")
    proc = subprocess.Popen([sys.executable, "-m", "swarm_inference_lab_b200.cli", "coordinator",
                             "--state-dir", str(st.root), "--ready-file", str(ready)],
                            stdout=log, stderr=subprocess.STDOUT, start_new_session=True)
    t0 = time.time()
    while not ready.exists():
        if proc.poll() is not None or time.time() - t0 > wait_s:
            typer.echo(f"coordinator did not start (see {st.root / 'coordinator.log'})", err=True)
            raise typer.Exit(EXIT_RUNTIME)
        time.sleep(0.1)
    info = json.loads(ready.read_text())
    typer.echo(json.dumps({"started": True, **info}))


@cluster_app.command("stop")
def cluster_stop(state: str = typer.Option(STATE, "--state-dir"), wait_s: float = 45.0):
    """Stop the coordinator process started by ``cluster start``: it admits no new request
    and lets the running ones finish (up to 30 s) before it exits."""
    import signal as _signal
    st = _store(state)
    rec = st.runtime().get("coordinator")
    if not rec:
        typer.echo("no running coordinator recorded", err=True)
        raise typer.Exit(EXIT_STATE)
    pid = int(rec["pid"])
    try:
        os.kill(pid, _signal.SIGTERM)
    except ProcessLookupError:
        pass
    t0 = time.time()
    while time.time() - t0 < wait_s:
        try:
            os.kill(pid, 0)
        except ProcessLookupError:
            break
        time.sleep(0.1)
    typer.echo(json.dumps({"stopped": True, "pid": pid}))


@app.command("coordinator")
def coordinator_command(state: str = typer.Option(STATE, "--state-dir"),
                        ready_file: str = typer.Option(None, "--ready-file"),
                        heartbeat_timeout: float = typer.Option(5.0, "--heartbeat-timeout")):
    """Run the cluster's coordinator in the foreground."""
    from .cluster.control import serve_coordinator
    asyncio.run(serve_coordinator(_store(state), ready_file=ready_file,
                                  heartbeat_timeout_s=heartbeat_timeout))


@app.command("submit")
def submit_command(model: str, prompt_ids: str = typer.Option(None, "--prompt-ids"),
                   prompt: str = typer.Option(None, "--prompt",
                                              help="text, tokenized by the coordinator with the "
                                                   "deployed checkpoint's tokenizer"),
                   max_tokens: int = typer.Option(16, "--max-tokens"),
                   state: str = typer.Option(STATE, "--state-dir"),
                   return_logits: bool = typer.Option(False, "--return-logits"),
                   speculate: int = typer.Option(0, "--speculate",
                                                 help="exact prompt-lookup speculation, up to K draft tokens"),
                   stop: str = typer.Option("", "--stop", help="extra stop token ids, comma separated"),
                   ignore_eos: bool = typer.Option(False, "--ignore-eos")):
    """Stream one request of an already deployed MODEL through the coordinator (NDJSON); it
    ends after MAX_TOKENS, the model's EOS token or a --stop token (each emitted)."""
    from .cluster.control import coordinator_client
    if (prompt_ids is None) == (prompt is None):
        raise typer.BadParameter("give exactly one of --prompt-ids and --prompt")
    ids = None if prompt_ids is None else [int(x) for x in prompt_ids.split(",") if x.strip()]

    async def go():
        cli = coordinator_client(_store(state))
        try:
            async for ev in cli.submit_stream(model, ids, max_tokens, return_logits=return_logits,
                                              prompt=prompt,
                                              speculate_k=speculate, ignore_eos=ignore_eos,
                                              stop_token_ids=[int(x) for x in stop.split(",")
                                                              if x.strip()]):
                typer.echo(json.dumps(ev))
        finally:
            await cli.close()
    asyncio.run(go())


@app.command("metrics")
def metrics_command(state: str = typer.Option(STATE, "--state-dir"),
                    workers: bool = typer.Option(False, "--workers",
                                                 help="add every worker's stage view and metrics"),
                    prometheus: bool = typer.Option(False, "--prometheus")):
    """The running coordinator's counters, gauges and latency summaries (registrations,
    heartbeats, requests, tokens, TTFT / TPOT, recoveries, transport errors), as JSON or
    Prometheus text; --workers adds each worker's stage (frames, rejections, forward time)
    and metrics."""
    rep = _with_coordinator(state, lambda c: c.metrics(workers=workers))
    if prometheus:
        typer.echo(rep["prometheus"])
    else:
        typer.echo(json.dumps({k: v for k, v in rep.items() if k != "prometheus"}, indent=1,
                              default=str))


@app.command("status")
def status_command(state: str = typer.Option(STATE, "--state-dir"),
                   json_output: bool = typer.Option(False, "--json")):
    """Coordinator identity, uptime, workers, active requests, tokens, throughput,
    recoveries and the last error, from the running coordinator."""
    from .cluster.control import coordinator_client

    async def go():
        cli = coordinator_client(_store(state))
        try:
            return await cli.status()
        finally:
            await cli.close()
    st = asyncio.run(go())
    if json_output:
        typer.echo(json.dumps(st, indent=1, default=str))
        return
    typer.echo(f"coordinator={st['coordinator_fingerprint'][:16]} uptime_s={st['uptime_s']:.1f}")
    typer.echo(f"workers={st['healthy_workers']}/{st['workers']} models={','.join(st['models']) or '-'} "
               f"active_requests={st['active_requests']}")
    typer.echo(f"tokens={st['generated_tokens']} throughput_tokens_s={st['throughput_tokens_s']:.3f} "
               f"recoveries={st['recoveries']}")
    for name, m in st["models"].items():
        typer.echo(f"model {name}: {json.dumps(m, default=str)}")
    if st.get("last_error"):
        typer.echo(f"last_error={st['last_error']}")


@app.command("sessions")
def sessions_command(state: str = typer.Option(STATE, "--state-dir"),
                     include_terminal: bool = typer.Option(False, "--include-terminal"),
                     json_output: bool = typer.Option(False, "--json")):
    """Requests known to the running coordinator: state, model, prompt and generated tokens,
    route generations (more than one: recovered), and errors."""
    from .cluster.control import coordinator_client

    async def go():
        cli = coordinator_client(_store(state))
        try:
            return await cli.status()
        finally:
            await cli.close()
    reqs = asyncio.run(go())["requests"]
    rows = {k: v for k, v in reqs.items() if include_terminal or v["state"] == "RUNNING"}
    if json_output:
        typer.echo(json.dumps(rows, indent=1, default=str))
        return
    for rid, r in rows.items():
        typer.echo(f"{rid} state={r['state']} model={r['model']} prompt={r['prompt_tokens']} "
                   f"tokens={r['tokens']} generations={r['generations']}"
                   + (f" error={r['error']}" if r.get("error") else ""))


def _with_coordinator(state: str, fn):
    """Runs ``fn(client)`` against the cluster's running coordinator."""
    from .cluster.control import coordinator_client

    async def go():
        cli = coordinator_client(_store(state))
        try:
            return await fn(cli)
        finally:
            await cli.close()
    return asyncio.run(go())


@app.command("cancel")
def cancel_command(request_id: str, state: str = typer.Option(STATE, "--state-dir")):
    """Cancel a running request: its stream ends with a ``cancelled`` event before the next
    token and every stage drops the session and its KV cache."""
    rep = _with_coordinator(state, lambda c: c.cancel(request_id))
    typer.echo(json.dumps(rep))
    if not rep.get("ok"):
        raise typer.Exit(1)


@app.command("workers")
def workers_command(state: str = typer.Option(STATE, "--state-dir"),
                    json_output: bool = typer.Option(False, "--json")):
    """Workers registered with the running coordinator and their last heartbeat."""
    ws = _with_coordinator(state, lambda c: c.workers())
    if json_output:
        typer.echo(json.dumps(ws, indent=1, default=str))
        return
    for w in ws:
        typer.echo(" ".join(f"{k}={v}" for k, v in w.items() if not isinstance(v, (dict, list))))


# ------------------------------------------------------------------ node
@node_app.command("agent")
def node_agent(state: str = typer.Option(STATE, "--state-dir"), host: str = typer.Option(None, "--host"),
               device: str = typer.Option(None, "--device"),
               ready_file: str = typer.Option(None, "--ready-file")):
    """Run this node's worker runtime: register with the coordinator, heartbeat, and host
    the stage the coordinator assigns."""
    from .cluster.control import run_node_agent
    asyncio.run(run_node_agent(_store(state), host=host, device=device, ready_file=ready_file))


@node_app.command("configure")
def node_configure(state: str = typer.Option(STATE, "--state-dir"),
                   host: str = typer.Option(None, "--host"), device: str = typer.Option(None, "--device"),
                   ring_port: int = typer.Option(None, "--ring-port"),
                   control_port: int = typer.Option(None, "--control-port"),
                   heartbeat_s: float = typer.Option(None, "--heartbeat")):
    """Persist this node's agent settings (host, device, ports, heartbeat period)."""
    st = _store(state)
    rt = st.runtime()
    conf = rt.setdefault("node_config", {})
    for k, v in (("host", host), ("device", device), ("ring_port", ring_port),
                 ("control_port", control_port), ("heartbeat_s", heartbeat_s)):
        if v is not None:
            conf[k] = v
    st.save_runtime(rt)
    typer.echo(json.dumps(conf))


@node_app.command("install-service")
def node_install_service(state: str = typer.Option(STATE, "--state-dir"),
                         path: str = typer.Option(None, "--path")):
    """Write (or print) a systemd unit that keeps ``swarm node agent`` running."""
    from .cluster.control import service_unit
    unit = service_unit(_store(state), sys.executable)
    if path:
        Path(path).write_text(unit)
        typer.echo(f"wrote {path}")
    else:
        typer.echo(unit)


@node_app.command("uninstall-service")
def node_uninstall_service(path: str = typer.Option(..., "--path"),
                           yes: bool = typer.Option(False, "--yes")):
    """Remove a unit file written by ``install-service --path`` (needs --yes).  Stopping and
    disabling the running service is left to the service manager (``systemctl``)."""
    p = Path(path).expanduser()
    if not p.is_file():
        typer.echo(f"no unit file at {p}", err=True)
        raise typer.Exit(EXIT_USAGE)
    if "swarm_inference_lab_b200" not in p.read_text() or "node" not in p.read_text():
        typer.echo(f"{p} is not a unit written by install-service; left in place", err=True)
        raise typer.Exit(EXIT_USAGE)
    if not yes:
        typer.echo("refusing to remove the unit file without --yes", err=True)
        raise typer.Exit(EXIT_USAGE)
    p.unlink()
    typer.echo(f"removed {p}")


@node_app.command("update")
def node_update(state: str = typer.Option(STATE, "--state-dir"),
                as_json: bool = typer.Option(True, "--json/--text")):
    """Report this node's runtime version and native-library build against the source."""
    import hashlib
    root = Path(__file__).resolve().parent
    so = sorted(root.glob("_C*.so"))
    src = sorted((root.parent / "csrc").rglob("*.c*")) if (root.parent / "csrc").is_dir() else []
    digest = hashlib.sha256(b"".join(p.read_bytes() for p in src)).hexdigest()[:16] if src else None
    stale = bool(so and src and max(p.stat().st_mtime for p in src) > so[0].stat().st_mtime)
    _out({"version": "0.1.0", "native_library": so[0].name if so else None,
          "source_digest": digest, "rebuild_needed": stale or not so,
          "update": "run `python setup.py build_ext --inplace` to rebuild" if (stale or not so)
          else "up to date"}, as_json)


@node_app.command("join")
def node_join(uri: str, node_id: str = typer.Option(None, "--name"),
              state: str = typer.Option(STATE, "--state-dir")):
    """Join a cluster with a pairing URI from `swarm cluster pair`: this node's identity is
    enrolled and it receives its TLS certificate."""
    from .cluster.pairing import join
    from .worker_caps import local_capabilities
    caps = local_capabilities(benchmark=False)
    rep = asyncio.run(join(uri, _store(state), node_id or os.uname().nodename, capabilities=caps))
    typer.echo(f"joined cluster {rep['cluster']} (coordinator {rep['coordinator_endpoint']})")


@node_app.command("status")
def node_status(state: str = typer.Option(STATE, "--state-dir"), as_json: bool = typer.Option(False, "--json")):
    """This node's identity, state directory and cluster membership."""
    st = _store(state)
    info = {"identity": st.identity().fingerprint, "state_dir": str(st.root)}
    if st.has_cluster():
        doc = st.load_cluster()
        info.update(cluster=doc["name"], role=doc["role"], coordinator=doc["coordinator_endpoint"])
    _out(info, as_json)


@node_app.command("doctor")
def node_doctor(as_json: bool = typer.Option(False, "--json")):
    """Check this host: torch and CUDA, GPU model and compute capability (sm_100a), driver
    and memory (nvidia-smi, read-only), and the built kernel and native libraries."""
    from .doctor import run_doctor
    rep = run_doctor()
    _out(rep, as_json)
    if not rep.get("ok"):
        raise typer.Exit(EXIT_RUNTIME)


@node_app.command("leave")
def node_leave(state: str = typer.Option(STATE, "--state-dir"), yes: bool = typer.Option(False, "--yes"),
               force: bool = typer.Option(False, "--force"),
               offline: bool = typer.Option(False, "--offline")):
    """Leave the cluster (needs --yes): the coordinator moves this node's stages to spares
    and forgets it (refused while a replica it serves has a running request, unless
    --force), this node's agent is stopped, and the local cluster state is removed.
    --offline skips the coordinator (it then finds the node silent and stops using it)."""
    if not yes:
        typer.echo("refusing to leave without --yes", err=True)
        raise typer.Exit(EXIT_USAGE)
    st = _store(state)
    if st.has_cluster() and not offline:
        doc = st.load_cluster()
        if doc.get("role") == "coordinator":
            typer.echo("the coordinator node deletes the cluster instead (cluster delete)", err=True)
            raise typer.Exit(EXIT_USAGE)
        node_id = doc.get("node_id") or st.identity().name
        fp = st.identity(node_id).fingerprint
        try:
            rep = _with_coordinator(state, lambda c: c.leave(node_id, fp, force=force))
        except Exception as exc:  # noqa: BLE001 - reported; --offline leaves anyway
            typer.echo(f"coordinator unreachable ({type(exc).__name__}: {exc}); "
                       "use --offline to leave without it", err=True)
            raise typer.Exit(EXIT_RUNTIME)
        if not rep.get("ok"):
            typer.echo(json.dumps(rep), err=True)
            raise typer.Exit(EXIT_STATE)
        typer.echo(json.dumps(rep))
    from .cluster.control import stop_local_agent
    stop_local_agent(st)
    st.delete()
    typer.echo("left the cluster; local state removed")


# ------------------------------------------------------------------ model / plan
@model_app.command("deploy")
def model_deploy(model: str, stages: int = typer.Option(None, "--stages"),
                 replicas: int = typer.Option(1, "--replicas"), seed: int = typer.Option(0, "--seed"),
                 name: str = typer.Option(None, "--name"),
                 state: str = typer.Option(STATE, "--state-dir")):
    """Deploy MODEL (a preset or a local checkpoint) across the cluster's nodes through the
    running coordinator: placement, stage loads, signed routes; prints the deployment."""
    cfg, res = _resolve_model(model)
    desc = _model_desc(model, cfg, _checkpoint_dir(model, res), seed)
    dep = _with_coordinator(state, lambda c: c.deploy(desc, name=name, stages=stages,
                                                      replicas=replicas))
    typer.echo(json.dumps(dep, indent=1, default=str))


@model_app.command("scale")
def model_scale(name: str, replicas: int = typer.Option(..., "--replicas"),
                state: str = typer.Option(STATE, "--state-dir")):
    """Set deployed model NAME's replica count: new pipelines go onto free healthy workers and
    join the scheduler when READY; shrinking unloads idle replicas only (exit 1 when the
    change cannot be made; nothing changes then)."""
    rep = _with_coordinator(state, lambda c: c.scale(name, replicas))
    typer.echo(json.dumps(rep))
    if not rep.get("ok"):
        raise typer.Exit(1)


@model_app.command("unload")
def model_unload(name: str, state: str = typer.Option(STATE, "--state-dir")):
    """Unload a deployed model: routes withdrawn, stages released on every node."""
    typer.echo(json.dumps(_with_coordinator(state, lambda c: c.unload(name)), default=str))


@model_app.command("plan")
def model_plan(model: str, stages: int = typer.Option(None, "--stages"),
               seed: int = typer.Option(0, "--seed"), state: str = typer.Option(STATE, "--state-dir")):
    """The running coordinator's placement of MODEL on the cluster's healthy nodes (nothing
    is deployed)."""
    cfg, res = _resolve_model(model)
    desc = _model_desc(model, cfg, _checkpoint_dir(model, res), seed)
    typer.echo(json.dumps(_with_coordinator(state, lambda c: c.plan(desc, stages)), indent=1,
                          default=str))


def _layer_bytes(res) -> list[float]:
    """Bytes of every decoder layer's tensors (from the checkpoint headers)."""
    n = res.profile.config.num_layers
    out = [0.0] * n
    for name, d in res.profile.tensors.items():
        if d.layer is not None and 0 <= d.layer < n:
            out[d.layer] += float(res.tensor_bytes.get(name, 0))
    return out


@model_app.command("validate")
def model_validate(checkpoint: str, as_json: bool = typer.Option(True, "--json/--text")):
    """Check a local safetensors checkpoint against its config without reading tensor data:
    every tensor the model needs is present with the shape the config implies; lists the
    problems and the tensors no layer uses.  Exit 1 when a problem is found."""
    from .model_io.loader import validate_checkpoint
    rep = validate_checkpoint(checkpoint)
    _out(rep, as_json)
    if not rep["ok"]:
        raise typer.Exit(1)


@model_app.command("build-microshards")
def model_build_microshards(checkpoint: str, out: str = typer.Option(..., "--out"),
                           layers: str = typer.Option(..., "--layers"),
                           experts: str = typer.Option(None, "--experts"),
                           parts: int = typer.Option(2, "--parts")):
    """Split routed experts of a local MoE checkpoint into PARTS microshards each (contiguous
    intermediate slices: gate / up rows, down columns), one file and manifest per shard."""
    from .runtime.microshards import build_microshards
    mans = build_microshards(checkpoint, out, layers=[int(x) for x in layers.split(",")],
                             experts=[int(x) for x in experts.split(",")] if experts else None,
                             parts=parts)
    typer.echo(json.dumps({"microshards": len(mans), "out": out}))


@model_app.command("validate-microshards")
def model_validate_microshards(directory: str, checkpoint: str,
                               as_json: bool = typer.Option(True, "--json/--text")):
    """Check microshards against their manifests (SHA-256), that each expert's slices tile its
    intermediate dimension, and that their fixed-order reduction reproduces the whole expert
    from CHECKPOINT (fp32, random inputs).  Exit 1 on a problem."""
    from .runtime.microshards import validate_microshards
    rep = validate_microshards(directory, checkpoint)
    _out(rep, as_json)
    if not rep["ok"]:
        raise typer.Exit(1)


@model_app.command("partition")
def model_partition(checkpoint: str, stages: int = typer.Option(..., "--stages"),
                    as_json: bool = typer.Option(True, "--json/--text")):
    """Contiguous layer intervals for STAGES pipeline stages of a local checkpoint, balanced
    by the layers' weight bytes (the largest stage is as small as possible); the embedding
    goes with stage 0 and the final norm / LM head with the last stage."""
    from .model_io.partition import balanced_ranges
    from .model_io.resolver import ModelSourceResolver
    res = ModelSourceResolver().inspect(checkpoint)
    if res.profile.config is None:
        raise typer.BadParameter(f"{checkpoint}: no runnable configuration")
    costs = _layer_bytes(res)
    ranges = balanced_ranges([c or 1.0 for c in costs], stages)
    _out({"layers": len(costs), "stages": [
        {"stage": i, "layers": [a, b], "bytes": sum(costs[a:b]), "embed": i == 0,
         "head": i == len(ranges) - 1} for i, (a, b) in enumerate(ranges)]}, as_json)


@model_app.command("shard")
def model_shard(checkpoint: str, stages: int = typer.Option(..., "--stages"),
                out: str = typer.Option(..., "--out")):
    """Write one content-addressed stage artifact per pipeline stage of a local checkpoint
    (safetensors with exactly that stage's tensors, and a manifest with the source revision,
    layer interval, tensor list and SHA-256), layer intervals balanced by weight bytes."""
    from .cluster.artifacts import build_stage_artifact
    from .model_io.partition import balanced_ranges
    from .model_io.resolver import ModelSourceResolver
    res = ModelSourceResolver().inspect(checkpoint)
    if res.profile.config is None:
        raise typer.BadParameter(f"{checkpoint}: no runnable configuration")
    costs = _layer_bytes(res)
    ranges = balanced_ranges([c or 1.0 for c in costs], stages)
    mans = []
    for i, (a, b) in enumerate(ranges):
        m = build_stage_artifact(res, out, a, b, embed=i == 0, head=i == len(ranges) - 1)
        mans.append(m.to_json())
    typer.echo(json.dumps(mans, indent=1))


@model_app.command("inspect")
def model_inspect(path: str, as_json: bool = typer.Option(True, "--json/--text")):
    """Inspect a model source (preset, local checkpoint or GGUF): format, revision, size and
    architecture profile."""
    from .model_io.resolver import ModelSourceResolver
    res = ModelSourceResolver().inspect(path)
    _out({"source": res.source, "revision": res.revision, "format": res.format,
          "total_bytes": res.total_bytes, **res.profile.summary()}, as_json)


@model_app.command("feasibility")
def model_feasibility(path: str, batch: int = 32, ctx: int = 4096,
                      as_json: bool = typer.Option(True, "--json/--text")):
    """Headers-only sizing of a checkpoint against B200 GPUs (180 GB each, 8 per box)."""
    from .model_io.facts import b200_feasibility
    from .model_io.resolver import ModelSourceResolver
    _out(b200_feasibility(ModelSourceResolver().inspect(path), batch=batch, context=ctx), as_json)


@model_app.command("variants")
def model_variants(directory: str, memory_gb: float = 180.0, objective: str = "balanced",
                   request: str = typer.Option(None, "--variant"),
                   as_json: bool = typer.Option(True, "--json/--text")):
    """Complete GGUF variants in a directory and the one selected for the objective."""
    from pathlib import Path
    from .model_io.facts import discover_gguf_variants, select_variant
    root = Path(directory)
    listing = {p.relative_to(root).as_posix(): p.stat().st_size for p in root.rglob("*.gguf")}
    vs = discover_gguf_variants(listing)
    sel = select_variant(vs, memory_bytes=int(memory_gb * 1e9), objective=objective, request=request)
    _out({"selected": sel.selected.variant_id, "feasible": sel.feasible,
          "candidates": [{"variant": c.variant.variant_id, "quant": c.variant.quant,
                          "bytes": c.variant.total_bytes, "bits_per_weight": c.variant.bits_per_weight,
                          "feasible": c.feasible, "reason": c.reason} for c in sel.candidates]},
         as_json)


@app.command("plan")
def plan_command(model: str, gpus: int = 8, batch: int = 32, ctx: int = 2304, prompt: int = 2048,
                 mode: str = "throughput", as_json: bool = typer.Option(False, "--json")):
    """Plan MODEL on one box of GPUS B200s: candidate layouts (TP / EP / PP / DP) ranked by
    predicted throughput from the measured peaks."""
    from .planner.box_planner import explain, plan_box, plan_json
    cfg, _ = _resolve_model(model)
    caps = _gpu_caps(gpus)
    plans = plan_box(cfg, gpus, caps.measurements, batch=batch, ctx=ctx, prompt=prompt, mode=mode)
    if as_json:
        typer.echo(json.dumps([plan_json(p) for p in plans[:8]], default=str))
    else:
        typer.echo(explain(plans, 8))


@app.command("worker")
def worker_command(stage: int, stages: int, preset: str = "tiny-llama-cpu", port: int = 0,
                   next_hop: str = typer.Option("", "--next"), seed: int = 0,
                   backend: str = "reference"):
    """Run one stage-ring worker process (stage STAGE of STAGES) on this host."""
    from .runtime.worker import main as worker_main
    worker_main(["--preset", preset, "--stage", str(stage), "--stages", str(stages), "--port",
                 str(port), "--next", next_hop, "--seed", str(seed), "--backend", backend])


@probe_app.command("nvlink")
def probe_nvlink(out: str = "nvlink_probe.json"):
    """Measure GPU-to-GPU copy bandwidth and latency on this box (one process per GPU under
    torchrun)."""
    from .parallel.nvlink_probe import main as probe_main
    sys.argv = ["nvlink_probe", "--out", out]
    probe_main()


@identity_app.command("show")
def identity_show(state: str = typer.Option(STATE, "--state-dir")):
    """This node's Ed25519 identity: name and fingerprint."""
    ident = _store(state).identity()
    typer.echo(json.dumps({"name": ident.name, "fingerprint": ident.fingerprint}))


@identity_app.command("create")
def identity_create(name: str = typer.Option("node", "--name"),
                    out: str = typer.Option(..., "--out"),
                    force: bool = typer.Option(False, "--force")):
    """Create an Ed25519 identity document at OUT (refuses to overwrite without --force)."""
    from .security.identity import Identity
    p = Path(out).expanduser()
    if p.exists() and not force:
        typer.echo(f"{p} exists; pass --force to replace it", err=True)
        raise typer.Exit(EXIT_USAGE)
    ident = Identity.generate(name)
    ident.save(p)
    typer.echo(json.dumps({"name": ident.name, "fingerprint": ident.fingerprint, "path": str(p)}))


@identity_app.command("fingerprint")
def identity_fingerprint(path: str):
    """The fingerprint of the identity document at PATH (what cluster membership and signed
    route leases are bound to)."""
    from .security.identity import Identity
    typer.echo(Identity.load(Path(path).expanduser()).fingerprint)


@experiment_app.command("loopback-matrix")
def experiment_loopback_matrix(workers: str = "2,4,8", concurrency: str = "1,16,64",
                               stages: int = 1, tokens: int = 16,
                               out: str = "loopback_matrix.json", csv_out: str = typer.Option(None, "--csv")):
    """Replica scaling x concurrency and worker fan-out (cold / warm deploy, lease economics)
    with verified tokens, on in-process workers."""
    from .testing.loopback_matrix import main as lm_main
    args = ["--workers", workers, "--concurrency", concurrency, "--stages", str(stages),
            "--tokens", str(tokens), "--out", out]
    lm_main(args + (["--csv", csv_out] if csv_out else []))


@experiment_app.command("wan-ring")
def experiment_wan_ring(profiles: str = "loopback,wifi,regional,global", tokens: int = 16,
                        out: str = typer.Option(None, "--out")):
    """Stage-ring decode through delaying proxies at emulated network profiles: exact tokens,
    messages, payload bytes and serial waits per token."""
    from .testing.wan_ring import main as wan_main
    wan_main(["--profiles", profiles, "--tokens", str(tokens)] + (["--out", out] if out else []))


@experiment_app.command("microsharding")
def experiment_microsharding(tokens: int = 16, repeats: int = 3,
                             out: str = typer.Option(None, "--out")):
    """One MoE decoder with its experts local, whole on a remote expert worker, and as
    microshards over 2 and 4 workers (SWARMEX1 over TCP): time per forward, remote requests
    and rows, and exactness against local execution."""
    from .testing.expert_backends import main as eb_main
    eb_main(["--tokens", str(tokens), "--repeats", str(repeats)] + (["--out", out] if out else []))


@experiment_app.command("real-loopback")
def experiment_real_loopback(checkpoint: str, stages: int = 4, tokens: int = 24,
                             out: str = typer.Option(None, "--out")):
    """A safetensors CHECKPOINT served as STAGES process-isolated pipeline stages on this host
    (cluster create/start, pair + join + agent per node, ``run --require-distributed``),
    checked token for token against the checkpoint's own greedy generation."""
    from .testing.real_loopback import main as rl_main
    raise typer.Exit(rl_main([checkpoint, "--stages", str(stages), "--tokens", str(tokens)]
                             + (["--out", out] if out else [])))


@experiment_app.command("heterogeneous")
def experiment_heterogeneous(seconds: float = 3.0, tokens: int = 16,
                             out: str = typer.Option(None, "--out")):
    """Whether a weaker node adds tokens/s, measured on this host: a background audit lane
    beside a primary decode lane, planner-assigned node roles against their observed aggregate,
    and a CPU expert host taking the experts local memory cannot hold (exact against
    all-local execution)."""
    from .testing.heterogeneous import main as het_main
    raise typer.Exit(het_main(["--seconds", str(seconds), "--tokens", str(tokens)]
                              + (["--out", out] if out else [])))


@experiment_app.command("node-roles")
def experiment_node_roles(nodes: str, model_gb: float = typer.Option(..., "--model-gb"),
                          expert_fraction: float = typer.Option(0.0, "--expert-fraction"),
                          as_json: bool = typer.Option(True, "--json/--text")):
    """Assign heterogeneous nodes (NODES: a JSON list of {node_id, decode_tok_s, memory_gb,
    link_ms}) to pipeline-stage, expert-host, draft-host or idle roles by marginal gain in
    aggregate tokens/s; a node that would slow the plan down stays idle."""
    from .planner.roles import NodeCaps, assign_roles
    doc = json.loads(Path(nodes).read_text())
    caps = [NodeCaps(n["node_id"], float(n["decode_tok_s"]), float(n["memory_gb"]) * 1e9,
                     float(n.get("link_ms", 0.0))) for n in doc]
    roles = assign_roles(caps, model_gb * 1e9, expert_fraction=expert_fraction)
    rows = [{"node_id": r.node_id, "role": r.role, "gain_tok_s": r.gain_tok_s} for r in roles]
    if as_json:
        typer.echo(json.dumps(rows, indent=1))
    else:
        for r in rows:
            typer.echo(f"{r['node_id']}: {r['role']} (+{r['gain_tok_s']:.1f} tok/s)")


@experiment_app.command("engine-performance")
def experiment_engine_performance(gpus: int = 1, steps: int = 64, warmup: int = 3,
                                  impl: str = typer.Option("ours", "--impl"),
                                  model: str = typer.Option("llama-3-8b-shape", "--model")):
    """The single-engine decode benchmark (``bench.py``: device-timed tokens/s, TTFT, TPOT, end
    to end through ``LLMEngine.step``) on this box; ``--impl reference`` runs the reference's
    own engine.  Multi-GPU runs use torchrun (127.0.0.1 rendezvous)."""
    root = Path(__file__).resolve().parent.parent
    args = ["bench.py", "--gpus", str(gpus), "--steps", str(steps), "--warmup", str(warmup),
            "--impl", impl, "--model", model]
    if gpus > 1:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={gpus}", "--master-addr", "127.0.0.1", "--master-port", "29555"] + args
    else:
        cmd = [sys.executable] + args
    raise typer.Exit(subprocess.call(cmd, cwd=str(root)))


@app.command("validate-run")
def validate_run(contract: str, evidence: str):
    """Check EVIDENCE (a JSON record, or the last JSON line of a log) against a frozen
    CONTRACT (a name under testing/contracts or a YAML path); exit 1 when a gate fails."""
    from .testing.acceptance import main as acc_main
    raise typer.Exit(acc_main([contract, evidence]))


@app.command("report")
def report_command(evidence: list[str],
                   fmt: str = typer.Option("md", "--format", help="md, html or csv"),
                   out: str = typer.Option(None, "--out", help="write a bundle to this directory"),
                   title: str = typer.Option("Evidence report", "--title")):
    """Render evidence files (JSON, JSON lines, or logs whose JSON lines are evidence: bench
    lines, contract results, ring strategies, WAN, loopback, real-loopback and expert-backend
    rows) as markdown, HTML with inline charts, or CSV, with scaling figures for bench lines
    at several GPU counts.  ``--out DIR`` writes the whole bundle (report.html, report.md,
    one CSV per kind, summary.json, records.jsonl) and exits 1 when a contract or an
    exactness check failed."""
    from .testing import reporting
    records = reporting.load(evidence)
    if out:
        s = reporting.write_bundle(records, out, title)
        typer.echo(json.dumps({k: s[k] for k in ("records", "kinds", "status", "failed")}))
        raise typer.Exit(0 if s["status"] == "PASS" else 1)
    if fmt == "html":
        typer.echo(reporting.to_html(records, title))
    elif fmt == "csv":
        for k, rows in reporting.rows_by_kind(records).items():
            typer.echo(f"# {k}")
            typer.echo(reporting.to_csv(rows))
    elif fmt == "md":
        typer.echo(reporting.to_markdown(records))
    else:
        raise typer.BadParameter("--format must be md, html or csv")


@app.command("simulate")
def simulate_command(stages: int = 2, requests: int = 32, prompt_tokens: int = 128,
                     output_tokens: int = 64, decode_ms: float = 5.0, prefill_us_per_token: float = 50.0,
                     latency_ms: float = 1.0, bandwidth_mbps: float = 1000.0, jitter_ms: float = 0.0,
                     loss: float = 0.0, hidden_bytes: int = 8192, arrival_ms: float = 0.0,
                     seed: int = 0, as_json: bool = typer.Option(False, "--json")):
    """Discrete-event simulation of a pipeline ring: STAGES equal stages, one link profile,
    REQUESTS arriving every ARRIVAL_MS; prints tokens/s, p50 TTFT / TPOT and resends."""
    from .testing.simulation import Link, StageNode, simulate_ring
    nodes = [StageNode(f"s{i}", decode_ms / 1e3 / stages, prefill_us_per_token / 1e6 / stages)
             for i in range(stages)]
    link = Link(latency_s=latency_ms / 1e3, bandwidth_Bps=bandwidth_mbps * 1e6 / 8,
                jitter_s=jitter_ms / 1e3, loss=loss)
    rep = simulate_ring(nodes, link, requests=requests, prompt_tokens=prompt_tokens,
                        output_tokens=output_tokens, hidden_bytes=hidden_bytes,
                        arrival_s=arrival_ms / 1e3, seed=seed)
    _out(rep, as_json)


@app.command("topology")
def topology_command(rtt_ms: float = typer.Option(None, "--rtt-ms"),
                     bandwidth_mbps: float = typer.Option(None, "--bandwidth-mbps"),
                     jitter_ms: float = 0.0, stability: float = 1.0,
                     nvlink: bool = typer.Option(False, "--nvlink"),
                     message_bytes: int = 8192, as_json: bool = typer.Option(False, "--json")):
    """Classify a link (NVLink, local-fast, regional, WAN, unknown) from its measured RTT,
    bandwidth, jitter and stability, and the one-way time of a MESSAGE_BYTES message."""
    from .planner.topology import LinkProfile, classify, transfer_ms
    link = LinkProfile("a", "b", rtt_ms, bandwidth_mbps / 8 if bandwidth_mbps else None,
                       jitter_ms=jitter_ms, stability=stability, kind="nvlink" if nvlink else "tcp",
                       measured=rtt_ms is not None or nvlink)
    _out({"domain": classify(link).value, "message_bytes": message_bytes,
          "one_way_ms": transfer_ms(link, message_bytes)}, as_json)


def _fingerprint_arg(value: str) -> str:
    """A fingerprint given directly (``sha256:...``) or read from an identity document."""
    if value.startswith("sha256:"):
        return value
    from .security.identity import Identity
    return Identity.load(Path(value).expanduser()).fingerprint


@identity_app.command("trust")
def identity_trust(identity: str, label: str = typer.Option("", "--label"),
                   notes: str = typer.Option("", "--notes"),
                   state: str = typer.Option(STATE, "--state-dir")):
    """Let the coordinator of this cluster admit a worker identity at registration without
    pairing (IDENTITY: a ``sha256:`` fingerprint or an identity document).  A revoked identity
    stays refused; with mutual TLS on, the worker still needs a certificate of the cluster CA."""
    fp = _fingerprint_arg(identity)
    added = _store(state).trust(fp, label=label, notes=notes)
    typer.echo(json.dumps({"status": "trusted" if added else "updated", "fingerprint": fp}))


@identity_app.command("untrust")
def identity_untrust(identity: str, state: str = typer.Option(STATE, "--state-dir")):
    """Remove a worker identity from the trust list."""
    fp = _fingerprint_arg(identity)
    gone = _store(state).untrust(fp)
    typer.echo(json.dumps({"status": "removed" if gone else "absent", "fingerprint": fp}))
    if not gone:
        raise typer.Exit(1)


@identity_app.command("list-trusted")
def identity_list_trusted(state: str = typer.Option(STATE, "--state-dir")):
    """Worker identities on the trust list, with their labels."""
    typer.echo(json.dumps(_store(state).trusted(), indent=1, default=str))


def main():  # console entry point
    app()


if __name__ == "__main__":
    main()
