"""The ``swarm`` command line.

    swarm cluster create NAME            # this machine becomes coordinator; prints a pairing URI
    swarm cluster pair                   # mint another single-use pairing URI
    swarm cluster status | nodes | revoke NODE | delete
    swarm node join URI                  # pair this machine with a cluster
    swarm node status | doctor | leave
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
Without a tokenizer on the box, ``--prompt`` text is mapped to ids byte-wise
(deterministic; documented as such in the output).

Reference: si/cli.py:129-2372 and si/commands/{run,cluster,node}.py.
"""
from __future__ import annotations

import asyncio
import json
import os
import sys
import time
from pathlib import Path

import typer

app = typer.Typer(add_completion=False, help="Blackwell-native distributed inference runtime")
cluster_app = typer.Typer(help="cluster lifecycle")
node_app = typer.Typer(help="this node")
model_app = typer.Typer(help="model inspection")
identity_app = typer.Typer(help="node identity")
probe_app = typer.Typer(help="measurements")
app.add_typer(cluster_app, name="cluster")
app.add_typer(node_app, name="node")
app.add_typer(model_app, name="model")
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


def _prompt_ids(prompt: str | None, prompt_ids: str | None, vocab: int) -> tuple[list[int], str]:
    if prompt_ids:
        return [int(x) for x in prompt_ids.split(",") if x.strip()], "ids"
    text = prompt or "Hello"
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
                seed: int = typer.Option(0, "--seed")):
    """Resolve, plan and run MODEL on this box, streaming tokens."""
    from .engines import EngineRegistry, RequestShape
    if mode not in ("speed", "throughput", "capacity", "balanced"):
        raise typer.BadParameter("mode must be speed|throughput|capacity|balanced")
    cfg, res = _resolve_model(model)
    ids, tok_kind = _prompt_ids(prompt, prompt_ids, cfg.vocab_size)
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
                   "rejected": comp.rejected, "prompt_tokenization": tok_kind}
    if explain_plan or dry_run:
        _out(explanation, as_json or ndjson)
        if dry_run:
            return
    if plan.parallelism.get("tp", 1) * plan.parallelism.get("pp", 1) > 1:
        typer.echo("multi-GPU plans run under torchrun (see bench.py); serving this request on one GPU",
                   err=True)
    from .engine.engine import LLMEngine, SamplingParams
    t0 = time.perf_counter()
    eng = LLMEngine(cfg, device="cuda", seed=seed, max_batch=1,
                    max_seq_len=len(ids) + max_tokens + 64,
                    weights=None)
    eng.add_request(ids, SamplingParams(max_new_tokens=max_tokens), request_id="cli")
    out = []
    while eng.scheduler.has_work():
        for rid, tok in eng.step():
            out.append(tok)
            if ndjson:
                typer.echo(json.dumps({"event": "TOKEN_GENERATED", "token": tok, "index": len(out) - 1}))
    dt = time.perf_counter() - t0
    result = {"tokens": out, "output_tokens": len(out), "seconds": round(dt, 3)}
    if ndjson:
        typer.echo(json.dumps({"event": "REQUEST_COMPLETED", **result}))
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
    st = _store(state)
    doc = st.load_cluster()
    _out({"cluster": doc["name"], "role": doc["role"], "coordinator": doc["coordinator_endpoint"],
          "members": len(doc["members"]), "revoked": len(doc["revoked"])}, as_json)


@cluster_app.command("nodes")
def cluster_nodes(state: str = typer.Option(STATE, "--state-dir")):
    doc = _store(state).load_cluster()
    typer.echo(json.dumps(doc["members"], indent=1, default=str))


@cluster_app.command("revoke")
def cluster_revoke(node: str, state: str = typer.Option(STATE, "--state-dir")):
    fp = _store(state).revoke(node)
    typer.echo(f"revoked {node} ({fp})")


@cluster_app.command("delete")
def cluster_delete(state: str = typer.Option(STATE, "--state-dir"), yes: bool = typer.Option(False, "--yes")):
    if not yes:
        typer.echo("refusing to delete cluster state without --yes", err=True)
        raise typer.Exit(EXIT_USAGE)
    _store(state).delete()
    typer.echo("deleted")


@cluster_app.command("pair")
def cluster_pair(serve: bool = typer.Option(False, "--serve"), ttl: float = 600.0,
                 state: str = typer.Option(STATE, "--state-dir")):
    """Mint a pairing URI (and with --serve, answer pairing requests until interrupted)."""
    from .cluster.pairing import PairingManager
    st = _store(state)
    doc = st.load_cluster()
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


# ------------------------------------------------------------------ node
@node_app.command("join")
def node_join(uri: str, node_id: str = typer.Option(None, "--name"),
              state: str = typer.Option(STATE, "--state-dir")):
    from .cluster.pairing import join
    from .worker_caps import local_capabilities
    caps = local_capabilities(benchmark=False)
    rep = asyncio.run(join(uri, _store(state), node_id or os.uname().nodename, capabilities=caps))
    typer.echo(f"joined cluster {rep['cluster']} (coordinator {rep['coordinator_endpoint']})")


@node_app.command("status")
def node_status(state: str = typer.Option(STATE, "--state-dir"), as_json: bool = typer.Option(False, "--json")):
    st = _store(state)
    info = {"identity": st.identity().fingerprint, "state_dir": str(st.root)}
    if st.has_cluster():
        doc = st.load_cluster()
        info.update(cluster=doc["name"], role=doc["role"], coordinator=doc["coordinator_endpoint"])
    _out(info, as_json)


@node_app.command("doctor")
def node_doctor(as_json: bool = typer.Option(False, "--json")):
    from .doctor import run_doctor
    rep = run_doctor()
    _out(rep, as_json)
    if not rep.get("ok"):
        raise typer.Exit(EXIT_RUNTIME)


@node_app.command("leave")
def node_leave(state: str = typer.Option(STATE, "--state-dir"), yes: bool = typer.Option(False, "--yes")):
    if not yes:
        typer.echo("refusing to leave without --yes", err=True)
        raise typer.Exit(EXIT_USAGE)
    _store(state).delete()
    typer.echo("left the cluster; local state removed")


# ------------------------------------------------------------------ model / plan
@model_app.command("inspect")
def model_inspect(path: str, as_json: bool = typer.Option(True, "--json/--text")):
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
    from .runtime.worker import main as worker_main
    worker_main(["--preset", preset, "--stage", str(stage), "--stages", str(stages), "--port",
                 str(port), "--next", next_hop, "--seed", str(seed), "--backend", backend])


@probe_app.command("nvlink")
def probe_nvlink(out: str = "nvlink_probe.json"):
    from .parallel.nvlink_probe import main as probe_main
    sys.argv = ["nvlink_probe", "--out", out]
    probe_main()


@identity_app.command("show")
def identity_show(state: str = typer.Option(STATE, "--state-dir")):
    ident = _store(state).identity()
    typer.echo(json.dumps({"name": ident.name, "fingerprint": ident.fingerprint}))


def main():  # console entry point
    app()


if __name__ == "__main__":
    main()
