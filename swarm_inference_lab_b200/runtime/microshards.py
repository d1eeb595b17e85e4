"""Expert microshard artifacts: build them from a checkpoint and validate them.

A microshard of routed expert (layer l, expert e) is a contiguous slice [i0, i1) of the
expert's intermediate dimension: rows i0..i1 of its gate and up projections and the same
columns of its down projection.  The SwiGLU expert is a sum over intermediate channels, so
the microshards' outputs, added in shard order, give the expert's output; a worker that owns
one microshard serves ``silu(x G_s^T) * (x U_s^T) D_s^T`` (``ExpertStore``) and the caller
reduces the partials in fixed order (``reduce_fixed_order``).

``build_microshards`` writes one safetensors file per microshard with a manifest (source
revision, layer, expert, slice, tensor names, SHA-256).  ``validate_microshards`` checks the
files against their manifests, that the slices of every expert tile [0, I) exactly, and that
the fixed-order reduction of the microshards' outputs equals the whole expert's output on
random inputs (fp32).

Reference: si/microsharding/ (microshard ownership, fixed-order partial reduction) and the
``build-microshards`` / ``validate-microshards`` commands of si/cli.py.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch

from .expert_service import ExpertStore, Microshard, reduce_fixed_order, split_microshards


def _names(layer: int, expert: int) -> dict[str, str]:
    base = f"model.layers.{layer}.mlp.experts.{expert}"
    return {"gate": f"{base}.gate_proj.weight", "up": f"{base}.up_proj.weight",
            "down": f"{base}.down_proj.weight"}


def _sha256(p: Path) -> str:
    h = hashlib.sha256()
    with open(p, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _expert(get, cfg, layer: int, expert: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    inter, hidden = cfg.moe_intermediate_size or cfg.intermediate_size, cfg.hidden_size
    n = _names(layer, expert)
    return (get(n["gate"], (inter, hidden)), get(n["up"], (inter, hidden)),
            get(n["down"], (hidden, inter)))


def build_microshards(checkpoint: str | Path, out: str | Path, *, layers: list[int],
                      experts: list[int] | None, parts: int) -> list[dict]:
    """Writes ``parts`` microshards of every listed routed expert (all experts when None) of
    the listed layers; returns the manifests."""
    from safetensors.torch import save_file

    from ..model_io.loader import checkpoint_config, safetensors_source
    cfg = checkpoint_config(checkpoint)
    if not cfg.num_experts:
        raise ValueError(f"{checkpoint}: not a mixture-of-experts checkpoint")
    get = safetensors_source(checkpoint)
    rev = hashlib.sha256(json.dumps(json.loads((Path(checkpoint) / "config.json").read_text()),
                                    sort_keys=True).encode()).hexdigest()[:16]
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    mans = []
    for layer in layers:
        for e in (experts if experts is not None else range(cfg.num_experts)):
            gate, up, down = _expert(get, cfg, layer, e)
            for k, s in enumerate(split_microshards(layer, e, gate.shape[0], parts)):
                stem = f"l{layer:03d}_e{e:04d}_s{k:02d}"
                f = out / f"{stem}.safetensors"
                save_file({"gate": gate[s.i0:s.i1].contiguous(), "up": up[s.i0:s.i1].contiguous(),
                           "down": down[:, s.i0:s.i1].contiguous()}, str(f),
                          metadata={"layer": str(layer), "expert": str(e), "slice": f"{s.i0}:{s.i1}"})
                man = {"source_revision": rev, "layer": layer, "expert": e, "index": k,
                       "parts": parts, "i0": s.i0, "i1": s.i1, "intermediate": gate.shape[0],
                       "file": f.name, "sha256": _sha256(f)}
                (out / f"{stem}.json").write_text(json.dumps(man, sort_keys=True))
                mans.append(man)
    return mans


def validate_microshards(directory: str | Path, checkpoint: str | Path, *, rows: int = 8,
                         tol: float = 1e-5, seed: int = 0) -> dict:
    """Checks every microshard in ``directory`` against its manifest and, per expert, that the
    slices tile the intermediate dimension and that their fixed-order reduction reproduces
    the whole expert from ``checkpoint`` on ``rows`` random inputs."""
    from safetensors.torch import load_file

    from ..model_io.loader import checkpoint_config, safetensors_source
    d = Path(directory)
    cfg = checkpoint_config(checkpoint)
    get = safetensors_source(checkpoint)
    problems: list[str] = []
    groups: dict[tuple[int, int], list[dict]] = {}
    for mp in sorted(d.glob("*.json")):
        man = json.loads(mp.read_text())
        f = d / man["file"]
        if not f.is_file():
            problems.append(f"{man['file']}: missing")
            continue
        if _sha256(f) != man["sha256"]:
            problems.append(f"{man['file']}: SHA-256 mismatch")
            continue
        groups.setdefault((man["layer"], man["expert"]), []).append(man)
    g = torch.Generator().manual_seed(seed)
    worst = 0.0
    for (layer, e), mans in sorted(groups.items()):
        mans.sort(key=lambda m: m["i0"])
        inter = mans[0]["intermediate"]
        edges = [(m["i0"], m["i1"]) for m in mans]
        if edges[0][0] != 0 or edges[-1][1] != inter or any(
                a[1] != b[0] for a, b in zip(edges, edges[1:])):
            problems.append(f"layer {layer} expert {e}: slices {edges} do not tile [0, {inter})")
            continue
        gate, up, down = _expert(get, cfg, layer, e)
        x = torch.randn(rows, cfg.hidden_size, generator=g)
        whole = (torch.nn.functional.silu(x @ gate.float().T) * (x @ up.float().T)) @ down.float().T
        partials = {}
        for m in mans:
            t = load_file(str(d / m["file"]))
            store = ExpertStore()
            # the file holds exactly the slice: register it as the slice [0, n) of itself
            n = m["i1"] - m["i0"]
            store.add(Microshard(layer, e, 0, n), t["gate"], t["up"], t["down"])
            partials[m["index"]] = store.forward(layer, e, x)
        err = (reduce_fixed_order(partials) - whole).abs().max().item()
        scale = max(1.0, whole.abs().max().item())
        worst = max(worst, err / scale)
        if err > tol * scale:
            problems.append(f"layer {layer} expert {e}: reduction differs by {err:.3g}")
    return {"ok": not problems, "experts": len(groups),
            "microshards": sum(len(v) for v in groups.values()), "max_rel_err": worst,
            "problems": problems[:50]}
