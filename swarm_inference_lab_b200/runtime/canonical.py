"""Canonical runtime facade: one entry for inspecting a model source, planning a
request over the interchangeable engines, and building the serving engine.

    rt = CanonicalRuntime()
    info = rt.inspect("kimi-k2-shape")                 # preset, local checkpoint or hf://org/m@rev
    report = rt.dry_run("llama-3-8b-shape", caps, RequestShape(batch=32, ...))
    engine = rt.engine("tiny-llama-gpu", device="cuda")

``dry_run`` never loads weights: it resolves the source (headers only), runs the
engine competition and returns the winner's explanation plus every rejected
alternative with its reason.

Reference: si/runtime/canonical.py:85 (model inspection and dry-run over the engines).
"""
from __future__ import annotations

from dataclasses import asdict

from ..engines import ClusterCapabilities, EngineRegistry, RequestShape
from ..models.config import PRESETS, ModelConfig


class CanonicalRuntime:
    def __init__(self, registry: EngineRegistry | None = None, resolver=None):
        self.registry = registry or EngineRegistry()
        self._resolver = resolver

    @property
    def resolver(self):
        if self._resolver is None:
            from ..model_io.resolver import ModelSourceResolver
            self._resolver = ModelSourceResolver()
        return self._resolver

    def resolve(self, source: str):
        """(ModelConfig, ResolvedModel or None for presets)."""
        if source in PRESETS:
            return PRESETS[source], None
        res = self.resolver.inspect(source)
        if res.profile.config is None:
            raise ValueError(f"{source}: no runnable configuration ({res.profile.notes})")
        return res.profile.config, res

    def inspect(self, source: str) -> dict:
        cfg, res = self.resolve(source)
        out = {"model": cfg.name, "family": cfg.family, "layers": cfg.num_layers,
               "hidden": cfg.hidden_size, "parameters": cfg.parameter_count(),
               "moe": cfg.is_moe, "mla": cfg.mla, "weight_dtype": cfg.weight_dtype,
               "revision": res.revision if res else "preset"}
        if res is not None:
            out.update(format=res.format, bytes=res.total_bytes, files=len(res.files),
                       tensors=len(res.profile.tensors))
        return out

    def plan(self, cfg: ModelConfig, caps: ClusterCapabilities, req: RequestShape):
        return self.registry.compete(cfg, caps, req)

    def dry_run(self, source: str, caps: ClusterCapabilities, req: RequestShape) -> dict:
        cfg, res = self.resolve(source)
        comp = self.plan(cfg, caps, req)
        w = comp.winner
        return {
            "model": cfg.name, "revision": res.revision if res else "preset",
            "request": asdict(req),
            "winner": None if w is None else {
                "engine": w.engine, "plan": w.description, "parallelism": w.parallelism,
                "predicted_tok_s": w.predicted_tok_s, "predicted_ttft_ms": w.predicted_ttft_ms,
                "mechanisms": w.mechanisms, "confidence": w.confidence, "terms": w.explain},
            "alternatives": [p.description for p in comp.ranked[1:4]],
            "rejected": comp.rejected,
        }

    def engine(self, source: str, *, device="cuda", seed: int = 0, max_batch: int = 8,
               max_seq_len: int = 4096, **kw):
        from ..engine.engine import LLMEngine
        cfg, _ = self.resolve(source)
        return LLMEngine(cfg, device=device, seed=seed, max_batch=max_batch,
                         max_seq_len=max_seq_len, **kw)
