"""An exact PyTorch backend for the universal worker ABI (``runtime/abi.py``).

``TorchRankBackend`` holds one real model -- a preset with its seeded weights or a
safetensors checkpoint -- in the fp32 reference decoder (CPU, or a GPU device) and serves
the ABI's jobs with no synthetic fallback:

* ``generate(prompt, max_new_tokens)`` -> ``{tokens}``: greedy decode with a KV cache;
* ``draft(context, k)`` -> ``{draft}``: prompt-lookup proposals (the tokens that followed the
  latest earlier match of the context's trailing n-gram);
* ``verify(context, candidates)`` -> ``{accepted, next}``: one forward over the context and
  the candidates; the longest candidate prefix equal to the greedy predictions is accepted
  and ``next`` is the greedy token after it -- the same answer as ``GreedyVerifier`` with
  one model call instead of one per candidate;
* ``background(name="integrity_audit", args={prompt, tokens})`` -> ``{agreed, first_mismatch}``:
  recomputes a claimed greedy continuation and reports where it first differs.

Reference: si/backends/torch_rank.py:39 (``TorchRankAdapter``: one real stage per process,
exact, no synthetic fallback; pipeline, tensor-rank and integrity-audit jobs).
"""
from __future__ import annotations

import torch

from ..engine.speculative import prompt_lookup_draft


class TorchRankBackend:
    def __init__(self, model: dict, *, device: str = "cpu", dtype=torch.float32):
        """``model``: ``{"preset": name, "seed": s}`` or ``{"checkpoint": dir}``."""
        from ..models.reference import ReferenceDecoder
        if "checkpoint" in model:
            from ..model_io.loader import checkpoint_config, safetensors_source
            cfg = checkpoint_config(model["checkpoint"])
            get = safetensors_source(model["checkpoint"])
        else:
            from ..models.config import preset
            from ..models.reference import random_source
            cfg = preset(model["preset"])
            get = random_source(int(model.get("seed", 0)))
        self.cfg = cfg
        self.model = ReferenceDecoder(cfg, get, device=device, dtype=dtype)
        self.jobs = 0

    @torch.no_grad()
    def _logits(self, ids: list[int]) -> torch.Tensor:
        return self.model.forward(torch.tensor(ids, dtype=torch.long), self.model.new_cache())

    @torch.no_grad()
    def generate(self, prompt: list[int], max_new_tokens: int) -> dict:
        self.jobs += 1
        if max_new_tokens == 0:
            return {"tokens": []}
        cache = self.model.new_cache()
        logits = self.model.forward(torch.tensor(prompt, dtype=torch.long), cache)
        out = [int(torch.argmax(logits[-1]))]
        while len(out) < max_new_tokens:
            logits = self.model.forward(torch.tensor([out[-1]], dtype=torch.long), cache)
            out.append(int(torch.argmax(logits[-1])))
        return {"tokens": out}

    def draft(self, context: list[int], k: int) -> dict:
        self.jobs += 1
        return {"draft": prompt_lookup_draft(list(context), int(k))}

    @torch.no_grad()
    def verify(self, context: list[int], candidates: list[int]) -> dict:
        self.jobs += 1
        if not context:
            raise ValueError("verify needs a non-empty context")
        logits = self._logits(list(context) + list(candidates))
        preds = torch.argmax(logits[len(context) - 1:], dim=-1).tolist()
        accepted = 0
        while accepted < len(candidates) and candidates[accepted] == preds[accepted]:
            accepted += 1
        return {"accepted": accepted, "next": int(preds[accepted])}

    def background(self, name: str, args: dict | None = None) -> dict:
        self.jobs += 1
        args = args or {}
        if name != "integrity_audit":
            raise ValueError(f"unknown background job {name!r}")
        prompt, claimed = list(args["prompt"]), list(args["tokens"])
        mine = self.generate(prompt, len(claimed))["tokens"]
        first = next((i for i, (a, b) in enumerate(zip(mine, claimed)) if a != b), None)
        return {"agreed": first is None, "first_mismatch": first, "recomputed": mine}
