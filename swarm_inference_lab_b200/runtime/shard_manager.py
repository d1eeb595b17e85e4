"""Stage-only shard loading with memory and integrity limits.

A stage owner loads exactly the tensors of its assignment (its layer interval,
plus embedding / final norm / LM head on the edge stages) from a local checkpoint
or a stage artifact: shard files are opened lazily (memory-mapped safetensors),
each file's SHA-256 is checked against the manifest when one is given, and the
load is refused before any tensor is materialised if the stage would exceed the
memory budget.  Loaded stages are tracked so an unload releases their memory.

Reference: si/worker/shard_manager.py:69.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field
from pathlib import Path

import torch

from ..model_io.resolver import ResolvedModel
from ..model_io.safetensors_io import CheckpointReader


class ShardLimitError(RuntimeError):
    pass


class ShardIntegrityError(RuntimeError):
    pass


def file_sha256(p: Path) -> str:
    h = hashlib.sha256()
    with open(p, "rb") as f:
        for b in iter(lambda: f.read(1 << 20), b""):
            h.update(b)
    return h.hexdigest()


@dataclass
class LoadedStage:
    key: str
    tensors: dict[str, torch.Tensor]
    bytes: int
    files: list[str] = field(default_factory=list)


class ShardManager:
    def __init__(self, *, budget_bytes: int, device="cpu", dtype: torch.dtype | None = None):
        self.budget = budget_bytes
        self.device = torch.device(device)
        self.dtype = dtype
        self.loaded: dict[str, LoadedStage] = {}

    @property
    def used(self) -> int:
        return sum(s.bytes for s in self.loaded.values())

    def load_stage(self, model: ResolvedModel, layer_start: int, layer_end: int, *, embed: bool,
                   head: bool, file_digests: dict[str, str] | None = None) -> LoadedStage:
        key = f"{model.revision}:{layer_start}:{layer_end}:{int(embed)}{int(head)}"
        if key in self.loaded:
            return self.loaded[key]
        need = model.stage_bytes(layer_start, layer_end, embed=embed, head=head)
        if self.used + need > self.budget:
            raise ShardLimitError(f"stage needs {need} B, {self.budget - self.used} B left of {self.budget}")
        files = model.select_files(layer_start, layer_end, embed=embed, head=head)
        if file_digests:
            for f in files:
                want = file_digests.get(f)
                if want is None or file_sha256(Path(model.path) / f) != want:
                    raise ShardIntegrityError(f"{f}: digest mismatch")
        names = []
        for n, d in model.profile.tensors.items():
            if d.layer is not None and layer_start <= d.layer < layer_end:
                names.append(n)
            elif d.layer is None and ((embed and d.role.value == "embedding")
                                      or (head and d.role.value in ("final_norm", "output_head"))):
                names.append(n)
        reader = CheckpointReader(model.path)
        try:
            tensors = {}
            for n in sorted(names):
                t = reader.tensor(n)
                if self.dtype is not None and t.is_floating_point():
                    t = t.to(self.dtype)
                tensors[n] = t.to(self.device)
        finally:
            reader.close()
        st = LoadedStage(key, tensors, sum(t.numel() * t.element_size() for t in tensors.values()), files)
        self.loaded[key] = st
        return st

    def unload(self, key: str) -> None:
        self.loaded.pop(key, None)
