"""Model source resolution: immutable local checkpoints and pinned Hugging Face revisions.

``ModelSourceResolver.inspect(source)`` accepts

* a local directory with ``config.json`` + safetensors (single file or
  index-sharded) - its revision is the SHA-256 of the config, the index (or
  file inventory) and the file sizes, so a changed checkpoint can never pass
  for an old one;
* a local ``.gguf`` file - revision = SHA-256 of its header bytes;
* ``hf://org/name@revision`` - resolved through ``huggingface_hub`` to a
  commit hash (needs network; offline it fails with a clear error unless
  the revision is already in the local cache).

It returns a :class:`ResolvedModel` with the architecture profile and the
tensor inventory, read from headers only.  ``select_files`` maps a stage's
layer interval to the shard files it needs (selective acquisition).

Reference: si/model/resolver.py:321-1034 (``ModelSourceResolver``,
``inspect``, ``_select_files``, ``acquire``).
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass, field
from pathlib import Path

from .architecture import ArchitectureProfile, default_registry
from .gguf import inspect_gguf
from .safetensors_io import inspect_checkpoint


class ResolutionError(RuntimeError):
    pass


@dataclass
class ResolvedModel:
    source: str
    path: Path
    revision: str
    format: str                     # safetensors | gguf
    profile: ArchitectureProfile
    files: dict[str, int] = field(default_factory=dict)   # file -> bytes
    tensor_files: dict[str, str] = field(default_factory=dict)  # tensor -> file
    tensor_bytes: dict[str, int] = field(default_factory=dict)

    @property
    def total_bytes(self) -> int:
        return sum(self.files.values())

    def select_files(self, layer_start: int, layer_end: int, *, embed: bool, head: bool) -> list[str]:
        """Shard files a stage owning layers [layer_start, layer_end) must acquire."""
        need = set()
        for name, d in self.profile.tensors.items():
            if d.layer is not None and layer_start <= d.layer < layer_end:
                need.add(self.tensor_files[name])
            elif d.layer is None:
                if (embed and d.role.value == "embedding") or (head and d.role.value in ("final_norm", "output_head")):
                    need.add(self.tensor_files[name])
        return sorted(need)

    def stage_bytes(self, layer_start: int, layer_end: int, *, embed: bool, head: bool) -> int:
        n = 0
        for name, d in self.profile.tensors.items():
            if d.layer is not None and layer_start <= d.layer < layer_end:
                n += self.tensor_bytes[name]
            elif d.layer is None and ((embed and d.role.value == "embedding")
                                      or (head and d.role.value in ("final_norm", "output_head"))):
                n += self.tensor_bytes[name]
        return n


class ModelSourceResolver:
    def __init__(self, registry=None, cache_dir: str | None = None):
        self.registry = registry or default_registry()
        self.cache_dir = cache_dir

    def inspect(self, source: str) -> ResolvedModel:
        if source.startswith("hf://"):
            return self._inspect_hub(source[5:])
        p = Path(source).expanduser()
        if p.is_file() and p.suffix == ".gguf":
            return self._inspect_gguf(p)
        if p.is_dir():
            return self._inspect_dir(p)
        raise ResolutionError(f"model source {source!r} is neither a checkpoint directory, a .gguf "
                              f"file nor an hf:// reference")

    def _inspect_dir(self, p: Path) -> ResolvedModel:
        cfg_path = p / "config.json"
        if not cfg_path.is_file():
            raise ResolutionError(f"{p}: config.json is missing")
        try:
            cfg = json.loads(cfg_path.read_text(encoding="utf-8"))
        except (OSError, UnicodeDecodeError, json.JSONDecodeError) as exc:
            raise ResolutionError(f"{cfg_path}: not valid UTF-8 JSON ({exc})") from None
        inv = inspect_checkpoint(p)
        prof = self.registry.resolve_config(cfg, sorted(inv))
        h = hashlib.sha256()
        h.update(cfg_path.read_bytes())
        idx = p / "model.safetensors.index.json"
        if idx.exists():
            h.update(idx.read_bytes())
        files = {}
        for f in sorted({t.file for t in inv.values()}):
            files[Path(f).name] = os.path.getsize(f)
            h.update(f"{Path(f).name}:{files[Path(f).name]}".encode())
        for name in sorted(inv):
            t = inv[name]
            h.update(f"{name}:{t.dtype}:{t.shape}:{t.begin}:{t.end}".encode())
        return ResolvedModel(str(p), p, "sha256:" + h.hexdigest(), "safetensors", prof, files,
                             {n: Path(t.file).name for n, t in inv.items()},
                             {n: t.nbytes for n, t in inv.items()})

    def _inspect_gguf(self, p: Path) -> ResolvedModel:
        desc = inspect_gguf(p)
        prof = self.registry.resolve_gguf(desc.metadata, [t.name for t in desc.tensors])
        with open(p, "rb") as f:
            head = f.read(desc.data_offset)
        rev = "sha256:" + hashlib.sha256(head).hexdigest()
        return ResolvedModel(str(p), p, rev, "gguf", prof, {p.name: p.stat().st_size},
                             {t.name: p.name for t in desc.tensors},
                             {t.name: t.nbytes for t in desc.tensors})

    def _inspect_hub(self, ref: str) -> ResolvedModel:
        repo, _, rev = ref.partition("@")
        if not rev:
            raise ResolutionError("hf:// references must pin a revision (commit hash or tag)")
        try:
            from huggingface_hub import snapshot_download
            local = snapshot_download(repo_id=repo, revision=rev, cache_dir=self.cache_dir,
                                      allow_patterns=["config.json", "*.safetensors.index.json"],
                                      local_files_only=os.environ.get("HF_HUB_OFFLINE") == "1")
        except Exception as exc:  # noqa: BLE001 - network / auth / cache misses
            raise ResolutionError(f"cannot resolve {ref}: {type(exc).__name__}: {exc}") from None
        return self._inspect_dir(Path(local))
