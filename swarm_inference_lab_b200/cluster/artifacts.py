"""Content-addressed stage artifacts and resumable, verified chunked transfer.

``build_stage_artifact`` writes the tensors one stage owns (its layer
interval, plus the embedding on stage 0 and norm/head on the last stage)
into a safetensors file and a manifest naming the source revision, the
interval, the tensor list and the SHA-256 of the file; the artifact id is
the manifest's hash, so identical stages share one artifact.

``ArtifactStore`` keeps artifacts under ``<root>/<id>/`` with LRU eviction
under a byte budget (leased artifacts are never evicted).  ``transfer``
copies an artifact in fixed-size chunks, each verified by its SHA-256, and
resumes from the last verified chunk after an interruption (the resume
state is a small JSON next to the partial file).

Reference: si/cluster/artifacts.py:287-1531 (StageArtifactBuilder,
ArtifactTransferResume, ArtifactManager with leases and LRU).
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import time
from dataclasses import dataclass
from pathlib import Path

from ..model_io.resolver import ResolvedModel
from ..model_io.safetensors_io import CheckpointReader, save_safetensors

CHUNK = 8 << 20


def _sha256_file(p: Path) -> str:
    h = hashlib.sha256()
    with open(p, "rb") as f:
        for b in iter(lambda: f.read(1 << 20), b""):
            h.update(b)
    return h.hexdigest()


@dataclass
class ArtifactManifest:
    artifact_id: str
    revision: str
    layer_start: int
    layer_end: int
    embed: bool
    head: bool
    tensors: list[str]
    file_sha256: str
    bytes: int

    def to_json(self) -> dict:
        return self.__dict__.copy()


def build_stage_artifact(model: ResolvedModel, out_root: str | Path, layer_start: int,
                         layer_end: int, *, embed: bool, head: bool) -> ArtifactManifest:
    names = []
    for n, d in model.profile.tensors.items():
        if d.layer is not None and layer_start <= d.layer < layer_end:
            names.append(n)
        elif d.layer is None and ((embed and d.role.value == "embedding")
                                  or (head and d.role.value in ("final_norm", "output_head"))):
            names.append(n)
    names.sort()
    key = json.dumps({"rev": model.revision, "range": [layer_start, layer_end], "embed": embed,
                      "head": head, "tensors": names}, sort_keys=True).encode()
    aid = hashlib.sha256(key).hexdigest()[:32]
    d = Path(out_root) / aid
    d.mkdir(parents=True, exist_ok=True)
    reader = CheckpointReader(model.path)
    try:
        save_safetensors(d / "stage.safetensors", {n: reader.tensor(n) for n in names},
                         metadata={"revision": model.revision, "layers": f"{layer_start}:{layer_end}"})
    finally:
        reader.close()
    man = ArtifactManifest(aid, model.revision, layer_start, layer_end, embed, head, names,
                           _sha256_file(d / "stage.safetensors"), (d / "stage.safetensors").stat().st_size)
    (d / "manifest.json").write_text(json.dumps(man.to_json(), sort_keys=True))
    return man


class ArtifactError(RuntimeError):
    pass


class ArtifactStore:
    def __init__(self, root: str | Path, budget_bytes: int = 1 << 40):
        self.root = Path(root)
        self.root.mkdir(parents=True, exist_ok=True)
        self.budget = budget_bytes
        self.leases: dict[str, int] = {}

    def path(self, aid: str) -> Path:
        return self.root / aid

    def has(self, aid: str) -> bool:
        return (self.path(aid) / "manifest.json").exists()

    def manifest(self, aid: str) -> ArtifactManifest:
        return ArtifactManifest(**json.loads((self.path(aid) / "manifest.json").read_text()))

    def verify(self, aid: str) -> bool:
        m = self.manifest(aid)
        return _sha256_file(self.path(aid) / "stage.safetensors") == m.file_sha256

    def lease(self, aid: str) -> None:
        self.leases[aid] = self.leases.get(aid, 0) + 1
        os.utime(self.path(aid))

    def release(self, aid: str) -> None:
        self.leases[aid] = max(0, self.leases.get(aid, 0) - 1)

    def usage(self) -> int:
        return sum(f.stat().st_size for f in self.root.rglob("*") if f.is_file())

    def evict(self) -> list[str]:
        """Evict least-recently-used unleased artifacts until under budget."""
        gone = []
        items = sorted((p for p in self.root.iterdir() if p.is_dir()), key=lambda p: p.stat().st_mtime)
        for p in items:
            if self.usage() <= self.budget:
                break
            if self.leases.get(p.name, 0) > 0:
                continue
            shutil.rmtree(p)
            gone.append(p.name)
        return gone


def transfer(src: ArtifactStore, dst: ArtifactStore, aid: str, *, chunk: int = CHUNK,
             fail_after_chunks: int | None = None) -> int:
    """Copy artifact ``aid`` chunk by chunk with per-chunk SHA-256; resumable.
    ``fail_after_chunks`` simulates an interruption (tests).  Returns chunks copied now."""
    man = src.manifest(aid)
    sd, dd = src.path(aid), dst.path(aid)
    dd.mkdir(parents=True, exist_ok=True)
    part = dd / "stage.safetensors.part"
    state_p = dd / "transfer.json"
    state = json.loads(state_p.read_text()) if state_p.exists() else {"done": 0, "digests": []}
    copied = 0
    with open(sd / "stage.safetensors", "rb") as fin, open(part, "ab" if state["done"] else "wb") as fout:
        fout.truncate(state["done"] * chunk)
        fin.seek(state["done"] * chunk)
        while True:
            if fail_after_chunks is not None and copied >= fail_after_chunks:
                raise ArtifactError("transfer interrupted")
            b = fin.read(chunk)
            if not b:
                break
            d = hashlib.sha256(b).hexdigest()
            fout.write(b)
            fout.flush()
            os.fsync(fout.fileno())
            with open(part, "rb") as check:
                check.seek(state["done"] * chunk)
                if hashlib.sha256(check.read(len(b))).hexdigest() != d:
                    raise ArtifactError("chunk verification failed")
            state["done"] += 1
            state["digests"].append(d)
            state_p.write_text(json.dumps(state))
            copied += 1
    if _sha256_file(part) != man.file_sha256:
        raise ArtifactError("artifact digest mismatch after transfer")
    os.replace(part, dd / "stage.safetensors")
    (dd / "manifest.json").write_text(json.dumps(man.to_json(), sort_keys=True))
    state_p.unlink(missing_ok=True)
    os.utime(dd, (time.time(), time.time()))
    return copied
