"""Model facts read from metadata only: the checkpoint's quantization scheme, the GGUF
variants a repository offers, whether a checkpoint fits a B200 box, bounded discovery
of several checkpoints, and the persisted model manifest.

Nothing here reads tensor data.  Every function works from ``config.json``, safetensors
headers, GGUF headers or file listings, so it runs on a host without a GPU and without
the weights.

* :func:`quantization_scheme` maps a ``quantization_config`` (compressed-tensors
  ``config_groups``, ``quant_method`` + ``fmt`` / ``bits`` / ``weight_block_size``,
  MXFP4) to one canonical name, and :func:`b200_kernel_for` says which sm_100a GEMM
  path executes it (bf16 tcgen05, or block-scaled e4m3 tcgen05 for 128x128 weight
  blocks) or why none does.
* :func:`discover_gguf_variants` groups split GGUF files (``stem-00001-of-00004.gguf``)
  atomically, drops auxiliary files (projectors, imatrix, tokenizer) and incomplete
  splits, and returns one variant per quantization tag with an estimated bits per
  weight; :func:`select_variant` picks one for an objective among the variants that
  fit the memory, or honours an explicit request even when it does not fit.
* :func:`b200_feasibility` sizes a resolved checkpoint against B200 GPUs
  (180 GB HBM3e each, 8 per NVLink box): weight bytes by layer and by expert /
  non-expert role, KV bytes per token (GQA pairs or the MLA latent row), the GPU and
  box counts for a target batch x context, and the layout the engine would use.
* :func:`discover_models` inspects a bounded explicit list and records, per
  reference, a profile or the inspection error.
* :func:`build_manifest`, :func:`save_manifest`, :func:`load_manifest`,
  :func:`verify_manifest_shards` and :func:`manifest_summary` persist a stage split
  with the SHA-256 of every shard file (directories hash their sorted file list).

Reference: si/model/quantization.py:9-95 (scheme names), si/model/variants.py:11-241
(GGUF variants and selection), si/model/feasibility.py:25-188 (index-only analysis),
si/model/discovery.py:73-105 (bounded discovery), si/model/manifest.py:12-82
(manifest persistence and shard hashes).
"""
from __future__ import annotations

import hashlib
import json
import math
import re
from dataclasses import dataclass
from pathlib import Path

from ..config.models import ConfigError, ModelManifest, StageDefinition

# ----------------------------------------------------------------------------------------
# quantization scheme names
# ----------------------------------------------------------------------------------------

_DTYPE_ALIASES = {"bfloat16": "bf16", "float16": "f16", "half": "f16", "float32": "f32",
                  "float": "f32", "float8-e4m3fn": "fp8-e4m3", "float8-e4m3": "fp8-e4m3",
                  "e4m3": "fp8-e4m3", "e4m3fn": "fp8-e4m3"}


def normalize_quant_name(value: str | None) -> str | None:
    """Lower-case, non-alphanumerics to ``-``, and fold spellings of one format together
    (``float8_e4m3fn`` / ``FP8-E4M3`` -> ``fp8-e4m3``, ``bfloat16`` -> ``bf16``)."""
    if value is None:
        return None
    s = re.sub(r"[^a-z0-9]+", "-", str(value).lower()).strip("-")
    if not s:
        return None
    if "mxfp4" in s:
        return "mxfp4"
    if "fp8" in s and "e4m3" in s or s.startswith("float8-e4m3"):
        return "fp8-e4m3"
    if "fp8" in s and "e5m2" in s:
        return "fp8-e5m2"
    return _DTYPE_ALIASES.get(s, s)


def _group_schemes(qc: dict) -> list[str]:
    """compressed-tensors style ``config_groups``: one scheme per weight group."""
    out = []
    groups = qc.get("config_groups")
    if not isinstance(groups, dict):
        return out
    for grp in groups.values():
        if not isinstance(grp, dict):
            continue
        fmt = normalize_quant_name(grp.get("format"))
        w = grp.get("weights")
        if fmt == "mxfp4" or (isinstance(w, dict) and "mxfp4" in json.dumps(w).lower()):
            out.append("mxfp4")
            continue
        if not isinstance(w, dict):
            continue
        bits = w.get("num_bits", w.get("bits"))
        kind = str(w.get("type", "")).lower()
        if kind == "float" and bits == 8:
            out.append("fp8-e4m3")
        elif kind in ("int", "integer") and isinstance(bits, int) and bits > 0:
            name = f"int{bits}"
            gs = w.get("group_size")
            if str(w.get("strategy", "")).lower() == "group" and isinstance(gs, int) and gs > 0:
                name += f"-g{gs}"
            out.append(name)
    return out


def _one_config(qc: dict) -> list[str]:
    if "mxfp4" in json.dumps(qc, default=str).lower():
        return ["mxfp4"]
    groups = _group_schemes(qc)
    if groups:
        return groups
    method = normalize_quant_name(qc.get("quant_method") or qc.get("quantization_method"))
    fmt = normalize_quant_name(qc.get("fmt") or qc.get("format") or qc.get("format_name"))
    bits = qc.get("bits", qc.get("num_bits"))
    if method == "fp8" or method == "fp8-e4m3":
        name = "fp8-e4m3" if method == "fp8-e4m3" or fmt in (None, "fp8-e4m3") else f"fp8-{fmt}"
        block = qc.get("weight_block_size")
        if isinstance(block, (list, tuple)) and len(block) == 2 and block[0] == block[1]:
            name += f"-b{int(block[0])}"
        return [name]
    if isinstance(bits, int) and bits > 0:
        return [f"{method}-int{bits}" if method else f"int{bits}"]
    if method and method != "compressed-tensors":
        return [method]
    if fmt and fmt not in ("pack-quantized", "compressed", "float-quantized"):
        return [fmt]
    return []


def quantization_scheme(config: dict) -> str | None:
    """Canonical storage scheme declared by ``config.json`` (top level or
    ``text_config``); None when the checkpoint declares no quantization.  Several
    distinct schemes come back as ``mixed:a+b``."""
    found: list[str] = []
    for owner in (config, config.get("text_config")):
        if isinstance(owner, dict) and isinstance(owner.get("quantization_config"), dict):
            found.extend(_one_config(owner["quantization_config"]))
    uniq = list(dict.fromkeys(found))
    if not uniq:
        return None
    return uniq[0] if len(uniq) == 1 else "mixed:" + "+".join(uniq)


def weight_dtype(config: dict) -> str:
    """Unquantized parameter dtype (``torch_dtype`` / ``dtype``), default bf16."""
    for owner in (config, config.get("text_config")):
        if isinstance(owner, dict):
            v = owner.get("torch_dtype") or owner.get("dtype")
            if v:
                return normalize_quant_name(v) or "bf16"
    return "bf16"


def canonical_scheme(name: str | None) -> str | None:
    """Profile quantization names (``fp8_block128``, a ``quant_method``, a GGUF file type)
    in the canonical spelling of :func:`quantization_scheme`."""
    if name is None or name == "":
        return None
    if isinstance(name, str) and name.startswith("fp8_block"):
        return "fp8-e4m3-b" + name[len("fp8_block"):]
    if isinstance(name, int) or str(name).isdigit():
        return f"gguf-ftype{int(name)}"
    return normalize_quant_name(name)


def b200_kernel_for(scheme: str | None, dtype: str = "bf16") -> tuple[str | None, str]:
    """(kernel, note): the sm_100a GEMM path that executes weights of this scheme, or
    (None, why not)."""
    if scheme is None:
        if dtype in ("bf16", "f16", "f32"):
            note = "native" if dtype == "bf16" else f"{dtype} weights are cast to bf16 at load"
            return "tcgen05 bf16 GEMM (kind::f16, fp32 TMEM accumulator)", note
        return None, f"unquantized dtype {dtype} has no GEMM path"
    if scheme == "fp8-e4m3-b128":
        return ("tcgen05 block-scaled e4m3 GEMM (kind::f8f6f4, 128x128 weight / 1x128 "
                "activation scales)", "native")
    if scheme.startswith("fp8-e4m3"):
        return None, "e4m3 weights without 128x128 block scales need re-quantization to blocks"
    if scheme == "mxfp4":
        return None, "MXFP4 weights have no sm_100a GEMM path here (inspect only)"
    return None, f"{scheme} weights have no sm_100a GEMM path here (inspect only)"


# ----------------------------------------------------------------------------------------
# GGUF variants
# ----------------------------------------------------------------------------------------

_SPLIT = re.compile(r"^(?P<stem>.+)-(?P<part>\d{5})-of-(?P<count>\d{5})\.gguf$", re.I)
_AUX = re.compile(r"(?:^|[-_.])(mmproj|projector|imatrix|tokenizer|vocab)(?:[-_.]|$)", re.I)
_TAG = re.compile(r"(UD-[IQF]\d[A-Z0-9_]*|IQ\d[A-Z0-9_]*|Q\d[A-Z0-9_]*|BF16|F16|F32|FP16|FP32)",
                  re.I)
# approximate bits per weight of the llama.cpp block formats (block bytes x 8 / block size)
_BPW = {"F32": 32.0, "FP32": 32.0, "BF16": 16.0, "F16": 16.0, "FP16": 16.0, "Q8_0": 8.5,
        "Q6_K": 6.5625, "Q5_K": 5.5, "Q5_0": 5.5, "Q5_1": 6.0, "Q4_K": 4.5, "Q4_0": 4.5,
        "Q4_1": 5.0, "Q3_K": 3.4375, "Q2_K": 2.625, "IQ4_XS": 4.25, "IQ4_NL": 4.5,
        "IQ3_XXS": 3.0625, "IQ3_S": 3.4375, "IQ2_XXS": 2.0625, "IQ2_XS": 2.3125, "IQ2_S": 2.5,
        "IQ1_S": 1.5625, "IQ1_M": 1.75}


@dataclass(frozen=True)
class GGUFVariant:
    variant_id: str
    quant: str
    files: tuple[str, ...]
    total_bytes: int
    bits_per_weight: float


@dataclass(frozen=True)
class VariantChoice:
    variant: GGUFVariant
    feasible: bool
    reason: str


@dataclass(frozen=True)
class VariantSelection:
    selected: GGUFVariant
    feasible: bool
    candidates: tuple[VariantChoice, ...]


def _quant_tag(name: str) -> str:
    tags = _TAG.findall(name.upper())
    return tags[-1].upper() if tags else "UNKNOWN"


def bits_per_weight(tag: str) -> float:
    """Estimated bits per weight of a GGUF quantization tag (K-quant size suffixes
    _S/_M/_L/_XL keep more tensors at the next format up, so they add a fraction)."""
    t = tag.upper().removeprefix("UD-")
    if t in _BPW:
        return _BPW[t]
    base = re.match(r"(IQ\d(?:_[A-Z]+)?|Q\d(?:_[A-Z0-9])?)", t)
    if base:
        core = base.group(1)
        for k in (core, core.split("_")[0] + "_K", core.split("_")[0] + "_0"):
            if k in _BPW:
                extra = {"_S": 0.0, "_M": 0.25, "_L": 0.5, "_XL": 0.75}
                sfx = next((v for s, v in extra.items() if t.endswith(s)), 0.0)
                return _BPW[k] + sfx
        m = re.search(r"(\d+)", core)
        if m:
            return float(m.group(1)) + 0.5
    return 0.0


def discover_gguf_variants(files: dict[str, int]) -> tuple[GGUFVariant, ...]:
    """``files`` maps repository-relative paths to byte sizes; returns complete variants."""
    groups: dict[str, dict[int, tuple[str, int]]] = {}
    expect: dict[str, int] = {}
    for path, size in sorted(files.items()):
        name = path.rsplit("/", 1)[-1]
        if not name.lower().endswith(".gguf") or _AUX.search(name):
            continue
        m = _SPLIT.match(name)
        if m:
            stem = path[: len(path) - len(name)] + m.group("stem")
            part, count = int(m.group("part")), int(m.group("count"))
        else:
            stem, part, count = path[:-5], 1, 1
        if expect.setdefault(stem, count) != count:
            expect[stem] = -1                      # contradictory split counts: never complete
        groups.setdefault(stem, {})[part] = (path, size)
    complete = []
    for stem, parts in sorted(groups.items()):
        n = expect[stem]
        if n <= 0 or sorted(parts) != list(range(1, n + 1)):
            continue
        complete.append((stem, _quant_tag(stem.rsplit("/", 1)[-1]), parts))
    per_tag: dict[str, int] = {}
    for _, tag, _ in complete:
        per_tag[tag] = per_tag.get(tag, 0) + 1
    out = []
    for stem, tag, parts in complete:
        vid = tag if tag != "UNKNOWN" and per_tag[tag] == 1 else stem.rsplit("/", 1)[-1]
        ordered = tuple(parts[i][0] for i in sorted(parts))
        out.append(GGUFVariant(vid, tag, ordered, sum(s for _, s in parts.values()),
                               bits_per_weight(tag)))
    return tuple(out)


def select_variant(variants: tuple[GGUFVariant, ...], *, memory_bytes: int,
                   objective: str = "balanced", request: str | None = None,
                   headroom: float = 0.10, kv_share: float = 0.35) -> VariantSelection:
    """Pick one variant.

    A variant fits when its bytes plus ``headroom`` stay within ``memory_bytes``.
    ``capacity`` takes the most bits per weight that fit; ``speed`` the fewest bytes
    among those keeping at least 4 bits per weight (decode streams every weight once
    per token, so bytes set the step time); ``throughput`` and ``balanced`` the most
    bits per weight that still leave ``kv_share`` (throughput: twice that) of the
    memory for the KV cache, falling back to ``capacity``.  An explicit ``request``
    (variant id or tag) is returned even when it does not fit, with
    ``feasible=False``; automatic selection only returns a variant that fits.
    """
    if not variants:
        raise ValueError("no complete GGUF variant")
    if memory_bytes <= 0:
        raise ValueError("memory_bytes must be positive")
    if objective not in ("speed", "throughput", "capacity", "balanced"):
        raise ValueError(f"unknown objective {objective!r}")
    cap = memory_bytes / (1.0 + headroom)
    choices = []
    for v in variants:
        why = []
        if request is not None and request.lower() not in (v.variant_id.lower(), v.quant.lower()):
            why.append("not the requested variant")
        if v.total_bytes > cap:
            why.append(f"needs {v.total_bytes / 1e9:.1f} GB of {cap / 1e9:.1f} GB usable")
        choices.append(VariantChoice(v, not why, "; ".join(why) or "fits"))
    fit = [c.variant for c in choices if c.feasible]
    if request is not None and not fit:
        asked = [c.variant for c in choices if request.lower() in (c.variant.variant_id.lower(),
                                                                   c.variant.quant.lower())]
        if asked:
            best = max(asked, key=lambda v: (v.bits_per_weight, -v.total_bytes))
            return VariantSelection(best, False, tuple(choices))
    if not fit:
        raise ValueError(f"no GGUF variant fits {memory_bytes / 1e9:.1f} GB"
                         + (f" for request {request!r}" if request else ""))
    by_quality = lambda v: (v.bits_per_weight, -v.total_bytes)  # noqa: E731
    if objective == "capacity":
        pick = max(fit, key=by_quality)
    elif objective == "speed":
        good = [v for v in fit if v.bits_per_weight >= 4.0] or fit
        pick = min(good, key=lambda v: (v.total_bytes, -v.bits_per_weight))
    else:
        share = kv_share * (2.0 if objective == "throughput" else 1.0)
        roomy = [v for v in fit if v.total_bytes <= cap * (1.0 - share)]
        pick = max(roomy or fit, key=by_quality)
    return VariantSelection(pick, True, tuple(choices))


# ----------------------------------------------------------------------------------------
# B200 feasibility (headers only)
# ----------------------------------------------------------------------------------------

B200_HBM_BYTES = 183_359 * 2**20          # memory nvidia-smi reports for one B200
GPUS_PER_BOX = 8


def kv_bytes_per_token(cfg) -> int:
    """Cache bytes one token adds over all layers (bf16): K and V rows for GQA, one
    latent row (kv_lora_rank + rope dims) for MLA."""
    if cfg is None:
        return 0
    if cfg.mla:
        return (cfg.kv_lora_rank + cfg.qk_rope_head_dim) * 2 * cfg.num_layers
    return 2 * cfg.num_kv_heads * cfg.head_dim * 2 * cfg.num_layers


def b200_feasibility(resolved, *, batch: int = 32, context: int = 4096,
                     usable_fraction: float = 0.90, gpu_bytes: int = B200_HBM_BYTES) -> dict:
    """Size a resolved checkpoint (see ``model_io.resolver.ResolvedModel``) against B200
    GPUs.  Reads only the tensor inventory already taken from headers."""
    if not 0 < usable_fraction <= 1:
        raise ValueError("usable_fraction must be in (0, 1]")
    prof = resolved.profile
    layer_bytes: dict[int, int] = {}
    expert = non_expert = 0
    largest = ("", 0)
    for name, nb in resolved.tensor_bytes.items():
        d = prof.tensors.get(name)
        if d is not None and d.layer is not None:
            layer_bytes[d.layer] = layer_bytes.get(d.layer, 0) + nb
        if d is not None and d.role.value in ("routed_expert", "shared_expert", "always_on_expert"):
            expert += nb
        else:
            non_expert += nb
        if nb > largest[1]:
            largest = (name, nb)
    total = expert + non_expert
    usable = int(gpu_bytes * usable_fraction)
    kv_tok = kv_bytes_per_token(prof.config)
    kv_total = kv_tok * batch * context
    min_gpus = max(1, math.ceil(total / usable))
    gpus = max(1, math.ceil((total + kv_total) / usable))
    scheme = canonical_scheme(prof.quantization)
    kernel, note = b200_kernel_for(scheme)
    blockers = []
    if resolved.format == "gguf":
        blockers.append("GGUF checkpoints are inspected, not executed, by the sm_100a engine")
    if kernel is None:
        blockers.append(note)
    if not prof.executable:
        blockers.append(f"family {prof.family} has no runtime config for the engine")
    n = 1 << max(0, math.ceil(math.log2(gpus)))          # power-of-two parallel group
    if prof.kind == "moe":
        layout = "tp1" if n == 1 else (f"dp{min(n, GPUS_PER_BOX)}-attention+ep{min(n, GPUS_PER_BOX)}"
                                       if prof.attention == "mla" else f"ep{min(n, GPUS_PER_BOX)}")
    else:
        layout = "tp1" if n == 1 else f"tp{min(n, GPUS_PER_BOX)}"
    if n > GPUS_PER_BOX:
        layout += f"+pp{math.ceil(n / GPUS_PER_BOX)}"
    return {
        "analysis": "headers-only",
        "source": resolved.source, "revision": resolved.revision, "format": resolved.format,
        "family": prof.family, "kind": prof.kind, "attention": prof.attention,
        "quantization": scheme, "b200_kernel": kernel, "kernel_note": note,
        "total_weight_bytes": total, "expert_bytes": expert, "non_expert_bytes": non_expert,
        "largest_tensor": {"name": largest[0], "bytes": largest[1]},
        "largest_layer_bytes": max(layer_bytes.values(), default=0),
        "layer_bytes": {str(k): v for k, v in sorted(layer_bytes.items())},
        "kv_bytes_per_token": kv_tok,
        "kv_bytes_for_target": kv_total, "target": {"batch": batch, "context": context},
        "usable_bytes_per_gpu": usable,
        "min_gpus_weights_only": min_gpus, "gpus_for_target": gpus,
        "boxes_for_target": math.ceil(gpus / GPUS_PER_BOX),
        "layout": layout, "blockers": blockers, "executable": not blockers,
    }


# ----------------------------------------------------------------------------------------
# bounded discovery
# ----------------------------------------------------------------------------------------

def discover_models(references, *, resolver=None, limit: int = 32) -> dict:
    """Inspect at most ``limit`` explicit references (no weight download); one record
    each: PROFILED, INSPECT_ONLY (profile without a runtime path) or FAILED."""
    refs = list(dict.fromkeys(r.strip() for r in references if r and r.strip()))
    if not refs:
        raise ValueError("discovery needs at least one reference")
    if not 1 <= limit <= 64:
        raise ValueError("limit must be in [1, 64]")
    if len(refs) > limit:
        raise ValueError(f"{len(refs)} references exceed the limit of {limit}")
    if resolver is None:
        from .resolver import ModelSourceResolver
        resolver = ModelSourceResolver()
    records = []
    for ref in refs:
        try:
            r = resolver.inspect(ref)
        except (OSError, RuntimeError, ValueError, KeyError) as exc:
            records.append({"reference": ref, "status": "FAILED",
                            "error": f"{type(exc).__name__}: {exc}"})
            continue
        p = r.profile
        records.append({"reference": ref, "status": "PROFILED" if p.executable else "INSPECT_ONLY",
                        "revision": r.revision, "format": r.format, "family": p.family,
                        "kind": p.kind, "attention": p.attention, "quantization": p.quantization,
                        "num_layers": p.num_layers, "num_experts": p.num_experts,
                        "total_bytes": r.total_bytes, "notes": list(p.notes)})
    return {"schema": 1, "inspected": len(records), "records": records}


# ----------------------------------------------------------------------------------------
# model manifest
# ----------------------------------------------------------------------------------------

def sha256_file(path: str | Path, chunk: int = 1 << 20) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(chunk)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def hash_directory(path: str | Path) -> str:
    """SHA-256 over (length-prefixed relative path, file SHA-256) of every file, sorted."""
    root = Path(path)
    h = hashlib.sha256()
    for f in sorted(p for p in root.rglob("*") if p.is_file()):
        rel = f.relative_to(root).as_posix().encode()
        h.update(len(rel).to_bytes(4, "big"))
        h.update(rel)
        h.update(sha256_file(f).encode())
    return h.hexdigest()


def build_manifest(resolved, stages: list[tuple[int, int]], *, model_id: str | None = None,
                   workers: list[str] | None = None, hash_files: bool = True) -> ModelManifest:
    """Manifest of a contiguous stage split of ``resolved``: per-stage weight bytes
    (embedding on stage 0, final norm and head on the last) and shard file hashes."""
    prof = resolved.profile
    defs = []
    for i, (a, b) in enumerate(stages):
        first, last = i == 0, i == len(stages) - 1
        defs.append(StageDefinition(stage_id=i, worker_id=(workers or [f"stage{i}"] * len(stages))[i],
                                    layer_start=a, layer_end=b, embed=first, head=last,
                                    weight_bytes=resolved.stage_bytes(a, b, embed=first, head=last)))
    m = ModelManifest(model_id=model_id or resolved.source, revision=resolved.revision,
                      family=prof.family, num_layers=prof.num_layers, stages=defs,
                      total_weight_bytes=resolved.total_bytes)
    m.check_union()                       # before hashing: a bad split fails fast
    if hash_files:
        for f in sorted(resolved.files):
            p = resolved.path / f if resolved.path.is_dir() else resolved.path
            m.shard_hashes[f] = hash_directory(p) if p.is_dir() else sha256_file(p)
    return m


def save_manifest(m: ModelManifest, path: str | Path) -> Path:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    tmp = p.with_suffix(p.suffix + ".tmp")
    tmp.write_text(m.model_dump_json(indent=2) + "\n", encoding="utf-8")
    tmp.replace(p)
    return p


def load_manifest(path: str | Path) -> ModelManifest:
    try:
        return ModelManifest.model_validate_json(Path(path).read_text(encoding="utf-8"))
    except (OSError, ValueError) as exc:
        raise ConfigError(f"invalid model manifest {path}: {exc}") from None


def verify_manifest_shards(m: ModelManifest, root: str | Path) -> None:
    """Raise ``ConfigError`` on a missing shard or a hash mismatch."""
    base = Path(root)
    for rel, want in sorted(m.shard_hashes.items()):
        p = base / rel if base.is_dir() else base
        if p.is_file():
            got = sha256_file(p)
        elif p.is_dir():
            got = hash_directory(p)
        else:
            raise ConfigError(f"manifest shard {rel} is missing under {base}")
        if got != want:
            raise ConfigError(f"shard {rel}: sha256 {got} != manifest {want}")


def manifest_summary(m: ModelManifest) -> dict:
    return {"model_id": m.model_id, "revision": m.revision, "family": m.family,
            "num_layers": m.num_layers, "stages": len(m.stages),
            "stage_layers": [[s.layer_start, s.layer_end] for s in m.stages],
            "stage_weight_bytes": [s.weight_bytes for s in m.stages],
            "largest_stage_bytes": max((s.weight_bytes for s in m.stages), default=0),
            "total_weight_bytes": m.total_weight_bytes, "shards": dict(m.shard_hashes)}


__all__ = ["normalize_quant_name", "quantization_scheme", "canonical_scheme", "weight_dtype", "b200_kernel_for",
           "GGUFVariant", "VariantChoice", "VariantSelection", "bits_per_weight",
           "discover_gguf_variants", "select_variant", "kv_bytes_per_token", "b200_feasibility",
           "discover_models", "sha256_file", "hash_directory", "build_manifest", "save_manifest",
           "load_manifest", "verify_manifest_shards", "manifest_summary", "B200_HBM_BYTES"]
