"""Checkpoint loading: Hugging Face safetensors directories -> the runtime's weights.

    cfg = checkpoint_config(path)                 # config.json -> ModelConfig
    get = safetensors_source(path)                # get(name, shape) in canonical names
    weights = load_weights(cfg, path, tp, device) # DenseWeights | MoEWeights | MLAWeights
    tok = load_tokenizer(path)                    # the checkpoint's tokenizer, if it has one

Canonical names are the Hugging Face Llama / Qwen3 / Qwen3-MoE / DeepSeek-V3 names
(``model.layers.{i}.self_attn.q_proj.weight``, ``...mlp.experts.{e}.gate_proj.weight``
...).  Other families are mapped onto them: Mixtral's ``block_sparse_moe.gate`` and
``experts.{e}.w1 / w3 / w2`` become ``mlp.gate`` and the experts' gate / up / down.
Tensors are read lazily, one at a time, from the shard that holds them (the index file's
weight map, else every ``*.safetensors`` file's header).  fp8 e4m3 tensors with a
``weight_scale_inv`` sibling (DeepSeek-V3 / Kimi-K2, 128x128 blocks) are dequantised for
the bf16 paths and passed through as (codes, scales) for the fp8 kernels.

Reference: si/model/qwen3.py:2413 (``load_weights``), si/model/qwen3_moe.py:28-297
(Qwen3-MoE tensor names and expert stacking), si/model/quantization.py (fp8 block scales).
"""
from __future__ import annotations

import json
import os
import re
from pathlib import Path

import torch

from ..models.config import ModelConfig, eos_ids, from_hf_config


class CheckpointError(RuntimeError):
    pass


def checkpoint_config(path: str | Path) -> ModelConfig:
    p = Path(path)
    cfg_file = p / "config.json"
    if not cfg_file.is_file():
        raise CheckpointError(f"{p}: no config.json")
    raw = json.loads(cfg_file.read_text())
    cfg = from_hf_config(raw)
    gen = p / "generation_config.json"          # what `generate` stops on takes precedence
    if gen.is_file():
        g = json.loads(gen.read_text())
        if g.get("eos_token_id") is not None:
            cfg = cfg.replace(eos_token_ids=eos_ids(g["eos_token_id"]))
    return cfg.replace(name=p.name)


_MIXTRAL = [
    (re.compile(r"^(model\.layers\.\d+\.)mlp\.gate\.weight$"), r"\1block_sparse_moe.gate.weight"),
    (re.compile(r"^(model\.layers\.\d+\.)mlp\.experts\.(\d+)\.gate_proj\.weight$"),
     r"\1block_sparse_moe.experts.\2.w1.weight"),
    (re.compile(r"^(model\.layers\.\d+\.)mlp\.experts\.(\d+)\.up_proj\.weight$"),
     r"\1block_sparse_moe.experts.\2.w3.weight"),
    (re.compile(r"^(model\.layers\.\d+\.)mlp\.experts\.(\d+)\.down_proj\.weight$"),
     r"\1block_sparse_moe.experts.\2.w2.weight"),
]


def checkpoint_name(family: str, canonical: str) -> str:
    """The checkpoint's tensor name for a canonical (Llama / Qwen3 / DeepSeek) name."""
    if family == "mixtral":
        for pat, rep in _MIXTRAL:
            if pat.match(canonical):
                return pat.sub(rep, canonical)
    return canonical


class SafetensorsIndex:
    """Lazy access to the tensors of a safetensors checkpoint directory."""

    def __init__(self, path: str | Path):
        from safetensors import safe_open
        self.root = Path(path)
        self._safe_open = safe_open
        idx = self.root / "model.safetensors.index.json"
        self.where: dict[str, str] = {}
        if idx.is_file():
            self.where = dict(json.loads(idx.read_text())["weight_map"])
        else:
            files = sorted(f for f in os.listdir(self.root) if f.endswith(".safetensors"))
            if not files:
                raise CheckpointError(f"{self.root}: no *.safetensors files")
            for f in files:
                with safe_open(str(self.root / f), framework="pt") as h:
                    for k in h.keys():
                        self.where[k] = f
        self._open: dict[str, object] = {}

    def __contains__(self, name: str) -> bool:
        return name in self.where

    def get(self, name: str) -> torch.Tensor:
        f = self.where.get(name)
        if f is None:
            raise CheckpointError(f"tensor {name} not in the checkpoint")
        h = self._open.get(f)
        if h is None:
            h = self._safe_open(str(self.root / f), framework="pt")
            self._open[f] = h
        return h.get_tensor(name)

    def meta(self, name: str) -> tuple[str, tuple[int, ...]]:
        """(dtype string, shape) of a tensor from the file header, without reading its data."""
        f = self.where.get(name)
        if f is None:
            raise CheckpointError(f"tensor {name} not in the checkpoint")
        h = self._open.get(f)
        if h is None:
            h = self._safe_open(str(self.root / f), framework="pt")
            self._open[f] = h
        sl = h.get_slice(name)
        return str(sl.get_dtype()), tuple(int(x) for x in sl.get_shape())

    def close(self) -> None:
        self._open.clear()


def _scale_name(name: str) -> str:
    return name + "_scale_inv" if name.endswith(".weight") else name + ".weight_scale_inv"


def dequantize_block_fp8(codes: torch.Tensor, scale_inv: torch.Tensor, block: int = 128) -> torch.Tensor:
    """fp32 weight from e4m3 codes [N, K] and per-block multipliers [ceil(N/b), ceil(K/b)]."""
    N, K = codes.shape
    w = codes.view(torch.float8_e4m3fn).float() if codes.dtype == torch.uint8 else codes.float()
    s = scale_inv.float().repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return w * s


def safetensors_source(path: str | Path, *, family: str | None = None):
    """``get(name, shape, dtype=None)`` over a checkpoint (fp32 unless ``dtype`` is given),
    in canonical names; fp8 block-scaled tensors come back dequantised."""
    idx = SafetensorsIndex(path)
    fam = family or checkpoint_config(path).family
    tie = False
    try:
        tie = bool(json.loads((Path(path) / "config.json").read_text()).get("tie_word_embeddings"))
    except Exception:  # noqa: BLE001
        pass

    def get(name, shape, dtype=None):
        real = checkpoint_name(fam, name)
        if real not in idx and name == "lm_head.weight" and tie:
            real = "model.embed_tokens.weight"
        t = idx.get(real)
        if t.dtype in (torch.float8_e4m3fn, torch.uint8) and _scale_name(real) in idx:
            t = dequantize_block_fp8(t, idx.get(_scale_name(real)))
        if tuple(t.shape) != tuple(shape):
            raise CheckpointError(f"{real}: shape {tuple(t.shape)}, expected {tuple(shape)}")
        return t.to(dtype or torch.float32)

    get.index = idx
    get.family = fam
    return get


def fp8_source(get):
    """``fp8w(name, shape)`` for the MLA / fp8 models: the checkpoint's e4m3 codes and
    128x128 scales when the tensor is stored that way, else quantised here."""
    from ..ops import fp8
    idx = get.index

    def fp8w(name, shape):
        real = checkpoint_name(get.family, name)
        t = idx.get(real)
        if t.dtype in (torch.float8_e4m3fn, torch.uint8) and _scale_name(real) in idx:
            if tuple(t.shape) != tuple(shape):
                raise CheckpointError(f"{real}: shape {tuple(t.shape)}, expected {tuple(shape)}")
            codes = t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t
            return codes.contiguous(), idx.get(_scale_name(real)).float().contiguous()
        w = get(name, shape)
        N = w.shape[0]
        pad = (-N) % 128
        if pad:
            w = torch.cat([w, torch.zeros(pad, w.shape[1], dtype=w.dtype)])
        q, s = fp8.quantize_weight(w.cuda() if torch.cuda.is_available() else w)
        return q[:N].contiguous(), s.contiguous()

    return fp8w


def load_weights(cfg: ModelConfig, path: str | Path, tp=None, device="cuda", *,
                 dtype=torch.bfloat16):
    """This rank's weights of a checkpoint, in the layout the sm_100a models use."""
    from ..models.dense import DenseWeights, TPInfo
    tp = tp or TPInfo()
    get = safetensors_source(path, family=cfg.family)
    if cfg.mla:
        from ..models.deepseek import MLAWeights
        dev = torch.device(device)

        def getd(name, shape, dt=torch.bfloat16):
            return get(name, shape).to(device=dev, dtype=dt)

        def fp8d(name, shape):
            q, s = fp8_source(get)(name, shape)
            return q.to(dev), s.to(dev)
        return MLAWeights.from_source(cfg, tp, getd, fp8d, dev)
    if cfg.is_moe:
        from ..models.moe import MoEWeights
        return MoEWeights.from_full(cfg, tp, get, device, dtype)
    return DenseWeights.from_full(cfg, tp, get, device, dtype)


def validate_checkpoint(path: str | Path) -> dict:
    """Header-only check of a checkpoint against its config: the model's weight builder runs on
    the ``meta`` device with a source that looks up every tensor it asks for (canonical name
    mapped to the checkpoint's) and compares the header shape with the shape the config
    implies; no tensor data is read.  Returns the problems found (missing tensors, shape
    mismatches) and the checkpoint tensors no layer used."""
    from ..models.dense import DenseWeights, TPInfo
    cfg = checkpoint_config(path)
    idx = SafetensorsIndex(path)
    fam = cfg.family
    tie = False
    try:
        tie = bool(json.loads((Path(path) / "config.json").read_text()).get("tie_word_embeddings"))
    except Exception:  # noqa: BLE001
        pass
    problems: list[str] = []
    used: set[str] = set()

    def resolve(name):
        real = checkpoint_name(fam, name)
        if real not in idx and name == "lm_head.weight" and tie:
            real = "model.embed_tokens.weight"
        return real

    def check(name, shape):
        real = resolve(name)
        if real not in idx:
            problems.append(f"missing {real}")
            return
        used.add(real)
        if _scale_name(real) in idx:
            used.add(_scale_name(real))
        _, sh = idx.meta(real)
        if sh != tuple(shape):
            problems.append(f"{real}: shape {sh}, expected {tuple(shape)}")

    def get(name, shape, dtype=None):
        check(name, shape)
        return torch.empty(tuple(shape), dtype=dtype or torch.float32, device="meta")

    get.index = idx
    get.family = fam
    try:
        if cfg.mla:
            from ..models.deepseek import MLAWeights

            def getd(name, shape, dt=torch.bfloat16):
                return get(name, shape, dt)

            def fp8d(name, shape):
                check(name, shape)
                rows = -(-shape[0] // 128) * 128
                return (torch.empty((rows, shape[1]), dtype=torch.uint8, device="meta"),
                        torch.empty((rows // 128, -(-shape[1] // 128)), device="meta"))
            MLAWeights.from_source(cfg, TPInfo(), getd, fp8d, torch.device("meta"))
        elif cfg.is_moe:
            from ..models.moe import MoEWeights
            MoEWeights.from_full(cfg, TPInfo(), get, "meta", torch.bfloat16)
        else:
            DenseWeights.from_full(cfg, TPInfo(), get, "meta", torch.bfloat16)
    finally:
        idx.close()
    unused = sorted(n for n in idx.where if n not in used)
    return {"family": fam, "layers": cfg.num_layers, "ok": not problems,
            "problems": problems[:50], "tensors_checked": len(used), "unused": unused[:50]}


def load_tokenizer(path: str | Path):
    """The checkpoint's tokenizer (``transformers.AutoTokenizer``), or None when the
    directory carries no tokenizer files."""
    p = Path(path)
    if not any((p / f).exists() for f in ("tokenizer.json", "tokenizer.model",
                                            "tokenizer_config.json", "vocab.json")):
        return None
    try:
        from transformers import AutoTokenizer
        return AutoTokenizer.from_pretrained(str(p), local_files_only=True)
    except Exception:  # noqa: BLE001 - an unreadable tokenizer is reported as absent
        return None
