"""Metadata-driven architecture profiles and the family registry.

An :class:`ArchitectureProfile` is derived from checkpoint metadata
(``config.json`` or GGUF ``general.architecture``), never from a repository
name.  It records the family, dense/MoE kind, attention kind (GQA or MLA),
routing, quantisation, and a role for every tensor (embedding, attention,
router, routed/shared expert, norms, head, ...) together with the shard
semantics the planner and the stage artifact builder need: which axis a
tensor-parallel shard cuts and how partial results recombine.

Families are registered as :class:`FamilySpec` entries; third parties can
add more through the ``swarm_inference_lab_b200.families`` entry point
group without touching the resolver, planner or engines.

Reference: si/model/architecture.py:34-357 (TensorRole, ShardReduction,
TensorShardSemantics, ModelArchitectureProfile) and
si/model/architecture_adapters.py:76-976 (family specs, metadata helpers).
The role and reduction names are kept identical so profiles compare across
the two implementations.
"""
from __future__ import annotations

import enum
import re
from dataclasses import asdict, dataclass, field
from importlib import metadata as importlib_metadata
from typing import Callable

from ..models.config import ModelConfig, from_hf_config


class TensorRole(str, enum.Enum):
    EMBEDDING = "embedding"
    ATTENTION = "attention"
    ATTENTION_NORM = "attention_norm"
    DENSE_MLP = "dense_mlp"
    ROUTER = "router"
    ROUTED_EXPERT = "routed_expert"
    SHARED_EXPERT = "shared_expert"
    ALWAYS_ON_EXPERT = "always_on_expert"
    FINAL_NORM = "final_norm"
    OUTPUT_HEAD = "output_head"
    POSITIONAL = "positional"
    MULTIMODAL = "multimodal"
    AUXILIARY = "auxiliary"
    UNKNOWN = "unknown"


class ShardReduction(str, enum.Enum):
    CONCATENATE = "concatenate"
    SUM = "sum"
    ALL_REDUCE_SUM = "all_reduce_sum"
    GATHER = "gather"
    NONE = "none"


@dataclass(frozen=True)
class ShardSemantics:
    role: TensorRole
    shard_axis: int | None          # axis a tensor-parallel shard cuts (None: replicated)
    reduction: ShardReduction
    alignment: int = 1


@dataclass(frozen=True)
class TensorDescriptor:
    name: str
    role: TensorRole
    layer: int | None
    expert: int | None
    semantics: ShardSemantics


@dataclass(frozen=True)
class ExpertDescriptor:
    layer: int
    expert: int
    tensors: tuple[str, ...]
    shared: bool = False


@dataclass
class ArchitectureProfile:
    family: str
    source: str
    kind: str                        # dense | moe
    attention: str                   # gqa | mla
    routing: str | None              # softmax | sigmoid_group | None
    quantization: str | None
    num_layers: int
    hidden_size: int
    num_experts: int = 0
    experts_per_token: int = 0
    config: ModelConfig | None = None
    tensors: dict[str, TensorDescriptor] = field(default_factory=dict)
    experts: list[ExpertDescriptor] = field(default_factory=list)
    executable: bool = True
    notes: tuple[str, ...] = ()

    def layer_tensors(self, layer: int) -> list[str]:
        return [t.name for t in self.tensors.values() if t.layer == layer]

    def summary(self) -> dict:
        d = {k: v for k, v in asdict(self).items() if k not in ("tensors", "experts", "config")}
        d["tensor_count"] = len(self.tensors)
        d["expert_count"] = len(self.experts)
        roles: dict[str, int] = {}
        for t in self.tensors.values():
            roles[t.role.value] = roles.get(t.role.value, 0) + 1
        d["roles"] = roles
        return d


# ----------------------------------------------------------------- tensor roles
_LAYER = re.compile(r"(?:^|\.)layers\.(\d+)\.")
_EXPERT = re.compile(r"\.experts\.(\d+)\.")
_COL = ShardSemantics(TensorRole.ATTENTION, 0, ShardReduction.CONCATENATE)

# (pattern, role, shard axis, reduction) - first match wins.
_RULES: list[tuple[str, TensorRole, int | None, ShardReduction]] = [
    (r"embed_tokens|tok_embeddings|wte|token_embd", TensorRole.EMBEDDING, None, ShardReduction.NONE),
    (r"(^|\.)(model\.)?norm\.weight$|final_layernorm|output_norm", TensorRole.FINAL_NORM, None, ShardReduction.NONE),
    (r"lm_head|(^|\.)output\.weight", TensorRole.OUTPUT_HEAD, 0, ShardReduction.GATHER),
    (r"(input_layernorm|post_attention_layernorm|attn_norm|ffn_norm|q_norm|k_norm|"
     r"q_a_layernorm|kv_a_layernorm)", TensorRole.ATTENTION_NORM, None, ShardReduction.NONE),
    (r"mlp\.gate\.(weight|e_score_correction_bias)|block_sparse_moe\.gate\.|ffn_gate_inp",
     TensorRole.ROUTER, None, ShardReduction.NONE),
    (r"shared_expert", TensorRole.SHARED_EXPERT, 0, ShardReduction.ALL_REDUCE_SUM),
    (r"\.experts\.\d+\.|_exps\.", TensorRole.ROUTED_EXPERT, None, ShardReduction.SUM),
    (r"(o_proj|wo|attn_output)", TensorRole.ATTENTION, 1, ShardReduction.ALL_REDUCE_SUM),
    (r"(q_proj|k_proj|v_proj|q_a_proj|q_b_proj|kv_a_proj|kv_b_proj|wq|wk|wv|attn_q|attn_k|attn_v)",
     TensorRole.ATTENTION, 0, ShardReduction.CONCATENATE),
    (r"(down_proj|w2|ffn_down)", TensorRole.DENSE_MLP, 1, ShardReduction.ALL_REDUCE_SUM),
    (r"(gate_proj|up_proj|w1|w3|ffn_gate|ffn_up)", TensorRole.DENSE_MLP, 0, ShardReduction.CONCATENATE),
    (r"rotary|rope", TensorRole.POSITIONAL, None, ShardReduction.NONE),
    (r"vision|visual|mm_projector|image", TensorRole.MULTIMODAL, None, ShardReduction.NONE),
]
_RULES_C = [(re.compile(p), r, a, red) for p, r, a, red in _RULES]


def classify_tensor(name: str) -> TensorDescriptor:
    lm = _LAYER.search(name)
    em = _EXPERT.search(name)
    layer = int(lm.group(1)) if lm else None
    expert = int(em.group(1)) if em else None
    for pat, role, axis, red in _RULES_C:
        if pat.search(name):
            return TensorDescriptor(name, role, layer, expert, ShardSemantics(role, axis, red))
    return TensorDescriptor(name, TensorRole.UNKNOWN, layer, expert,
                            ShardSemantics(TensorRole.UNKNOWN, None, ShardReduction.NONE))


# ----------------------------------------------------------------- families
@dataclass(frozen=True)
class FamilySpec:
    name: str
    model_types: tuple[str, ...]
    kind: str
    attention: str = "gqa"
    routing: str | None = None
    executable: bool = True
    notes: tuple[str, ...] = ()


BUILTIN_FAMILIES = (
    FamilySpec("llama", ("llama",), "dense"),
    FamilySpec("mistral", ("mistral",), "dense"),
    FamilySpec("qwen3", ("qwen3",), "dense"),
    FamilySpec("qwen3_moe", ("qwen3_moe",), "moe", routing="softmax"),
    FamilySpec("mixtral", ("mixtral",), "moe", routing="softmax"),
    FamilySpec("deepseek_v3", ("deepseek_v3", "kimi_k2"), "moe", attention="mla",
               routing="sigmoid_group"),
    FamilySpec("qwen3_5", ("qwen3_5", "qwen3_next"), "dense", executable=False,
               notes=("hybrid linear attention layers are not implemented",)),
    FamilySpec("qwen3_5_moe", ("qwen3_5_moe",), "moe", routing="softmax", executable=False,
               notes=("hybrid linear attention layers are not implemented",)),
    FamilySpec("gemma", ("gemma", "gemma2", "gemma3"), "dense", executable=False,
               notes=("soft-capping / sliding-window layers are not implemented",)),
    FamilySpec("llama4", ("llama4",), "moe", routing="sigmoid_group", executable=False),
    FamilySpec("glm_moe", ("glm4_moe",), "moe", routing="sigmoid_group", executable=False),
    FamilySpec("minimax", ("minimax", "minimax_m1"), "moe", executable=False),
    FamilySpec("kimi_k3", ("kimi_k3",), "moe", attention="mla", routing="sigmoid_group",
               executable=False, notes=("MXFP4 experts are described, not executed",)),
)


class ArchitectureRegistry:
    def __init__(self, specs=BUILTIN_FAMILIES, load_entry_points: bool = True):
        self.by_type: dict[str, FamilySpec] = {}
        for s in specs:
            self.register(s)
        if load_entry_points:
            try:
                for ep in importlib_metadata.entry_points(group="swarm_inference_lab_b200.families"):
                    obj = ep.load()
                    for s in (obj() if callable(obj) else obj):
                        self.register(s)
            except Exception:  # noqa: BLE001 - a broken plugin must not break resolution
                pass

    def register(self, spec: FamilySpec) -> None:
        for t in spec.model_types:
            self.by_type[t] = spec

    def resolve_config(self, cfg: dict, tensor_names: list[str] | None = None) -> ArchitectureProfile:
        mt = cfg.get("model_type")
        source = "config.model_type"
        if mt is None and isinstance(cfg.get("text_config"), dict):
            mt = cfg["text_config"].get("model_type")
            source = "config.text_config.model_type"
        if mt is None and cfg.get("architectures"):
            arch = cfg["architectures"][0].lower()
            source = "config.architectures"
            mt = next((t for t in self.by_type if arch.startswith(t.replace("_", ""))), None)
        spec = self.by_type.get(mt or "")
        if spec is None:
            raise KeyError(f"no architecture family for model_type {mt!r}")
        qc = cfg.get("quantization_config") or {}
        quant = qc.get("quant_method")
        if quant == "fp8" and qc.get("weight_block_size"):
            quant = f"fp8_block{qc['weight_block_size'][0]}"
        mc = None
        notes = list(spec.notes)
        try:
            mc = from_hf_config(cfg)
        except (KeyError, ValueError) as exc:
            notes.append(f"runtime config unavailable: {exc}")
        prof = ArchitectureProfile(
            family=spec.name, source=source, kind=spec.kind, attention=spec.attention,
            routing=spec.routing, quantization=quant,
            num_layers=int(cfg.get("num_hidden_layers", 0)), hidden_size=int(cfg.get("hidden_size", 0)),
            num_experts=int(cfg.get("num_experts") or cfg.get("num_local_experts")
                            or cfg.get("n_routed_experts") or 0),
            experts_per_token=int(cfg.get("num_experts_per_tok") or 0), config=mc,
            executable=spec.executable and mc is not None, notes=tuple(notes))
        if tensor_names:
            self.attach_tensors(prof, tensor_names)
        return prof

    def resolve_gguf(self, meta: dict, tensor_names: list[str]) -> ArchitectureProfile:
        arch = meta.get("general.architecture", "")
        spec = self.by_type.get(arch) or self.by_type.get({"qwen3moe": "qwen3_moe",
                                                            "deepseek2": "deepseek_v3"}.get(arch, ""))
        if spec is None:
            raise KeyError(f"no architecture family for GGUF architecture {arch!r}")
        p = arch + "."
        prof = ArchitectureProfile(
            family=spec.name, source="gguf.general.architecture", kind=spec.kind,
            attention=spec.attention, routing=spec.routing, quantization=meta.get("general.file_type"),
            num_layers=int(meta.get(p + "block_count", 0)), hidden_size=int(meta.get(p + "embedding_length", 0)),
            num_experts=int(meta.get(p + "expert_count", 0)),
            experts_per_token=int(meta.get(p + "expert_used_count", 0)), executable=False,
            notes=("GGUF checkpoints are inspected, not executed, by the sm_100a engine",))
        self.attach_tensors(prof, tensor_names)
        return prof

    @staticmethod
    def attach_tensors(prof: ArchitectureProfile, names: list[str]) -> None:
        experts: dict[tuple[int, int], list[str]] = {}
        for n in names:
            d = classify_tensor(n)
            prof.tensors[n] = d
            if d.role == TensorRole.ROUTED_EXPERT and d.layer is not None and d.expert is not None:
                experts.setdefault((d.layer, d.expert), []).append(n)
        prof.experts = [ExpertDescriptor(l, e, tuple(sorted(v))) for (l, e), v in sorted(experts.items())]


_default: ArchitectureRegistry | None = None


def default_registry() -> ArchitectureRegistry:
    global _default
    if _default is None:
        _default = ArchitectureRegistry()
    return _default


Resolver = Callable[[dict], ArchitectureProfile]
