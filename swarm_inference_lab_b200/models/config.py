"""Model configurations for the supported decoder families.

One dataclass covers the three shapes the runtime executes:

* dense GQA decoders (Llama, Mistral, Qwen3 with per-head q/k RMSNorm),
* softmax-routed MoE decoders (Mixtral, Qwen3-MoE),
* MLA + sigmoid-routed MoE decoders (DeepSeek-V3 / Kimi-K2, fp8 block-scaled).

``from_hf_config`` maps a Hugging Face ``config.json`` dictionary onto it
(the metadata-driven family mapping of the reference,
si/model/architecture_adapters.py:735-976).  Named presets reproduce the
benchmark shapes with random initialisation.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field
from typing import Any


@dataclass(frozen=True)
class ModelConfig:
    name: str
    family: str                       # llama | qwen3 | mistral | mixtral | qwen3_moe | deepseek_v3
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int            # dense FFN width
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_scaling: dict | None = None
    qk_norm: bool = False             # Qwen3 per-head q/k RMSNorm
    tie_word_embeddings: bool = False
    max_position_embeddings: int = 8192
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    router: str = "softmax"           # softmax | sigmoid_group
    n_group: int = 1
    topk_group: int = 1
    routed_scaling_factor: float = 1.0
    n_shared_experts: int = 0
    first_k_dense: int = 0            # leading dense layers (DeepSeek/Kimi)
    # MLA (DeepSeek-V3 / Kimi-K2)
    mla: bool = False
    q_lora_rank: int = 0
    kv_lora_rank: int = 0
    qk_nope_head_dim: int = 0
    qk_rope_head_dim: int = 0
    v_head_dim: int = 0
    # weights
    weight_dtype: str = "bf16"        # bf16 | fp8_block128
    # generation stops after emitting one of these (the checkpoint's eos_token_id)
    eos_token_ids: tuple[int, ...] = ()
    extra: dict = field(default_factory=dict)

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def replace(self, **kw: Any) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    def parameter_count(self) -> int:
        H, L, V = self.hidden_size, self.num_layers, self.vocab_size
        emb = V * H * (1 if self.tie_word_embeddings else 2)
        if self.mla:
            qk = self.qk_nope_head_dim + self.qk_rope_head_dim
            attn = (H * self.q_lora_rank + self.q_lora_rank * self.num_heads * qk
                    + H * (self.kv_lora_rank + self.qk_rope_head_dim)
                    + self.kv_lora_rank * self.num_heads * (self.qk_nope_head_dim + self.v_head_dim)
                    + self.num_heads * self.v_head_dim * H)
        else:
            attn = H * (self.q_size + 2 * self.kv_size) + self.q_size * H
        dense_ffn = 3 * H * self.intermediate_size
        if self.is_moe:
            moe = 3 * H * self.moe_intermediate_size * (self.num_experts + self.n_shared_experts)
            moe += H * self.num_experts
            n_dense = self.first_k_dense
            ffn = n_dense * dense_ffn + (L - n_dense) * moe
        else:
            ffn = L * dense_ffn
        return emb + L * attn + ffn

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)


def eos_ids(value) -> tuple[int, ...]:
    """``eos_token_id`` of a Hugging Face config (an int, a list of ints or absent)."""
    if value is None:
        return ()
    if isinstance(value, (list, tuple)):
        return tuple(sorted({int(v) for v in value}))
    return (int(value),)


def from_hf_config(cfg: dict) -> ModelConfig:
    """Build a :class:`ModelConfig` from a Hugging Face ``config.json`` dictionary."""
    mt = cfg.get("model_type", "llama")
    H = int(cfg["hidden_size"])
    nh = int(cfg["num_attention_heads"])
    hd = int(cfg.get("head_dim") or H // nh)
    common = dict(
        name=cfg.get("_name_or_path", mt) or mt,
        vocab_size=int(cfg["vocab_size"]),
        hidden_size=H,
        num_layers=int(cfg["num_hidden_layers"]),
        num_heads=nh,
        num_kv_heads=int(cfg.get("num_key_value_heads", nh)),
        head_dim=hd,
        intermediate_size=int(cfg.get("intermediate_size", 4 * H)),
        rms_norm_eps=float(cfg.get("rms_norm_eps", 1e-6)),
        rope_theta=float(cfg.get("rope_theta", 10000.0)),
        rope_scaling=cfg.get("rope_scaling"),
        tie_word_embeddings=bool(cfg.get("tie_word_embeddings", False)),
        max_position_embeddings=int(cfg.get("max_position_embeddings", 8192)),
        eos_token_ids=eos_ids(cfg.get("eos_token_id")),
    )
    if mt in ("llama", "mistral"):
        return ModelConfig(family=mt, **common)
    if mt == "qwen3":
        return ModelConfig(family="qwen3", qk_norm=True, **common)
    if mt == "mixtral":
        return ModelConfig(family="mixtral", num_experts=int(cfg["num_local_experts"]),
                           num_experts_per_tok=int(cfg["num_experts_per_tok"]),
                           moe_intermediate_size=int(cfg["intermediate_size"]),
                           norm_topk_prob=True, **common)
    if mt == "qwen3_moe":
        if int(cfg.get("decoder_sparse_step", 1)) != 1 or cfg.get("mlp_only_layers"):
            raise ValueError("qwen3_moe with dense interleaved layers is not supported")
        n_exp = cfg.get("num_experts", cfg.get("num_local_experts"))
        return ModelConfig(family="qwen3_moe", qk_norm=True, num_experts=int(n_exp),
                           num_experts_per_tok=int(cfg["num_experts_per_tok"]),
                           moe_intermediate_size=int(cfg["moe_intermediate_size"]),
                           norm_topk_prob=bool(cfg.get("norm_topk_prob", True)), **common)
    if mt in ("deepseek_v3", "kimi_k2"):
        common["head_dim"] = int(cfg["qk_nope_head_dim"]) + int(cfg["qk_rope_head_dim"])
        qc = cfg.get("quantization_config") or {}
        return ModelConfig(
            family="deepseek_v3", num_experts=int(cfg["n_routed_experts"]),
            num_experts_per_tok=int(cfg["num_experts_per_tok"]),
            moe_intermediate_size=int(cfg["moe_intermediate_size"]),
            norm_topk_prob=bool(cfg.get("norm_topk_prob", True)), router="sigmoid_group",
            n_group=int(cfg.get("n_group", 1)), topk_group=int(cfg.get("topk_group", 1)),
            routed_scaling_factor=float(cfg.get("routed_scaling_factor", 1.0)),
            n_shared_experts=int(cfg.get("n_shared_experts", 0)),
            first_k_dense=int(cfg.get("first_k_dense_replace", 0)), mla=True,
            q_lora_rank=int(cfg.get("q_lora_rank") or 0), kv_lora_rank=int(cfg["kv_lora_rank"]),
            qk_nope_head_dim=int(cfg["qk_nope_head_dim"]),
            qk_rope_head_dim=int(cfg["qk_rope_head_dim"]), v_head_dim=int(cfg["v_head_dim"]),
            weight_dtype="fp8_block128" if qc.get("quant_method") == "fp8" else "bf16",
            **common)
    raise ValueError(f"unsupported model_type {mt!r}")


# ---------------------------------------------------------------- presets
LLAMA3_8B = ModelConfig(
    name="llama-3-8b-shape", family="llama", vocab_size=128256, hidden_size=4096, num_layers=32,
    num_heads=32, num_kv_heads=8, head_dim=128, intermediate_size=14336, rms_norm_eps=1e-5,
    rope_theta=500000.0, max_position_embeddings=8192)

TINY_LLAMA_CPU = ModelConfig(
    name="tiny-llama-cpu", family="llama", vocab_size=32000, hidden_size=256, num_layers=4,
    num_heads=4, num_kv_heads=2, head_dim=64, intermediate_size=688, rms_norm_eps=1e-5,
    rope_theta=10000.0, max_position_embeddings=2048)

# Smallest dense shape the GPU kernels accept (head_dim 128, dims multiple of 128).
TINY_LLAMA_GPU = ModelConfig(
    name="tiny-llama-gpu", family="llama", vocab_size=4096, hidden_size=512, num_layers=2,
    num_heads=4, num_kv_heads=2, head_dim=128, intermediate_size=1024, rms_norm_eps=1e-5,
    rope_theta=10000.0, max_position_embeddings=4096)

QWEN3_0_6B = ModelConfig(
    name="qwen3-0.6b-shape", family="qwen3", vocab_size=151936, hidden_size=1024, num_layers=28,
    num_heads=16, num_kv_heads=8, head_dim=128, intermediate_size=3072, rms_norm_eps=1e-6,
    rope_theta=1000000.0, qk_norm=True, tie_word_embeddings=True, max_position_embeddings=40960)

MIXTRAL_8X7B = ModelConfig(
    name="mixtral-8x7b-shape", family="mixtral", vocab_size=32000, hidden_size=4096, num_layers=32,
    num_heads=32, num_kv_heads=8, head_dim=128, intermediate_size=14336, rms_norm_eps=1e-5,
    rope_theta=1000000.0, num_experts=8, num_experts_per_tok=2, moe_intermediate_size=14336)

QWEN3_30B_A3B = ModelConfig(
    name="qwen3-30b-a3b-shape", family="qwen3_moe", vocab_size=151936, hidden_size=2048,
    num_layers=48, num_heads=32, num_kv_heads=4, head_dim=128, intermediate_size=6144,
    rms_norm_eps=1e-6, rope_theta=1000000.0, qk_norm=True, num_experts=128,
    num_experts_per_tok=8, moe_intermediate_size=768, norm_topk_prob=True)

KIMI_K2 = ModelConfig(
    name="kimi-k2-shape", family="deepseek_v3", vocab_size=163840, hidden_size=7168, num_layers=61,
    num_heads=64, num_kv_heads=64, head_dim=192, intermediate_size=18432, rms_norm_eps=1e-6,
    rope_theta=50000.0, num_experts=384, num_experts_per_tok=8, moe_intermediate_size=2048,
    norm_topk_prob=True, router="sigmoid_group", n_group=1, topk_group=1,
    routed_scaling_factor=2.827, n_shared_experts=1, first_k_dense=1, mla=True, q_lora_rank=1536,
    kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128,
    weight_dtype="fp8_block128")

TINY_MLA_GPU = ModelConfig(
    name="tiny-mla-gpu", family="deepseek_v3", vocab_size=1024, hidden_size=256, num_layers=3,
    num_heads=4, num_kv_heads=4, head_dim=192, intermediate_size=384, rms_norm_eps=1e-6,
    rope_theta=10000.0, num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128,
    norm_topk_prob=True, router="sigmoid_group", n_group=2, topk_group=1,
    routed_scaling_factor=2.5, n_shared_experts=1, first_k_dense=1, mla=True, q_lora_rank=256,
    kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128,
    weight_dtype="fp8_block128", max_position_embeddings=4096)

PRESETS: dict[str, ModelConfig] = {
    c.name: c for c in (LLAMA3_8B, TINY_LLAMA_CPU, TINY_LLAMA_GPU, QWEN3_0_6B, MIXTRAL_8X7B,
                        QWEN3_30B_A3B, KIMI_K2, TINY_MLA_GPU)
}


def preset(name: str) -> ModelConfig:
    try:
        return PRESETS[name]
    except KeyError:
        raise KeyError(f"unknown preset {name!r}; known: {sorted(PRESETS)}") from None
