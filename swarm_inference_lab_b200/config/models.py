"""Strict configuration models (pydantic, unknown keys rejected) and the YAML loader.

``load_yaml`` supports relative ``include:`` lists (merged depth-first, later
files override earlier ones, cycles rejected).  ``ProductConfig`` carries the
coordinator/product knobs (timeouts, planner beam, cost weights, trust);
``NodeProfile`` / ``NetworkProfile`` describe nodes and links for the planner
and simulator; ``EngineOptions`` the per-stage runtime switches.

Reference: si/config/models.py:17-687 (``StrictModel`` with extra=forbid),
si/config/loader.py:15-109, si/config/product.py:14-83,
si/model/qwen3_runtime.py:15-140 (engine options).
"""
from __future__ import annotations

from pathlib import Path
from typing import Any, Literal

import yaml
from pydantic import BaseModel, ConfigDict, Field, PositiveInt


class StrictModel(BaseModel):
    model_config = ConfigDict(extra="forbid", frozen=False, validate_assignment=True)


class ConfigError(ValueError):
    pass


def _merge(a: dict, b: dict) -> dict:
    out = dict(a)
    for k, v in b.items():
        if isinstance(v, dict) and isinstance(out.get(k), dict):
            out[k] = _merge(out[k], v)
        else:
            out[k] = v
    return out


def load_yaml(path: str | Path, _stack: tuple = ()) -> dict:
    path = Path(path).resolve()
    if path in _stack:
        raise ConfigError(f"include cycle: {' -> '.join(str(p) for p in (*_stack, path))}")
    try:
        data = yaml.safe_load(path.read_text(encoding="utf-8")) or {}
    except (OSError, yaml.YAMLError) as exc:
        raise ConfigError(f"{path}: {exc}") from None
    if not isinstance(data, dict):
        raise ConfigError(f"{path}: top level must be a mapping")
    merged: dict = {}
    for inc in data.pop("include", []) or []:
        merged = _merge(merged, load_yaml(path.parent / inc, (*_stack, path)))
    return _merge(merged, data)


class PlannerWeights(StrictModel):
    ttft: float = 1.0
    decode: float = 1.0
    aggregate: float = 1.0
    unmeasured_penalty: float = 0.98


class ProductConfig(StrictModel):
    coordinator_host: str = "127.0.0.1"
    coordinator_port: int = Field(default=7650, ge=0, le=65535)
    worker_heartbeat_timeout_s: float = 15.0
    route_lease_ttl_s: float = 300.0
    request_timeout_s: float = 120.0
    planning_max_sequence_tokens: PositiveInt = 2048
    planner_beam_width: PositiveInt = 512
    planner_max_stages: PositiveInt = 32
    planner_max_workers: PositiveInt = 64
    planner_mode: Literal["speed", "throughput", "capacity", "balanced"] = "balanced"
    weights: PlannerWeights = PlannerWeights()
    max_recoveries: int = 3
    trust_fingerprints: list[str] = []
    state_dir: str = "~/.swarm-b200"

    @classmethod
    def from_yaml(cls, path) -> "ProductConfig":
        return cls(**load_yaml(path))


class EngineOptions(StrictModel):
    profile: Literal["correctness", "fast"] = "fast"
    attention_backend: Literal["sm100_paged"] = "sm100_paged"
    cache_backend: Literal["paged"] = "paged"
    cache_dtype: Literal["bfloat16"] = "bfloat16"
    max_sequence_length: PositiveInt = 4096
    max_batch_size: PositiveInt = 64
    cuda_graph_batch_sizes: tuple[int, ...] = (1, 2, 4, 8, 16, 32, 48, 64, 96, 128)
    prefill_token_budget: PositiveInt = 16384
    scheduler_policy: Literal["latency", "balanced", "throughput"] = "balanced"
    tensor_parallel: PositiveInt = 1
    expert_parallel: PositiveInt = 1
    comm: Literal["fused", "nccl"] = "fused"
    nvtx: bool = False


class NodeProfile(StrictModel):
    name: str
    gpus: int = 0
    gpu_name: str = ""
    gpu_memory_gb: float = 0.0
    host_memory_gb: float = 0.0
    decode_gbps: float = 0.0     # measured weight-streaming bandwidth
    tflops: float = 0.0
    labels: dict[str, str] = {}


class NetworkProfile(StrictModel):
    name: str
    rtt_ms: float
    bandwidth_mbps: float
    jitter_ms: float = 0.0
    stability: float = 1.0
    loss: float = 0.0

    @classmethod
    def from_yaml(cls, path) -> "NetworkProfile":
        return cls(**load_yaml(path))


class StageDefinition(StrictModel):
    stage_id: int = Field(ge=0)
    worker_id: str
    layer_start: int = Field(ge=0)
    layer_end: int = Field(ge=1)
    embed: bool = False
    head: bool = False
    endpoint: str = ""
    weight_bytes: int = Field(default=0, ge=0)


class ModelManifest(StrictModel):
    model_id: str
    revision: str
    family: str
    num_layers: PositiveInt
    dtype: str = "bfloat16"
    stages: list[StageDefinition] = []
    shard_hashes: dict[str, str] = {}       # shard file (or directory) -> sha256
    total_weight_bytes: int = Field(default=0, ge=0)

    def check_union(self) -> None:
        """Every layer in exactly one stage, in order."""
        cur = 0
        for s in sorted(self.stages, key=lambda s: s.stage_id):
            if s.layer_start != cur or s.layer_end <= s.layer_start:
                raise ConfigError(f"stage {s.stage_id} breaks the layer union at {cur}")
            cur = s.layer_end
        if cur != self.num_layers:
            raise ConfigError(f"stages cover {cur} of {self.num_layers} layers")


def parse(model: type[StrictModel], data: dict[str, Any]) -> StrictModel:
    try:
        return model(**data)
    except Exception as exc:  # pydantic.ValidationError
        raise ConfigError(str(exc)) from None
