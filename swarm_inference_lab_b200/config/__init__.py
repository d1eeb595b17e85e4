"""Strict configuration models and YAML loading."""
from .models import (ConfigError, EngineOptions, ModelManifest, NetworkProfile, NodeProfile,  # noqa: F401
                     ProductConfig, StageDefinition, StrictModel, load_yaml)
