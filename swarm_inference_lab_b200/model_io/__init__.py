"""Checkpoint inspection (safetensors, GGUF), architecture profiles, resolver, partitioning."""
