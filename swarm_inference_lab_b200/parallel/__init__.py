"""Intra-box parallelism: tensor, expert and pipeline parallel plumbing."""
