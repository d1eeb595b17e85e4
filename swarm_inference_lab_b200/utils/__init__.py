"""Shared utilities (device timing, clocks sampling, distributed setup)."""
