"""Tracing, telemetry and lifecycle events."""
