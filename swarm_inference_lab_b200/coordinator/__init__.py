"""Coordinator: session control, deployment, registry, durable state."""
