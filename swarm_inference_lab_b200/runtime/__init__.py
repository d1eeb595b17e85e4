"""Persistent stage owners (workers) and their executors."""
