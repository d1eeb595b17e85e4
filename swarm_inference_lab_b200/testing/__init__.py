"""Process harness and fixtures for multi-process tests."""
