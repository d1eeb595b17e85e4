"""Identities, signatures, route leases and cluster TLS."""
