"""Cluster product: state store, pairing, node agent, artifacts, network probes."""
