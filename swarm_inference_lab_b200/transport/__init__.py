"""Byte transports: the SWRING01 stage ring over TCP/TLS, tensor codec, fault injection."""
