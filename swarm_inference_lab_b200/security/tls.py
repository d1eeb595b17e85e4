"""Cluster TLS: a cluster CA, node certificates bound to identity fingerprints,
and TLS 1.3 client/server contexts with fingerprint pinning.

Node certificates carry the node's identity fingerprint in a URI SAN
(``swarm-node:<fingerprint>``), so a peer can check that the TLS endpoint is
the identity named by the route lease, independent of its address.

Reference: si/security/tls.py:157-600.
"""
from __future__ import annotations

import datetime
import ssl
from dataclasses import dataclass
from pathlib import Path

from cryptography import x509
from cryptography.hazmat.primitives import hashes, serialization
from cryptography.hazmat.primitives.asymmetric import ec
from cryptography.x509.oid import NameOID

URI_PREFIX = "swarm-node:"


@dataclass
class PemPair:
    cert: bytes
    key: bytes

    def write(self, cert_path: Path, key_path: Path) -> None:
        cert_path.write_bytes(self.cert)
        key_path.write_bytes(self.key)
        key_path.chmod(0o600)


def _key_pem(key) -> bytes:
    return key.private_bytes(serialization.Encoding.PEM, serialization.PrivateFormat.PKCS8,
                             serialization.NoEncryption())


def create_ca(cluster_name: str, days: int = 3650) -> PemPair:
    key = ec.generate_private_key(ec.SECP256R1())
    name = x509.Name([x509.NameAttribute(NameOID.COMMON_NAME, f"{cluster_name} cluster CA")])
    now = datetime.datetime.now(datetime.timezone.utc)
    cert = (x509.CertificateBuilder().subject_name(name).issuer_name(name)
            .public_key(key.public_key()).serial_number(x509.random_serial_number())
            .not_valid_before(now - datetime.timedelta(minutes=5))
            .not_valid_after(now + datetime.timedelta(days=days))
            .add_extension(x509.BasicConstraints(ca=True, path_length=0), critical=True)
            .sign(key, hashes.SHA256()))
    return PemPair(cert.public_bytes(serialization.Encoding.PEM), _key_pem(key))


def issue_node_cert(ca: PemPair, node_name: str, fingerprint: str, hosts: list[str],
                    days: int = 365) -> PemPair:
    ca_cert = x509.load_pem_x509_certificate(ca.cert)
    ca_key = serialization.load_pem_private_key(ca.key, password=None)
    key = ec.generate_private_key(ec.SECP256R1())
    now = datetime.datetime.now(datetime.timezone.utc)
    import ipaddress
    sans: list[x509.GeneralName] = [x509.UniformResourceIdentifier(URI_PREFIX + fingerprint)]
    for h in hosts:
        try:
            sans.append(x509.IPAddress(ipaddress.ip_address(h)))
        except ValueError:
            sans.append(x509.DNSName(h))
    cert = (x509.CertificateBuilder()
            .subject_name(x509.Name([x509.NameAttribute(NameOID.COMMON_NAME, node_name)]))
            .issuer_name(ca_cert.subject).public_key(key.public_key())
            .serial_number(x509.random_serial_number())
            .not_valid_before(now - datetime.timedelta(minutes=5))
            .not_valid_after(now + datetime.timedelta(days=days))
            .add_extension(x509.SubjectAlternativeName(sans), critical=False)
            .add_extension(x509.BasicConstraints(ca=False, path_length=None), critical=True)
            .sign(ca_key, hashes.SHA256()))
    return PemPair(cert.public_bytes(serialization.Encoding.PEM), _key_pem(key))


def cert_fingerprint_binding(cert_pem_or_der: bytes) -> str | None:
    try:
        cert = x509.load_pem_x509_certificate(cert_pem_or_der)
    except ValueError:
        cert = x509.load_der_x509_certificate(cert_pem_or_der)
    try:
        san = cert.extensions.get_extension_for_class(x509.SubjectAlternativeName).value
    except x509.ExtensionNotFound:
        return None
    for uri in san.get_values_for_type(x509.UniformResourceIdentifier):
        if uri.startswith(URI_PREFIX):
            return uri[len(URI_PREFIX):]
    return None


def _write_tmp(data: bytes, directory: Path, name: str) -> str:
    p = directory / name
    p.write_bytes(data)
    p.chmod(0o600)
    return str(p)


def server_context(ca: PemPair, node: PemPair, workdir: Path) -> ssl.SSLContext:
    ctx = ssl.SSLContext(ssl.PROTOCOL_TLS_SERVER)
    ctx.minimum_version = ssl.TLSVersion.TLSv1_3
    ctx.load_cert_chain(_write_tmp(node.cert, workdir, "node.crt"), _write_tmp(node.key, workdir, "node.key"))
    ctx.load_verify_locations(cadata=ca.cert.decode())
    ctx.verify_mode = ssl.CERT_REQUIRED
    return ctx


def client_context(ca: PemPair, node: PemPair, workdir: Path) -> ssl.SSLContext:
    ctx = ssl.SSLContext(ssl.PROTOCOL_TLS_CLIENT)
    ctx.minimum_version = ssl.TLSVersion.TLSv1_3
    ctx.load_cert_chain(_write_tmp(node.cert, workdir, "client.crt"), _write_tmp(node.key, workdir, "client.key"))
    ctx.load_verify_locations(cadata=ca.cert.decode())
    ctx.check_hostname = False  # identity is pinned by fingerprint, not by address
    ctx.verify_mode = ssl.CERT_REQUIRED
    return ctx


def peer_fingerprint(ssl_object) -> str | None:
    der = ssl_object.getpeercert(binary_form=True)
    return cert_fingerprint_binding(der) if der else None
