"""Process glue of the cluster product: the coordinator process (pairing server + gRPC
control plane) and a node's agent process (worker runtime), both configured from the
cluster state store.

The coordinator serves pairing on the cluster endpoint ``host:port`` and the
``swarm.v1.Coordinator`` gRPC service on ``host:port+1``, both from one process that
``swarm cluster start`` launches (``swarm cluster stop`` ends it).  Every gRPC channel
is mutual TLS with the cluster CA: the coordinator holds a certificate the CA issues to
its own identity, each node the certificate it received when it paired, and both bind
the holder's identity fingerprint so the other side can check it.

Reference: si/cluster/orchestrator.py:702 (local coordinator + worker runtimes per
node), si/commands/cluster.py:626-662 (start / stop), si/commands/node.py:330-616
(agent, configure, install-service, update).
"""
from __future__ import annotations

import asyncio
import json
import os
import signal
import time
from pathlib import Path

from ..security.tls import PemPair, issue_node_cert
from .state import ClusterStateStore

CONTROL_PORT_OFFSET = 1


def control_endpoint(cluster_endpoint: str) -> str:
    host, port = cluster_endpoint.rsplit(":", 1)
    return f"{host}:{int(port) + CONTROL_PORT_OFFSET}"


def coordinator_tls(store: ClusterStateStore) -> tuple[bytes, bytes, bytes]:
    """(CA cert, coordinator cert, coordinator key); the certificate is issued by the
    cluster CA to the coordinator's identity on first use."""
    ca_crt, ca_key = store.ca()
    crt_p, key_p = store.root / "tls" / "coordinator.crt", store.root / "tls" / "coordinator.key"
    if not crt_p.exists():
        if ca_key is None:
            raise RuntimeError("this node holds no cluster CA key (not the coordinator)")
        doc = store.load_cluster()
        host = doc["coordinator_endpoint"].rsplit(":", 1)[0]
        ident = store.identity("coordinator")
        pair = issue_node_cert(PemPair(ca_crt, ca_key), "coordinator", ident.fingerprint,
                               sorted({host, "127.0.0.1", "localhost"}))
        (store.root / "tls").mkdir(exist_ok=True)
        crt_p.write_bytes(pair.cert)
        key_p.write_bytes(pair.key)
        key_p.chmod(0o600)
    return ca_crt, crt_p.read_bytes(), key_p.read_bytes()


def node_tls(store: ClusterStateStore) -> tuple[bytes, bytes, bytes]:
    ca = (store.root / "ca" / "ca.crt").read_bytes()
    return (ca, (store.root / "tls" / "node.crt").read_bytes(),
            (store.root / "tls" / "node.key").read_bytes())


def server_credentials(ca: bytes, cert: bytes, key: bytes):
    import grpc
    return grpc.ssl_server_credentials([(key, cert)], root_certificates=ca, require_client_auth=True)


def channel_credentials(ca: bytes, cert: bytes, key: bytes):
    import grpc
    return grpc.ssl_channel_credentials(root_certificates=ca, private_key=key, certificate_chain=cert)


def coordinator_client(store: ClusterStateStore, timeout: float = 600.0):
    """A ``CoordinatorClient`` of the cluster this state store belongs to, authenticated
    as this node (the coordinator's own identity on the coordinator machine)."""
    from ..coordinator.service import CoordinatorClient
    doc = store.load_cluster()
    creds = channel_credentials(*(coordinator_tls(store) if doc["role"] == "coordinator"
                                  else node_tls(store)))
    return CoordinatorClient(control_endpoint(doc["coordinator_endpoint"]), creds, timeout=timeout)


async def serve_coordinator(store: ClusterStateStore, *, heartbeat_timeout_s: float = 5.0,
                            heartbeat_s: float = 1.0, ready_file: str | None = None,
                            drain_s: float = 30.0) -> None:
    """The coordinator process: pairing + gRPC control plane until SIGTERM / SIGINT; on the
    signal it stops admitting requests and lets running ones finish (at most ``drain_s``)."""
    from ..coordinator.service import CoordinatorCore, CoordinatorRpcServer
    from .pairing import PairingManager
    doc = store.load_cluster()
    if doc["role"] != "coordinator":
        raise RuntimeError("only the cluster's coordinator node serves the control plane")
    ident = store.identity("coordinator")
    ca, crt, key = coordinator_tls(store)
    core = CoordinatorCore(ident, state_dir=store.root, cluster_store=store,
                           heartbeat_timeout_s=heartbeat_timeout_s, heartbeat_s=heartbeat_s,
                           worker_credentials=channel_credentials(ca, crt, key))
    host, port = doc["coordinator_endpoint"].rsplit(":", 1)
    pm = PairingManager(store, doc["coordinator_endpoint"])
    core.pairing = pm
    await pm.start(host, int(port))
    rpc = CoordinatorRpcServer(core, host=host, port=int(port) + CONTROL_PORT_OFFSET,
                               credentials=server_credentials(ca, crt, key))
    cport = await rpc.start()
    # models deployed before a restart come back once their workers have re-registered
    restoring = asyncio.get_running_loop().create_task(core.restore())
    rt = store.runtime()
    rt["coordinator"] = {"pid": os.getpid(), "pairing": doc["coordinator_endpoint"],
                         "control": f"{host}:{cport}", "started": time.time()}
    store.save_runtime(rt)
    if ready_file:
        Path(ready_file).write_text(json.dumps(rt["coordinator"]))
    stop = asyncio.Event()
    loop = asyncio.get_running_loop()
    for s in (signal.SIGTERM, signal.SIGINT):
        try:
            loop.add_signal_handler(s, stop.set)
        except NotImplementedError:  # pragma: no cover
            pass
    try:
        await stop.wait()
        await core.drain(drain_s)
    finally:
        restoring.cancel()
        await rpc.stop()
        await pm.close()
        rt = store.runtime()
        rt.pop("coordinator", None)
        store.save_runtime(rt)


async def run_node_agent(store: ClusterStateStore, *, host: str | None = None, device: str | None = None,
                         ring_port: int | None = None, control_port: int | None = None,
                         ready_file: str | None = None) -> None:
    """A paired node's worker runtime until SIGTERM / SIGINT."""
    from ..runtime.worker_runtime import TlsFiles, WorkerRuntime
    doc = store.load_cluster()
    conf = store.runtime().get("node_config", {})
    ca, crt, key = node_tls(store)
    node_id = doc.get("node_id") or store.identity().name
    ident = store.identity(node_id)
    wr = WorkerRuntime(node_id, ident, control_endpoint(doc["coordinator_endpoint"]),
                       coordinator_fingerprint=doc["coordinator_fingerprint"],
                       host=host or conf.get("host", "127.0.0.1"),
                       ring_port=ring_port if ring_port is not None else int(conf.get("ring_port", 0)),
                       control_port=(control_port if control_port is not None
                                     else int(conf.get("control_port", 0))),
                       tls=TlsFiles(ca, crt, key), device=device or conf.get("device", "cpu"),
                       heartbeat_s=float(conf.get("heartbeat_s", 1.0)))
    await wr.start()
    rt = store.runtime()
    rt["agent"] = {"pid": os.getpid(), "worker_id": node_id, "ring": wr.ring_endpoint,
                   "control": wr.control_endpoint, "started": time.time()}
    store.save_runtime(rt)
    if ready_file:
        Path(ready_file).write_text(json.dumps({"worker_id": node_id, "ring": wr.ring_endpoint,
                                                "control": wr.control_endpoint, "pid": os.getpid()}))
    stop = asyncio.Event()
    loop = asyncio.get_running_loop()
    for s in (signal.SIGTERM, signal.SIGINT):
        try:
            loop.add_signal_handler(s, stop.set)
        except NotImplementedError:  # pragma: no cover
            pass
    try:
        await stop.wait()
    finally:
        await wr.stop()
        if store.cluster_path().exists():        # gone after `node leave`
            rt = store.runtime()
            if rt.get("agent", {}).get("pid") == os.getpid():
                rt.pop("agent")
                store.save_runtime(rt)


def stop_local_agent(store: ClusterStateStore, timeout_s: float = 20.0) -> bool:
    """Stops this node's agent process, found by the pid it recorded (and only if that pid
    still runs ``node agent``); True if one was stopped."""
    pid = store.runtime().get("agent", {}).get("pid")
    if not pid:
        return False
    try:
        cmd = Path(f"/proc/{int(pid)}/cmdline").read_bytes().split(b"\0")
    except OSError:
        return False
    if b"agent" not in cmd or not any(b"swarm_inference_lab_b200" in c or b"swarm" in c for c in cmd):
        return False
    try:
        os.kill(int(pid), signal.SIGTERM)
    except ProcessLookupError:
        return False
    t0 = time.time()
    while time.time() - t0 < timeout_s:
        try:
            state = Path(f"/proc/{int(pid)}/stat").read_text().rsplit(")", 1)[1].split()[0]
        except (OSError, IndexError):
            break
        if state == "Z":            # exited, not yet reaped by its parent
            break
        time.sleep(0.1)
    return True


SYSTEMD_UNIT = """[Unit]
Description=swarm-inference-lab B200 node agent ({node})
After=network-online.target
Wants=network-online.target

[Service]
Type=simple
Environment=SWARM_STATE_DIR={state}
ExecStart={python} -m swarm_inference_lab_b200.cli node agent --state-dir {state}
Restart=on-failure
RestartSec=2
LimitMEMLOCK=infinity

[Install]
WantedBy=multi-user.target
"""


def service_unit(store: ClusterStateStore, python: str) -> str:
    doc = store.load_cluster()
    return SYSTEMD_UNIT.format(node=doc.get("node_id", "node"), state=store.root, python=python)
