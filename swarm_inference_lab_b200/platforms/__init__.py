"""Platform adapters: service files, firewall hints, hardware facts and paths per OS.

``current()`` returns the adapter for this host.  Linux (the B200 platform) is
implemented fully: a systemd unit for the node agent, an nftables rule set for the
control / data / probe ports (generated, not applied), hardware facts from /proc and
``nvidia-smi`` queries (read-only), and XDG-style paths.  macOS and Windows adapters
produce their service definitions (launchd plist / ``sc.exe`` command line) but
report that the sm_100a runtime does not run there.

Reference: si/platforms/base.py, linux.py, macos.py, windows.py.
"""
from __future__ import annotations

import os
import platform
import shutil
import subprocess
from dataclasses import dataclass
from pathlib import Path


@dataclass
class Paths:
    config: Path
    state: Path
    cache: Path
    logs: Path


class PlatformAdapter:
    name = "base"
    runtime_supported = False

    def paths(self, app: str = "swarm-b200") -> Paths:
        home = Path.home()
        return Paths(home / f".{app}" / "config", home / f".{app}" / "state", home / f".{app}" / "cache",
                     home / f".{app}" / "logs")

    def service_definition(self, exec_argv: list[str], *, name: str = "swarm-node") -> str:
        raise NotImplementedError

    def firewall_rules(self, ports: list[int]) -> str:
        return ""

    def hardware(self) -> dict:
        return {"os": platform.system(), "machine": platform.machine(), "cpus": os.cpu_count()}


class LinuxAdapter(PlatformAdapter):
    name = "linux"
    runtime_supported = True

    def paths(self, app: str = "swarm-b200") -> Paths:
        env = os.environ
        home = Path.home()
        return Paths(Path(env.get("XDG_CONFIG_HOME", home / ".config")) / app,
                     Path(env.get("XDG_STATE_HOME", home / ".local" / "state")) / app,
                     Path(env.get("XDG_CACHE_HOME", home / ".cache")) / app,
                     Path(env.get("XDG_STATE_HOME", home / ".local" / "state")) / app / "logs")

    def service_definition(self, exec_argv: list[str], *, name: str = "swarm-node") -> str:
        cmd = " ".join(exec_argv)
        return (f"[Unit]\nDescription={name} (swarm inference node agent)\nAfter=network-online.target\n"
                f"Wants=network-online.target\n\n[Service]\nType=simple\nExecStart={cmd}\n"
                f"Restart=on-failure\nRestartSec=5\nKillSignal=SIGTERM\nTimeoutStopSec=30\n"
                f"LimitMEMLOCK=infinity\nLimitNOFILE=1048576\n\n[Install]\nWantedBy=multi-user.target\n")

    def firewall_rules(self, ports: list[int]) -> str:
        plist = ", ".join(str(p) for p in sorted(set(ports)))
        return ("table inet swarm {\n  chain input {\n    type filter hook input priority 0; policy accept;\n"
                f"    tcp dport {{ {plist} }} ct state new accept\n  }}\n}}\n")

    def hardware(self) -> dict:
        hw = super().hardware()
        try:
            with open("/proc/meminfo") as f:
                for line in f:
                    if line.startswith("MemTotal:"):
                        hw["host_memory_gb"] = round(int(line.split()[1]) * 1024 / 1e9, 1)
        except OSError:
            pass
        if shutil.which("nvidia-smi"):
            try:
                out = subprocess.run(["nvidia-smi", "--query-gpu=name,memory.total,driver_version",
                                      "--format=csv,noheader"], capture_output=True, text=True, timeout=10)
                hw["gpus"] = [dict(zip(("name", "memory", "driver"), (x.strip() for x in l.split(","))))
                              for l in out.stdout.strip().splitlines() if l.strip()]
            except (OSError, subprocess.SubprocessError):
                pass
        return hw


class MacAdapter(PlatformAdapter):
    name = "macos"

    def service_definition(self, exec_argv: list[str], *, name: str = "swarm-node") -> str:
        args = "".join(f"    <string>{a}</string>\n" for a in exec_argv)
        return ('<?xml version="1.0" encoding="UTF-8"?>\n<plist version="1.0"><dict>\n'
                f"  <key>Label</key><string>dev.swarm.{name}</string>\n  <key>ProgramArguments</key>\n"
                f"  <array>\n{args}  </array>\n  <key>KeepAlive</key><true/>\n</dict></plist>\n")


class WindowsAdapter(PlatformAdapter):
    name = "windows"

    def service_definition(self, exec_argv: list[str], *, name: str = "swarm-node") -> str:
        cmd = " ".join(f'"{a}"' if " " in a else a for a in exec_argv)
        return f'sc.exe create {name} binPath= "{cmd}" start= auto'

    def firewall_rules(self, ports: list[int]) -> str:
        return "\n".join(f'netsh advfirewall firewall add rule name="swarm-{p}" dir=in action=allow '
                         f"protocol=TCP localport={p}" for p in sorted(set(ports)))


def current() -> PlatformAdapter:
    s = platform.system()
    return {"Linux": LinuxAdapter, "Darwin": MacAdapter, "Windows": WindowsAdapter}.get(s, PlatformAdapter)()
