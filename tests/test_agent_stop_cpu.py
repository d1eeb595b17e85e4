"""``node leave`` stops this node's agent by the pid the agent recorded, and only if that pid
still runs a ``node agent`` command line: a recycled pid that belongs to another program is
left alone."""
import subprocess
import sys

from swarm_inference_lab_b200.cluster.control import stop_local_agent
from swarm_inference_lab_b200.cluster.state import ClusterStateStore


def test_a_foreign_pid_is_not_signalled(tmp_path):
    st = ClusterStateStore(tmp_path / "node")
    assert stop_local_agent(st) is False                       # nothing recorded
    other = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(60)"])
    try:
        st.save_runtime({"agent": {"pid": other.pid}})
        assert stop_local_agent(st, timeout_s=1.0) is False
        assert other.poll() is None                            # still running
    finally:
        other.kill()
        other.wait(timeout=10)


def test_the_recorded_agent_is_stopped(tmp_path):
    st = ClusterStateStore(tmp_path / "node")
    # a stand-in whose command line names the agent command and exits on SIGTERM
    agent = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(60)",
                              "swarm_inference_lab_b200.cli", "node", "agent"])
    try:
        st.save_runtime({"agent": {"pid": agent.pid}})
        assert stop_local_agent(st, timeout_s=10.0) is True
        assert agent.wait(timeout=10) != 0
    finally:
        if agent.poll() is None:
            agent.kill()
            agent.wait(timeout=10)
