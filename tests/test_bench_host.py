"""Host-side logic of bench.py that the GPU runs depend on, checked on CPU:
the sub-result children of a torchrun job form a process group of their own
(torchrun's agent-store variables must not reach them)."""
import os
import socket
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))

import bench  # noqa: E402


def test_child_env_drops_torchrun_agent_variables(monkeypatch):
    monkeypatch.setenv("TORCHELASTIC_USE_AGENT_STORE", "True")
    monkeypatch.setenv("TORCHELASTIC_RUN_ID", "x")
    env = bench.child_env(1, 2, 1, 12345)
    assert not any(k.startswith("TORCHELASTIC_") for k in env)
    assert (env["RANK"], env["WORLD_SIZE"], env["LOCAL_RANK"], env["MASTER_PORT"]) == ("1", "2", "1", "12345")
    assert env["MASTER_ADDR"] == "127.0.0.1"


def test_children_rendezvous_under_torchrun():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), str(REPO / "tests" / "helpers" / "child_rendezvous.py")]
    env = dict(os.environ)
    env["OMP_NUM_THREADS"] = "1"
    proc = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=240)
    assert proc.returncode == 0, proc.stderr[-3000:]
