"""bench.py's launch contract on the CPU: under torchrun with two gloo ranks
(127.0.0.1) the parent ranks rendezvous, rank 0 alone runs the one-process
N-GPU worker, and exactly one JSON line is printed. With no GPU visible the
worker reports the run as unavailable instead of failing."""
import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import REPO, gpu_count


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_bench_under_torchrun_prints_one_line():
    if gpu_count():
        pytest.skip("CPU plumbing test")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), "bench.py", "--gpus", "2",
           "--steps", "1", "--warmup", "3"]
    env = dict(os.environ)
    env.pop("LD_PRELOAD", None)
    r = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert "unavailable" in d and "need 2 GPUs" in d["unavailable"], d


def test_bench_reference_arm_reports_itself():
    if gpu_count():
        pytest.skip("CPU plumbing test")
    env = dict(os.environ)
    env.pop("LD_PRELOAD", None)
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "1", "--steps", "1",
                        "--warmup", "3"], cwd=REPO, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    assert json.loads(lines[0])["impl"] == "reference"
