"""The mixed-group configuration (scaled to 64 MiB per call here; the
profile run goes to 1 GiB): one ncclGroupStart/End batch of 64 seeded calls
with log-uniform sizes and random collectives, dtypes and reduce ops,
including an operation the interposer never handles. The mixed group must
fall back to libnccl as a whole, in order, with correct results, and the
interposer must run none of it itself. And 64 eligible back-to-back groups
with the host lane forced on, checked after the run: the pinned-host lanes
are reused under stream ordering only."""
import os
import subprocess
import sys

import pytest

from conftest import REPO, need_gpus

pytestmark = pytest.mark.gpu


def run(args, env=None):
    r = subprocess.run([sys.executable, "-m", "scc26_nccl_shim_b200.parallel.mixed", *args], cwd=REPO,
                       env=dict(os.environ, **(env or {})), capture_output=True, text=True, timeout=900)
    import json
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    return r.returncode, (json.loads(lines[-1]) if lines else None), r.stdout[-2000:] + r.stderr[-3000:]


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_mixed_64_call_group_falls_back_in_order(n):
    need_gpus(n)
    rc, res, log = run(["--mode", "mixed", "--gpus", str(n), "--calls", "64", "--max", "64M"])
    assert rc == 0 and res, log
    assert res["mismatches"] == 0, log
    assert res["custom_routes"] == {}, log  # the whole group went to libnccl
    assert res["kinds"]["send_recv"] >= 1
    print("mixed group of", res["calls"], "calls per rank:", res["device_ms"], "ms")


@pytest.mark.parametrize("n", [2, 4, 8])
def test_eligible_groups_back_to_back_with_host_lanes(n):
    need_gpus(n)
    env = {"NCCL_B200_HOST_SHARE_PPM": "1200", "NCCL_B200_HOST_PIECE": "1M", "NCCL_B200_MIN_HOST_BYTES": "64K",
           "NCCL_B200_LANES": "2", "NCCL_B200_TUNE": "0", "NCCL_B200_ALGO": "ar=twoshot,rs=pull,ag=pull,bc=pull",
           "NCCL_SHIM_SUMMARY": "1", "NCCL_B200_AR_MIN": "4M", "NCCL_B200_AG_MIN": "4M",
           "NCCL_B200_RS_MIN": "4M", "NCCL_B200_BC_MIN": "4M"}
    rc, res, log = run(["--mode", "eligible", "--gpus", str(n), "--calls", "64", "--min", "32M", "--max", "96M"],
                       env=env)
    assert rc == 0 and res, log
    assert res["mismatches"] == 0, log
    assert sum(res["custom_routes"].values()) == 64, log
