"""The back-to-back stress harness (scc26_nccl_shim_b200.parallel.stress) on
the GPUs this run sees: every standard and boundary case must PASS with no
guard damage, and the checker mutation self-test must make cases FAIL."""
import os
import subprocess
import sys

import pytest

from conftest import REPO, gpu_count, need_gpus

pytestmark = pytest.mark.gpu

# Small thresholds keep the cases small while they still take the custom
# routes; tuning is skipped (the routes' defaults are exercised).
SMALL = {"NCCL_B200_AR_MIN": "4M", "NCCL_B200_AG_MIN": "4M", "NCCL_B200_RS_MIN": "4M",
         "NCCL_B200_BC_MIN": "4M", "NCCL_B200_TUNE": "0"}


def run(args, env=None):
    r = subprocess.run([sys.executable, "-m", "scc26_nccl_shim_b200.parallel.stress", *args],
                       cwd=REPO, env=dict(os.environ, **SMALL, **(env or {})), capture_output=True, text=True,
                       timeout=900)
    rows = [l.split("\t") for l in r.stdout.splitlines() if "\t" in l and not l.startswith("case\t")]
    return r.returncode, rows, r.stdout + r.stderr[-3000:]


def test_stress_all_cases_pass():
    need_gpus(1)
    n = min(2, gpu_count())
    rc, rows, log = run(["--gpus", str(n), "--iters", "3", "--scale", "4"])
    assert rc == 0, log
    assert rows and all(r[4] == "PASS" and r[5] == "0" for r in rows), log
    # The eligible large cases ran on the interposer's own routes.
    custom = {r[0] for r in rows if r[6] == "custom"}
    assert any(c.startswith("allreduce_float32") for c in custom), log
    assert "allreduce_max" in custom  # ncclMax runs on the fused kernels too


def test_stress_checker_mutation_fails():
    need_gpus(1)
    n = min(2, gpu_count())
    rc, rows, log = run(["--gpus", str(n), "--iters", "2", "--scale", "8", "--corrupt-shift", "3",
                         "--filter", "float32_oop", "--no-boundary"])
    assert rc != 0, log
    assert rows and all(r[4] == "FAIL" for r in rows), log


def test_stress_differential_against_stock_nccl():
    need_gpus(2)
    rc, rows, log = run(["--gpus", "2", "--iters", "2", "--scale", "8", "--diff", "--no-boundary",
                         "--filter", "oop"])
    assert rc == 0, log


def test_stress_ordering_controls():
    """A delayed input producer on the last rank, inputs overwritten right
    after every call, and new caller streams every iteration: all cases
    must still PASS (reference counterparts: STRESS_DELAY_INPUT_DEVICE,
    STRESS_TEST_OVERWRITE_AFTER_GROUP, V4_FRESH_STREAMS)."""
    need_gpus(2)
    n = min(4, gpu_count())
    rc, rows, log = run(["--gpus", str(n), "--iters", "3", "--scale", "4", "--no-boundary",
                         "--filter", "float32", "--delay-input-device", str(n - 1), "--delay-ms", "20",
                         "--overwrite-after", "--fresh-streams"])
    assert rc == 0, log
    assert rows and all(r[4] == "PASS" for r in rows), log
    assert any(r[6] == "custom" for r in rows), log


@pytest.mark.parametrize("algo", ["ar=push,rs=push,ag=push,bc=ring", "ar=nvls,rs=nvls,ag=nvls,bc=nvls"])
def test_stress_gang_routes(algo):
    """The in-kernel-synchronized routes under the back-to-back harness on
    up to four GPUs, with the ordering controls on."""
    need_gpus(2)
    n = min(4, gpu_count())
    rc, rows, log = run(["--gpus", str(n), "--iters", "3", "--scale", "4", "--no-boundary",
                         "--filter", "_", "--algo", algo, "--overwrite-after", "--fresh-streams"],
                        env={"NCCL_B200_NVLS": "on"})
    assert rc == 0, log
    assert rows and all(r[4] == "PASS" for r in rows), log
