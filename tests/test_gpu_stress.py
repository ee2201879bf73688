"""The back-to-back stress harness (scc26_nccl_shim_b200.parallel.stress) on
the GPUs this run sees, at every clique size in {1, 2, 4, 8} the box has:
every standard, boundary and pipeline-edge case must PASS with no guard
damage and on the route the independent oracle predicts; the checker
mutation self-test must make cases FAIL."""
import os
import subprocess
import sys

import pytest

from conftest import REPO, need_gpus

pytestmark = pytest.mark.gpu

# Small thresholds keep the cases small while they still take the custom
# routes; tuning is skipped (the routes' static rules, which the oracle
# restates, are exercised).
SMALL = {"NCCL_B200_AR_MIN": "4M", "NCCL_B200_AG_MIN": "4M", "NCCL_B200_RS_MIN": "4M",
         "NCCL_B200_BC_MIN": "4M", "NCCL_B200_TUNE": "0"}
# Small pipeline units, so the edge cases are small too: a 4 MiB NVLS round,
# a 32 KiB push-chain chunk, a 256 KiB host-lane piece with a forced share.
EDGES = {"NCCL_B200_NVLS_ROUND": "4M", "NCCL_B200_RING_CHUNK": "32K", "NCCL_B200_HOST_PIECE": "256K",
         "NCCL_B200_MIN_HOST_BYTES": "64K"}


def run(args, env=None, timeout=900):
    full = dict(os.environ)
    full.update(SMALL)
    full.update(env or {})  # a test's own settings win over the small thresholds
    r = subprocess.run([sys.executable, "-m", "scc26_nccl_shim_b200.parallel.stress", *args],
                       cwd=REPO, env=full, capture_output=True, text=True, timeout=timeout)
    rows = [l.split("\t") for l in r.stdout.splitlines() if "\t" in l and not l.startswith("case\t")]
    return r.returncode, rows, r.stdout + r.stderr[-3000:]


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_stress_all_cases_pass(n):
    need_gpus(n)
    rc, rows, log = run(["--gpus", str(n), "--iters", "3", "--scale", "4"])
    assert rc == 0, log
    assert rows and all(r[4] == "PASS" and r[5] == "0" for r in rows), log
    # The eligible large cases ran on the interposer's own routes.
    custom = {r[0] for r in rows if r[6] != "nccl"}
    assert any(c.startswith("allreduce_float32") for c in custom), log
    for op in ("max", "prod", "min", "avg", "premulsum"):
        assert f"allreduce_{op}" in custom, (op, log)


def test_stress_checker_mutation_fails():
    need_gpus(1)
    rc, rows, log = run(["--gpus", "1", "--iters", "2", "--scale", "8", "--corrupt-shift", "3",
                         "--filter", "float32_oop", "--no-boundary"])
    assert rc != 0, log
    assert rows and all(r[4] == "FAIL" for r in rows), log


def test_stress_route_oracle_catches_a_wrong_route():
    """The route check can fail: the library is told to force one-shot while
    the oracle does not see that setting, so every AllReduce case that runs
    one-shot disagrees with the oracle's two-shot and reports ROUTE."""
    need_gpus(2)
    rc, rows, log = run(["--gpus", "2", "--iters", "1", "--scale", "8", "--no-boundary",
                         "--filter", "allreduce_float32_oop", "--oracle-drop", "NCCL_B200_ALGO"],
                        env={"NCCL_B200_ALGO": "ar=oneshot"})
    assert rc != 0, log
    assert rows and all(r[4] == "ROUTE" and r[6] == "ar_oneshot" and r[7] == "ar_twoshot" for r in rows), log


@pytest.mark.parametrize("n", [2, 4, 8])
def test_stress_differential_against_stock_nccl(n):
    need_gpus(n)
    rc, rows, log = run(["--gpus", str(n), "--iters", "2", "--scale", "8", "--diff", "--no-boundary",
                         "--filter", "oop"])
    assert rc == 0, log


@pytest.mark.parametrize("n", [2, 4, 8])
def test_stress_ordering_controls(n):
    """A delayed input producer on the last rank, inputs overwritten right
    after every call, and new caller streams every iteration: all cases
    must still PASS (reference counterparts: STRESS_DELAY_INPUT_DEVICE,
    STRESS_TEST_OVERWRITE_AFTER_GROUP, V4_FRESH_STREAMS)."""
    need_gpus(n)
    rc, rows, log = run(["--gpus", str(n), "--iters", "3", "--scale", "4", "--no-boundary",
                         "--filter", "float32", "--delay-input-device", str(n - 1), "--delay-ms", "20",
                         "--overwrite-after", "--fresh-streams"])
    assert rc == 0, log
    assert rows and all(r[4] == "PASS" for r in rows), log
    assert any(r[6] != "nccl" for r in rows), log


GANGS = ["ar=push,rs=push,ag=push,bc=ring", "ar=nvls,rs=nvls,ag=nvls,bc=nvls",
         "ar=oneshot,rs=pull,ag=pull,bc=scatter",
         "ar=twoshot_ll,rs=ll,ag=ll,bc=ll"]


@pytest.mark.parametrize("algo", GANGS)
@pytest.mark.parametrize("n", [2, 4, 8])
def test_stress_gang_routes(algo, n):
    """The in-kernel-synchronized routes under the back-to-back
    harness, with the ordering controls on."""
    need_gpus(n)
    rc, rows, log = run(["--gpus", str(n), "--iters", "3", "--scale", "4", "--no-boundary",
                         "--filter", "_", "--algo", algo, "--overwrite-after", "--fresh-streams"],
                        env={"NCCL_B200_NVLS": "on"})
    assert rc == 0, log
    assert rows and all(r[4] == "PASS" for r in rows), log


@pytest.mark.parametrize("algo", GANGS + ["ar=twoshot,rs=pull,ag=pull,bc=pull"])
@pytest.mark.parametrize("n", [2, 4, 8])
def test_stress_pipeline_edges(algo, n):
    """-1/0/+1 vector around every engine's pipeline unit (NVLS round and
    per-slot part, push-reduce round, push-chain step, host-lane piece with
    a forced host share), on each route set."""
    need_gpus(n)
    env = dict(EDGES, NCCL_B200_NVLS="on")
    if "twoshot" in algo:
        env["NCCL_B200_HOST_SHARE_PPM"] = "1500"
    rc, rows, log = run(["--gpus", str(n), "--iters", "2", "--no-standard", "--no-boundary", "--edges",
                         "--algo", algo], env=env)
    assert rc == 0, log
    assert len(rows) >= 24 and all(r[4] == "PASS" for r in rows), log


@pytest.mark.parametrize("n", [1, 2, 8])
def test_stress_large_size_edges_and_cap(n):
    """2 GiB and 4 GiB logical-size edges and the 8 GiB cap: at the cap the
    interposer runs the call, one element above it NCCL does."""
    need_gpus(n)
    rc, rows, log = run(["--gpus", str(n), "--iters", "1", "--no-standard", "--no-boundary", "--big"],
                        env={"NCCL_B200_AR_MIN": "32M", "NCCL_B200_AG_MIN": "32M", "NCCL_B200_RS_MIN": "32M",
                             "NCCL_B200_BC_MIN": "32M"}, timeout=1800)
    assert rc == 0, log
    by = {r[0]: r for r in rows}
    assert by["cap_allreduce_at"][6] != "nccl" and by["cap_allreduce_above"][6] == "nccl", log
    assert by["cap_broadcast_above"][6] == "nccl", log


@pytest.mark.parametrize("n", [2, 4, 8])
def test_stress_nvls_copy_in_ahead_edges(n):
    """The NVLS AllReduce with every copy-in first (NCCL_B200_NVLS_AHEAD=1,
    a scratch buffer per round): every pipeline edge exact."""
    need_gpus(n)
    env = dict(EDGES, NCCL_B200_NVLS="on", NCCL_B200_NVLS_AHEAD="1")
    rc, rows, log = run(["--gpus", str(n), "--iters", "2", "--no-standard", "--no-boundary", "--edges",
                         "--algo", "ar=nvls", "--filter", "_ar"], env=env)
    assert rc == 0, log
    assert rows and all(r[4] == "PASS" for r in rows), log
