"""Planner + happens-before checker + CPU simulator (the CPU plumbing test).

Every plan is checked for unordered conflicting accesses (including against
the caller's own work before and after the call on each rank's stream) and
then executed on host memory in a random topological order; every output
byte must equal the direct oracle (host fold over whole buffers, rank order).
"""
import ctypes as C
import random

import pytest

from scc26_nccl_shim_b200 import _core as c

SMALL = {"NCCL_B200_MIN_HOST_BYTES": "4096", "NCCL_B200_HOST_PIECE": "262144",
         "NCCL_B200_SM_CHUNK": "1M", "NCCL_B200_STAGE_PIECE": "131072", "NCCL_B200_STAGE_DEPTH": "2"}
CASES = [("ar_twoshot", "allreduce"), ("rs_pull", "reducescatter"), ("ag_pull", "allgather"),
         ("bc_pull", "broadcast"), ("bc_scatter", "broadcast"), ("ar_staged", "allreduce"),
         ("rs_staged", "reducescatter"), ("bc_chain", "broadcast"), ("ar_nvls", "allreduce"),
         ("bc_nvls", "broadcast"), ("ag_nvls", "allgather"), ("rs_nvls", "reducescatter"),
         ("ag_push", "allgather"), ("bc_ring", "broadcast"), ("rs_push", "reducescatter"),
         ("ar_push", "allreduce"), ("ar_hybrid", "allreduce"), ("ar_oneshot", "allreduce"),
         ("rs_hybrid", "reducescatter"), ("ar_twoshot_ll", "allreduce"),
         ("rs_ll", "reducescatter"), ("ag_ll", "allgather"), ("bc_ll", "broadcast")]


def test_baseline_cpu_plumbing_config():
    """The CPU plumbing configuration: 2 simulated ranks, fp32 AllReduce(sum) of 1,048,576
    uniform[-1,1] elements from seed 0, split into NVLink (SM), copy-engine
    and pinned-host shares; the host-lane fold is bit-exact against a serial
    host sum (the oracle folds rank 0 + rank 1 in fp32)."""
    rc, err, st = c.plan_simulate("ar_twoshot", "allreduce", "float32", 2, 1_048_576,
                                  host_ppm=1500, ce_ppm=2000, env=SMALL, seed=0, data_mode=1)
    assert rc == 0, err
    assert st.mismatches == 0
    assert st.sm_bytes > 0 and st.ce_bytes > 0 and st.host_bytes > 0
    assert st.lanes >= 1


@pytest.mark.parametrize("algo,kind", CASES)
@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 8])
def test_plans_race_free_and_exact(algo, kind, n):
    if algo == "bc_scatter" and n < 3:
        pytest.skip("needs 3 ranks")
    rng = random.Random(n * 31 + len(algo))
    for host, ce in [(0, 0), (1200, 0), (0, 2500), (900, 1700)]:
        for inplace in (0, (1 << n) - 1, rng.randrange(1 << n)):
            count = (1 << 18) + (0 if kind == "reducescatter" else rng.choice([0, 1, 3, 7]))
            root = rng.randrange(n)
            rc, err, st = c.plan_simulate(algo, kind, "float32", n, count, root=root,
                                          inplace_mask=inplace, host_ppm=host, ce_ppm=ce,
                                          env=SMALL, seed=rng.randrange(1 << 30))
            assert rc == 0, (algo, n, host, ce, inplace, err)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float64", "int32", "int8", "uint8",
                                   "int64", "uint32", "uint64"])
@pytest.mark.parametrize("op", ["sum", "prod", "max", "min", "avg"])
def test_reductions_all_types(dtype, op):
    for algo, kind in [("ar_twoshot", "allreduce"), ("rs_pull", "reducescatter"),
                       ("ar_staged", "allreduce"), ("rs_staged", "reducescatter")]:
        rc, err, _ = c.plan_simulate(algo, kind, dtype, 3, 40_000, op=op, host_ppm=1000,
                                     env=SMALL, seed=7)
        assert rc == 0, (algo, dtype, op, err)


def test_premulsum_scalars():
    rc, err, _ = c.plan_simulate("ar_twoshot", "allreduce", "float32", 4, 100_000, op="premulsum",
                                 host_ppm=1500, env=SMALL, seed=3, data_mode=1,
                                 scalars=[0.5, -2.0, 1.5, 0.25])
    assert rc == 0, err


def test_share_accounting():
    n, count = 4, 1 << 20
    _, _, a = c.plan_simulate("ar_twoshot", "allreduce", "float32", n, count, env=SMALL)
    # two-shot: every GPU receives 2(N-1)/N of the buffer over NVLink
    assert a.sm_bytes == count * 4 * 2 * (n - 1)
    _, _, b = c.plan_simulate("ar_twoshot", "allreduce", "float32", n, count, host_ppm=2000,
                              env=SMALL)
    assert b.sm_bytes < a.sm_bytes and b.host_bytes > 0


def test_no_host_share_below_minimum():
    _, _, st = c.plan_simulate("ar_twoshot", "allreduce", "float32", 2, 1 << 20, host_ppm=2000)
    assert st.host_bytes == 0 and st.lanes == 0  # default minimum is 64 MiB per GPU


def mutation(algo, kind, n, host, ce, drop):
    L = c.lib()
    L.nb_plan_mutation.argtypes = [C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_int, C.c_int,
                                   C.c_char_p, C.c_int, C.c_char_p, C.c_size_t]
    buf = C.create_string_buffer(256)
    return L.nb_plan_mutation(c.ALGO[algo], c.KIND[kind], n, 1 << 20, host, ce,
                              c.env_spec(SMALL), drop, buf, 256)


@pytest.mark.parametrize("algo,kind", CASES[:7])
def test_checker_catches_every_dropped_wait(algo, kind):
    """Mutation self-test of the checker: in plans without host or CE shares
    every Wait is load-bearing, so deleting any one must be reported. The
    staged routes have two waits per rank that order nothing inside one call:
    the first scratch fill waits for the previous call's last fold
    (TempFree, ordering across calls), and the join's wait for the pull
    stream is implied by the folds' waits for their pulls."""
    n = 3
    i = missed = 0
    while True:
        r = mutation(algo, kind, n, 0, 0, i)
        if r < 0:
            break
        missed += r == 0
        i += 1
    assert i > 0
    assert missed == (2 * n if "staged" in algo else 0), (algo, missed)


def test_checker_catches_lane_reuse_bug():
    # With host lanes some waits are redundant, but most must still be caught.
    caught = total = 0
    while True:
        r = mutation("ar_twoshot", "allreduce", 2, 1500, 0, total)
        if r < 0:
            break
        caught += r
        total += 1
    assert total > 10 and caught > total // 2
