"""The independent route oracle (parallel/oracle.py) against the library's
own gate on CPU: for a grid of calls, the oracle's fallback-or-route answer
must equal what the C++ clique gate decides. A disagreement means one of the
two restatements drifted."""
import itertools

import pytest

from scc26_nccl_shim_b200 import _core as c
from scc26_nccl_shim_b200.parallel import oracle

KINDS = ["allreduce", "allgather", "reducescatter", "broadcast"]


def library_route(kind, dtype, op, count, n, env, nvls, inplace=False, aligned=True):
    calls = []
    base = 1 << 40
    es = oracle.ELEM[dtype]
    slot = count * es
    for r in range(n):
        send = base + r * (1 << 36)
        recv = send + (1 << 35)
        if inplace:
            recv = send
            if kind == "allgather":
                send = recv + r * slot
            elif kind == "reducescatter":
                recv = send + r * slot
        if not aligned:
            send += 4
            recv += 4
        calls.append(c.call(kind=kind, dtype=dtype, op=op, count=count, send=send, recv=recv, device=r,
                            rank=r, nranks=n, root=0))
    flags = c.KNOWN | c.FIRST_PASS_DONE | (c.NVLS if nvls else 0)
    reason, algo = c.gate_clique(calls, flags, env)
    if reason != "None":
        return "nccl"
    return algo


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("nvls", [False, True])
def test_oracle_matches_library_gate(n, nvls):
    envs = [{}, {"NCCL_B200_AR_MIN": "1M", "NCCL_B200_RS_MIN": "64K"},
            {"NCCL_B200_ALGO": "ar=oneshot,rs=push,ag=push,bc=ring", "NCCL_B200_AR_MIN": "4K"},
            {"NCCL_B200_ALGO": "ar=hybrid,rs=hybrid,ag=nvls,bc=nvls"},
            {"NCCL_B200_ALGO": "ar=twoshot_ll,rs=ll,ag=ll,bc=ll", "NCCL_B200_AR_MIN": "4K",
             "NCCL_B200_AG_MIN": "4K", "NCCL_B200_RS_MIN": "4K", "NCCL_B200_BC_MIN": "4K"},
            {"NCCL_B200_NVLS": "off"}, {"NCCL_B200_MAX_BYTES": "64M"},
            {"NCCL_B200_ALLGATHER": "0"}, {"NCCL_B200_DISABLE": "1"}]
    counts = [0, 1, 1023, (32 << 20) // 4 - 1, (32 << 20) // 4, (32 << 20) // 4 + 3, (40 << 20) // 4,
              (2 << 30) // 4, (8 << 30) // 4, (8 << 30) // 4 + 1]
    checked = 0
    for env, kind, dtype, op, count in itertools.product(
            envs, KINDS, ["float32", "bfloat16", "int32", "int8", "float8e4m3"],
            ["sum", "avg", "max", "prod"], counts):
        if kind not in ("allreduce", "reducescatter") and op != "sum":
            continue
        if kind in ("allgather", "reducescatter") and count:
            count = max(1, count // n)
        want = oracle.expected_route(kind, dtype, op, count, n, nvls=nvls, rules=oracle.Rules(env))
        got = library_route(kind, dtype, op, count, n, env, nvls)
        assert got == want, (env, kind, dtype, op, count, n, nvls)
        checked += 1
    assert checked > 500


@pytest.mark.parametrize("n", [2, 4, 8])
def test_oracle_switch_and_inplace_substitutions(n):
    env = {"NCCL_B200_ALGO": "ar=nvls,rs=nvls", "NCCL_B200_AR_MIN": "1K", "NCCL_B200_RS_MIN": "1K"}
    for kind in ("allreduce", "reducescatter"):
        count = 1 << 20
        want = oracle.expected_route(kind, "float32", "sum", count, n, nvls=True, aligned=False,
                                     rules=oracle.Rules(env))
        got = library_route(kind, "float32", "sum", count, n, env, True, aligned=False)
        # Misaligned buffers fail the call gate for reductions before any route choice.
        assert got == "nccl" and want in ("ar_twoshot", "rs_pull")
    env = {"NCCL_B200_ALGO": "ar=oneshot", "NCCL_B200_AR_MIN": "1K"}
    assert oracle.expected_route("allreduce", "float32", "sum", 1 << 20, n, inplace=True,
                                 rules=oracle.Rules(env)) == "ar_twoshot_ll"
    assert oracle.expected_route("allreduce", "float32", "sum", 1 << 20, n, inplace=False,
                                 rules=oracle.Rules(env)) == "ar_oneshot"


def test_tuned_bands_from_a_cache_record():
    rec = {"pref0": 2, "spref0": 1, "tpref0": 18, "small_below_mib": 512, "tiny_below_kib": 16384}
    assert oracle.tuned_route(rec, "allreduce", 8 << 30) == "ar_nvls"
    assert oracle.tuned_route(rec, "allreduce", 100 << 20) == "ar_twoshot"
    assert oracle.tuned_route(rec, "allreduce", 1 << 20) == "ar_oneshot"
    assert oracle.expected_route("allreduce", "float32", "sum", (1 << 20) // 4, 4, nvls=True,
                                 rules=oracle.Rules({"NCCL_B200_AR_MIN": "512K"}), calib=rec) == "ar_oneshot"


def test_measured_crossover_lowers_unset_thresholds_only():
    rec = {"pref0": 1, "engage0": 256}
    small = (512 << 10) // 4
    assert oracle.expected_route("allreduce", "float32", "sum", small, 2, calib=rec,
                                 rules=oracle.Rules({})) == "ar_twoshot"
    assert oracle.expected_route("allreduce", "float32", "sum", (128 << 10) // 4, 2, calib=rec,
                                 rules=oracle.Rules({})) == "nccl"
    # An explicit threshold wins over the measurement.
    assert oracle.expected_route("allreduce", "float32", "sum", small, 2, calib=rec,
                                 rules=oracle.Rules({"NCCL_B200_AR_MIN": "32M"})) == "nccl"


@pytest.mark.parametrize("n", [2, 4, 8])
def test_oracle_low_latency_copies_need_whole_vectors(n):
    """The low-latency AllGather/Broadcast copies move whole 16-byte vectors:
    an odd payload or a misaligned buffer takes the static route, in the
    library and in the oracle alike."""
    env = {"NCCL_B200_ALGO": "ag=ll,bc=ll", "NCCL_B200_AG_MIN": "1", "NCCL_B200_BC_MIN": "1"}
    rules = oracle.Rules(env)
    for kind in ("allgather", "broadcast"):
        for count, aligned in (((1 << 20) // 4, True), ((1 << 20) // 4 + 1, True), ((1 << 20) // 4, False)):
            want = oracle.expected_route(kind, "float32", "sum", count, n, aligned=aligned, rules=rules)
            got = library_route(kind, "float32", "sum", count, n, env, False, aligned=aligned)
            assert got == want, (kind, count, aligned, got, want)
            assert (want in ("ag_ll", "bc_ll")) == (aligned and count % 4 == 0), (kind, count, aligned, want)
