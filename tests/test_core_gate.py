"""Gates (message, call, clique) of the pure core, on the CPU."""
import pytest

from scc26_nccl_shim_b200 import _core as c

MiB = 1 << 20


def test_eligible_allreduce():
    assert c.gate_call(c.call()) == "None"


@pytest.mark.parametrize("kw,reason", [
    (dict(count=1000), "BelowThreshold"),
    (dict(dtype="float8e4m3"), "UnsupportedType"),
    (dict(op="unsupported"), "UnsupportedOp"),
    (dict(dtype="int32", op="premulsum"), "UnsupportedOp"),
    (dict(send=0), "NullBuffer"),
    (dict(recv=0), "NullBuffer"),
    (dict(send=(1 << 32) + 4), "Misaligned"),
    (dict(rank=2), "BadRank"),
    (dict(nranks=9, rank=0), "BadRank"),
    (dict(count=(9 << 30) // 4), "AboveLimit"),
    (dict(send=(1 << 64) - 4096, recv=1 << 32, count=16 << 20), "AddressOverflow"),
    (dict(send=1 << 32, recv=(1 << 32) + 4096), "PartialOverlap"),
])
def test_call_rejections(kw, reason):
    assert c.gate_call(c.call(**kw)) == reason


def test_in_place_layouts_accepted():
    n = 16 << 20
    # AllReduce: send == recv
    assert c.gate_call(c.call(send=1 << 32, recv=1 << 32)) == "None"
    # AllGather: send == recv + rank * n * elem
    assert c.gate_call(c.call(kind="allgather", count=n, rank=1, recv=1 << 32,
                              send=(1 << 32) + n * 4)) == "None"
    # ReduceScatter: recv == send + rank * n * elem
    assert c.gate_call(c.call(kind="reducescatter", count=n, rank=1, send=1 << 32,
                              recv=(1 << 32) + n * 4)) == "None"
    # off by one element is a partial overlap
    assert c.gate_call(c.call(kind="allgather", count=n, rank=1, recv=1 << 32,
                              send=(1 << 32) + n * 4 + 16)) == "PartialOverlap"


def test_reducescatter_slot_alignment():
    assert c.gate_call(c.call(kind="reducescatter", count=(16 << 20) + 1)) == "BadSlot"
    assert c.gate_call(c.call(kind="reducescatter", count=(16 << 20) + 4)) == "None"


def test_broadcast_nonroot_send_ignored():
    assert c.gate_call(c.call(kind="broadcast", send=0, rank=1, root=0)) == "None"
    assert c.gate_call(c.call(kind="broadcast", send=0, rank=0, root=0)) == "NullBuffer"
    assert c.gate_call(c.call(kind="broadcast", root=5)) == "BadRank"


def test_copy_collectives_need_no_alignment():
    assert c.gate_call(c.call(kind="allgather", count=(16 << 20) + 1, send=(1 << 32) + 2)) == "None"


def test_logical_size_threshold_uses_all_slots():
    # 8 ranks x 4 MiB slots = 32 MiB logical: at the default 32 MiB threshold.
    assert c.gate_call(c.call(kind="allgather", count=MiB, nranks=8, rank=3)) == "None"
    assert c.gate_call(c.call(kind="allgather", count=MiB, nranks=4, rank=3)) == "BelowThreshold"


def test_policy_overrides():
    assert c.gate_call(c.call(), {"NCCL_B200_DISABLE": "1"}) == "Disabled"
    assert c.gate_call(c.call(), {"NCCL_B200_ALLREDUCE": "0"}) == "PolicyFallback"
    assert c.gate_call(c.call(count=1000), {"NCCL_B200_AR_MIN": "1K"}) == "None"
    assert c.gate_call(c.call(count=(9 << 30) // 4, send=1 << 36, recv=1 << 38),
                       {"NCCL_B200_MAX_BYTES": "16G"}) == "None"


def clique_calls(n, **kw):
    return [c.call(device=d, rank=d, nranks=n, **kw) for d in range(n)]


def test_clique_gate_order():
    calls = clique_calls(2)
    F = c.KNOWN | c.FIRST_PASS_DONE
    assert c.gate_clique(calls, F) == ("None", "ar_twoshot")
    assert c.gate_clique(calls, F | c.POISONED) == ("Poisoned", "fallback")
    assert c.gate_clique(calls, F | c.NCCL_UNSUPPORTED) == ("UnsupportedNccl", "fallback")
    assert c.gate_clique(calls, c.FIRST_PASS_DONE) == ("NotClique", "fallback")
    assert c.gate_clique(calls, F | c.CAPTURING) == ("Capturing", "fallback")
    assert c.gate_clique(calls, c.KNOWN) == ("FirstPass", "fallback")
    assert c.gate_clique(calls, c.KNOWN, {"NCCL_B200_FIRST_PASS": "0"}) == ("None", "ar_twoshot")


def test_clique_gate_shapes():
    F = c.KNOWN | c.FIRST_PASS_DONE
    calls = clique_calls(3)
    assert c.gate_clique(calls[:2], F)[0] == "NotClique"  # 2 calls for 3 ranks
    dup = clique_calls(2)
    dup[1].rank = 0
    assert c.gate_clique(dup, F)[0] == "NotClique"
    dupdev = clique_calls(2)
    dupdev[1].device = 0
    assert c.gate_clique(dupdev, F)[0] == "NotClique"
    mis = clique_calls(2)
    mis[1].count += 4
    assert c.gate_clique(mis, F)[0] == "Mismatch"
    mis = clique_calls(2)
    mis[1].dtype = c.DTYPE["bfloat16"]
    assert c.gate_clique(mis, F)[0] == "Mismatch"
    bc = clique_calls(2, kind="broadcast", root=0)
    bc[1].root = 1
    assert c.gate_clique(bc, F)[0] == "Mismatch"
    bad = clique_calls(2)
    bad[1].send += 4
    assert c.gate_clique(bad, F)[0] == "Misaligned"


@pytest.mark.parametrize("n,kind,flags,algo", [
    (2, "allreduce", 0, "ar_twoshot"),
    (2, "allreduce", c.NVLS, "ar_twoshot"),   # NVLS only from 4 ranks by default
    (4, "allreduce", c.NVLS, "ar_nvls"),
    (8, "allreduce", c.NVLS, "ar_nvls"),
    (8, "allreduce", 0, "ar_twoshot"),
    (4, "reducescatter", c.NVLS, "rs_pull"),
    (4, "allgather", 0, "ag_pull"),
    (2, "broadcast", 0, "bc_pull"),
    (3, "broadcast", 0, "bc_scatter"),
    (8, "broadcast", 0, "bc_scatter"),
])
def test_algorithm_choice(n, kind, flags, algo):
    kw = dict(kind=kind)
    if kind == "broadcast":
        kw["root"] = 0
    if kind in ("allgather", "reducescatter"):
        kw["count"] = 16 << 20
    calls = clique_calls(n, **kw)
    assert c.gate_clique(calls, c.KNOWN | c.FIRST_PASS_DONE | flags) == ("None", algo)


def test_nvls_only_for_sum_and_avg_of_floats():
    calls = clique_calls(4, op="max")
    assert c.gate_clique(calls, c.KNOWN | c.FIRST_PASS_DONE | c.NVLS) == ("None", "ar_twoshot")
    calls = clique_calls(4, dtype="bfloat16", op="avg")
    assert c.gate_clique(calls, c.KNOWN | c.FIRST_PASS_DONE | c.NVLS) == ("None", "ar_nvls")


def test_nvls_premulsum_needs_one_host_scalar():
    import ctypes as C
    L = c.lib()
    L.nb_gate_clique_scalars.argtypes = [C.POINTER(c.Call), C.c_int, C.c_int, C.c_char_p,
                                         C.POINTER(C.c_int), C.POINTER(C.c_double), C.POINTER(C.c_int)]
    inv = {v: k for k, v in c.ALGO.items()}

    def gate(scalars, residence):
        calls = clique_calls(4, dtype="bfloat16", op="premulsum")
        arr = (c.Call * 4)(*calls)
        algo = C.c_int(-1)
        r = L.nb_gate_clique_scalars(arr, 4, c.KNOWN | c.FIRST_PASS_DONE | c.NVLS, b"", C.byref(algo),
                                     (C.c_double * 4)(*scalars), (C.c_int * 4)(*residence))
        return c.REASONS[r], inv[algo.value]
    # One shared host scalar (e.g. 1/N): the switch's sum is scaled once.
    assert gate([0.25] * 4, [1] * 4) == ("None", "ar_nvls")
    # Per-rank scalars, or a scalar in device memory: the fused P2P fold.
    assert gate([0.25, 0.5, 0.25, 0.25], [1] * 4) == ("None", "ar_twoshot")
    assert gate([0.25] * 4, [1, 0, 1, 1]) == ("None", "ar_twoshot")


def test_forced_algorithm():
    calls = clique_calls(8)
    env = {"NCCL_B200_ALGO": "ar=twoshot,bc=pull"}
    assert c.gate_clique(calls, c.KNOWN | c.FIRST_PASS_DONE | c.NVLS, env) == ("None", "ar_twoshot")
    calls = clique_calls(4)
    env = {"NCCL_B200_ALGO": "allreduce=nvls"}
    # forcing NVLS without multicast support is ignored
    assert c.gate_clique(calls, c.KNOWN | c.FIRST_PASS_DONE, env) == ("None", "ar_twoshot")
    env = {"NCCL_B200_ALGO": "ar=nccl"}
    assert c.gate_clique(calls, c.KNOWN | c.FIRST_PASS_DONE, env)[1] == "ar_twoshot"


def test_policy_parsing():
    assert c.policy_value({"NCCL_B200_AR_MIN": "64M"}, "ar_min") == 64 << 20
    assert c.policy_value({"NCCL_B200_AR_MIN": "2GiB"}, "ar_min") == 2 << 30
    assert c.policy_value({"NCCL_B200_AR_MIN": "junk"}, "ar_min") == 32 << 20
    assert c.policy_value({"NCCL_SHIM_SUMMARY": "1"}, "summary") == 1
    assert c.policy_value({"NCCL_SHIM_SUMMARY": "yes"}, "summary") == 0
    assert c.policy_value({"NCCL_B200_NVLS": "0"}, "nvls") == 0
    assert c.policy_value({"NCCL_B200_LANES": "99"}, "lanes") == 4
    assert c.policy_value({"NCCL_B200_HOST_PIECE": "1000"}, "host_piece") == 16 << 20  # not 16B-aligned
    assert c.policy_value({"NCCL_B200_TIMEOUT_MS": "250"}, "timeout_ns") == 250e6
    assert c.policy_value({"NCCL_B200_ALGO": "bc=scatter"}, "force_bc") == c.ALGO["bc_scatter"]


def test_policy_parsing_of_engine_knobs():
    A = c.ALGO
    env = {"NCCL_B200_ALGO": "ar=hybrid,ag=push,rs=push,bc=ring"}
    assert c.policy_value(env, "force_ar") == A["ar_hybrid"]
    assert c.policy_value(env, "force_ag") == A["ag_push"]
    assert c.policy_value(env, "force_rs") == A["rs_push"]
    assert c.policy_value(env, "force_bc") == A["bc_ring"]
    assert c.policy_value({"NCCL_B200_RING_CHUNK": "64K"}, "ring_chunk") == 64 << 10
    assert c.policy_value({"NCCL_B200_RING_CHUNK": "100"}, "ring_chunk") == 256 << 10  # not a 32-byte multiple
    assert c.policy_value({"NCCL_B200_HYBRID_NVLS_PPM": "5000"}, "hybrid_nvls_ppm") == 5000
    assert c.policy_value({"NCCL_B200_HYBRID_NVLS_PPM": "9500"}, "hybrid_nvls_ppm") == 6000
    assert c.policy_value({"NCCL_B200_HYBRID_BLOCKS": "100"}, "hybrid_blocks") == 100
    assert c.policy_value({}, "nvls_tma") == 1
    assert c.policy_value({"NCCL_B200_NVLS_TMA": "0"}, "nvls_tma") == 0
    assert c.policy_value({}, "nvls_ramp") == 0
    assert c.policy_value({}, "nvls_strong") == 1
    assert c.policy_value({}, "nvls_buffers") == 0  # 0: one per round of the largest message
    assert c.policy_value({"NCCL_B200_NVLS_BUFFERS": "8"}, "nvls_buffers") == 8
    assert c.policy_value({"NCCL_B200_NVLS_BUFFERS": "2"}, "nvls_buffers") == 0  # at least 3
    assert c.policy_value({"NCCL_B200_NVLS_RAMP": "1"}, "nvls_ramp") == 1
    assert c.policy_value({"NCCL_B200_NVLS_TRACE": "1", "NCCL_B200_NVTX": "on"}, "nvls_trace") == 1
    assert c.policy_value({"NCCL_B200_NVTX": "on"}, "nvtx") == 1
    assert c.policy_value({"NCCL_B200_NVLS_MOVERS": "384"}, "nvls_movers") == 384
    assert c.policy_value({"NCCL_B200_NVLS_MOVERS": "400"}, "nvls_movers") == 512  # not a warp multiple
    assert c.policy_value({}, "tune_bytes") == 4 << 30
