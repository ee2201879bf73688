"""ctypes bindings to the CUDA-free core library (libnb_core.so).

The enum values mirror src/core/types.h; they are checked against the
library's own name tables at import time.
"""
import ctypes as C
import functools

from . import CORE_PATH, require

# src/core/types.h
KIND = {"allreduce": 0, "allgather": 1, "reducescatter": 2, "broadcast": 3}
DTYPE = {"int8": 1, "uint8": 2, "int32": 3, "uint32": 4, "int64": 5, "uint64": 6,
         "float16": 7, "float32": 8, "float64": 9, "bfloat16": 10, "float8e4m3": 11,
         "float8e5m2": 12}
OP = {"sum": 0, "prod": 1, "max": 2, "min": 3, "avg": 4, "premulsum": 5, "unsupported": 6}
ALGO = {"fallback": 0, "ar_twoshot": 1, "ar_nvls": 2, "rs_pull": 3, "ag_pull": 4,
        "bc_pull": 5, "bc_scatter": 6, "ar_staged": 7, "rs_staged": 8, "bc_chain": 9,
        "bc_nvls": 10, "ag_nvls": 11, "rs_nvls": 12, "ag_push": 13, "bc_ring": 14,
        "rs_push": 15, "ar_push": 16, "ar_hybrid": 17, "ar_oneshot": 18,
        "rs_hybrid": 19, "ar_twoshot_ll": 20,
        "rs_ll": 21, "ag_ll": 22, "bc_ll": 23}
REASONS = ["None", "NotGrouped", "UnsupportedType", "UnsupportedOp", "NullBuffer",
           "SizeOverflow", "BelowThreshold", "Misaligned", "BadSlot", "PartialOverlap",
           "BadRank", "GroupShape", "NotClique", "Mismatch", "Capturing", "FirstPass",
           "SetupFailed", "SubmitFailedEarly", "Poisoned", "AboveLimit", "AddressOverflow",
           "PolicyFallback", "MetadataQuery", "RuntimeUnsupported", "UnsupportedNccl",
           "Disabled", "FaultInjected", "DeviceTimeout"]
REASON = {n: i for i, n in enumerate(REASONS)}
# clique flags for nb_gate_clique
KNOWN, CAPTURING, FIRST_PASS_DONE, POISONED, NCCL_UNSUPPORTED, NVLS = 1, 2, 4, 8, 16, 32


class Call(C.Structure):
    _fields_ = [("kind", C.c_int), ("dtype", C.c_int), ("op", C.c_int),
                ("count", C.c_uint64), ("send", C.c_uint64), ("recv", C.c_uint64),
                ("device", C.c_int), ("rank", C.c_int), ("nranks", C.c_int), ("root", C.c_int)]


class PlanStats(C.Structure):
    _fields_ = [("ops", C.c_uint64), ("records", C.c_uint64), ("waits", C.c_uint64),
                ("data_ops", C.c_uint64), ("sm_bytes", C.c_uint64), ("ce_bytes", C.c_uint64),
                ("host_bytes", C.c_uint64), ("lanes", C.c_int), ("bounce_bytes", C.c_uint64),
                ("phase_events", C.c_int), ("mismatches", C.c_uint64)]


@functools.lru_cache(maxsize=1)
def lib() -> C.CDLL:
    L = C.CDLL(require(CORE_PATH))
    L.nb_reason_name.restype = C.c_char_p
    L.nb_algo_name.restype = C.c_char_p
    L.nb_elem_size.restype = C.c_uint64
    L.nb_gate_message.argtypes = [C.POINTER(Call), C.c_char_p]
    L.nb_gate_call.argtypes = [C.POINTER(Call), C.c_char_p]
    L.nb_gate_clique.argtypes = [C.POINTER(Call), C.c_int, C.c_int, C.c_char_p, C.POINTER(C.c_int)]
    L.nb_plan_simulate.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64,
                                   C.c_int, C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_uint64,
                                   C.c_int, C.POINTER(C.c_double), C.POINTER(PlanStats),
                                   C.c_char_p, C.c_size_t]
    L.nb_host_fold.argtypes = [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p), C.c_int,
                               C.c_void_p, C.c_uint64, C.POINTER(C.c_double), C.c_int]
    L.nb_float_to_half.argtypes = [C.c_float]
    L.nb_float_to_half.restype = C.c_uint16
    L.nb_half_to_float.argtypes = [C.c_uint16]
    L.nb_half_to_float.restype = C.c_float
    L.nb_float_to_bf16.argtypes = [C.c_float]
    L.nb_float_to_bf16.restype = C.c_uint16
    L.nb_bf16_to_float.argtypes = [C.c_uint16]
    L.nb_bf16_to_float.restype = C.c_float
    L.nb_nvls_ar_round.argtypes = [C.c_uint64, C.c_uint64, C.c_int, C.c_uint,
                                   C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
    L.nb_policy_value.argtypes = [C.c_char_p, C.c_char_p]
    L.nb_policy_value.restype = C.c_double
    L.nb_shares_from.argtypes = [C.c_double] * 7 + [C.c_int, C.c_int, C.POINTER(C.c_int),
                                                   C.POINTER(C.c_int)]
    L.nb_calib_roundtrip.argtypes = [C.c_double, C.c_char_p, C.POINTER(C.c_double)]
    L.nb_group_script.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_char_p, C.c_size_t]
    L.nb_clique_add.argtypes = [C.POINTER(C.c_uint64), C.POINTER(C.c_int), C.c_int]
    L.nb_clique_forget.argtypes = [C.c_uint64]
    L.nb_clique_same.argtypes = [C.POINTER(C.c_uint64), C.c_int]
    L.nb_inits_form_clique.argtypes = [C.POINTER(C.c_int)] * 3 + [C.c_int]
    L.nb_fault_policy.argtypes = [C.c_char_p, C.c_int, C.c_uint64, C.POINTER(C.c_uint64),
                                  C.POINTER(C.c_uint64)]
    L.nb_summary_sample.argtypes = [C.c_char_p, C.c_size_t]
    # Enum tables must agree with the native ones.
    assert L.nb_reason_count() == len(REASONS)
    for i, n in enumerate(REASONS):
        assert L.nb_reason_name(i).decode() == n, (i, n)
    for n, i in ALGO.items():
        assert L.nb_algo_name(i).decode() == n, (i, n)
    return L


def call(kind="allreduce", dtype="float32", op="sum", count=1 << 24, send=1 << 32,
         recv=(1 << 32) + (1 << 31), device=0, rank=0, nranks=2, root=-1) -> Call:
    return Call(KIND[kind], DTYPE[dtype], OP[op], count, send, recv, device, rank, nranks, root)


def env_spec(env: dict | None) -> bytes:
    return ";".join(f"{k}={v}" for k, v in (env or {}).items()).encode()


def gate_call(c: Call, env=None) -> str:
    return REASONS[lib().nb_gate_call(C.byref(c), env_spec(env))]


def gate_message(c: Call, env=None) -> str:
    return REASONS[lib().nb_gate_message(C.byref(c), env_spec(env))]


def gate_clique(calls, flags, env=None):
    arr = (Call * len(calls))(*calls)
    algo = C.c_int(-1)
    r = lib().nb_gate_clique(arr, len(calls), flags, env_spec(env), C.byref(algo))
    inv = {v: k for k, v in ALGO.items()}
    return REASONS[r], inv[algo.value]


def plan_simulate(algo, kind, dtype, nranks, count, op="sum", root=0, inplace_mask=0,
                  host_ppm=0, ce_ppm=0, env=None, seed=0, data_mode=0, scalars=None):
    stats = PlanStats()
    err = C.create_string_buffer(512)
    sc = (C.c_double * 8)(*(scalars or [1.0] * 8)) if scalars else None
    rc = lib().nb_plan_simulate(ALGO[algo], KIND[kind], DTYPE[dtype], OP[op], nranks, count,
                                root, inplace_mask, host_ppm, ce_ppm, env_spec(env), seed,
                                data_mode, sc, C.byref(stats), err, 512)
    return rc, err.value.decode(), stats


def nvls_ar_rounds(nbytes: int, round_bytes: int, ramp: bool = True) -> list[tuple[int, int]]:
    """The NVLS AllReduce round schedule: [(base, len), ...]."""
    b, l = C.c_uint64(), C.c_uint64()
    n = lib().nb_nvls_ar_round(nbytes, round_bytes, int(ramp), 0, C.byref(b), C.byref(l))
    assert n >= 0
    out = []
    for s in range(n):
        lib().nb_nvls_ar_round(nbytes, round_bytes, int(ramp), s, C.byref(b), C.byref(l))
        out.append((b.value, l.value))
    return out


def group_script(script: str, nranks: int, run_result: int = 0) -> list[str]:
    buf = C.create_string_buffer(1 << 16)
    n = lib().nb_group_script(script.encode(), nranks, run_result, buf, 1 << 16)
    assert n >= 0, "bad script"
    return buf.value.decode().splitlines()


def policy_value(env: dict | None, field: str) -> float:
    return lib().nb_policy_value(env_spec(env), field.encode())
