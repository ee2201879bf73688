"""Independent route oracle: which grouped calls the interposer runs itself,
and on which route, restated in Python from the routing rules.

The stress harness compares this prediction with the route the library
reports running (its per-route counters), so a regression in the library's
gate or route choice shows up as a disagreement instead of being reported
back as correct by the library itself.

Restated rules (the C++ originals are src/core/gate.cc and
src/core/calib_model.cc):

* Message gate, in order: the element type has a size; reductions need a
  reducible type and an op the type supports (PreMulSum only for floating
  types); the byte size fits; the logical message (nccl-tests
  "size": N slots for AllGather/ReduceScatter) is at most the cap
  (NCCL_B200_MAX_BYTES, 8 GiB); the library and the kind are enabled; the
  logical message reaches the kind's threshold (NCCL_B200_{AR,AG,RS,BC}_MIN,
  32 MiB, or, when unset, the crossover with NCCL measured at init and kept
  in the calibration record) and is not empty; a ReduceScatter slot is a multiple of 16 bytes.
* Route: a forced route (NCCL_B200_ALGO) when it is valid for the call; else
  the tuned route of the message's size band (tiny, small or large, from a
  calibration cache file) when valid; else the static rule (AllReduce: NVLS
  from 4 ranks when the switch offers multicast, else two-shot;
  ReduceScatter: pull; AllGather: pull; Broadcast: scatter from 3 ranks,
  else pull). A switch route needs 16-byte aligned buffers and, for
  PreMulSum, one host scalar for every rank; otherwise the static non-switch
  route runs (a payload that is not a whole number of 16-byte vectors counts
  as unaligned). An in-place one-shot AllReduce runs the two-shot plan.

Counterpart: expect_route in the reference's tests/stress_check.cu:348-357,
which restates its gate_message for the stress cases.
"""
from __future__ import annotations

import json
import os

KIB, MIB, GIB = 1 << 10, 1 << 20, 1 << 30
ELEM = {"int8": 1, "uint8": 1, "int32": 4, "uint32": 4, "int64": 8, "uint64": 8, "float16": 2,
        "float32": 4, "float64": 8, "bfloat16": 2, "float8e4m3": 1, "float8e5m2": 1}
REDUCIBLE = {"int8", "uint8", "int32", "uint32", "int64", "uint64", "float16", "float32",
             "float64", "bfloat16"}
FLOATS = {"float16", "float32", "float64", "bfloat16"}
SWITCH_TYPES = {"float32", "float16", "bfloat16"}
KEYS = {"allreduce": "AR", "allgather": "AG", "reducescatter": "RS", "broadcast": "BC"}
KIND_ENV = {"allreduce": "ALLREDUCE", "allgather": "ALLGATHER", "reducescatter": "REDUCESCATTER",
            "broadcast": "BROADCAST"}
KIND_INDEX = {"allreduce": 0, "allgather": 1, "reducescatter": 2, "broadcast": 3}
# Route names of the NCCL_B200_ALGO syntax, per kind.
FORCE_NAMES = {
    "allreduce": {"twoshot": "ar_twoshot", "oneshot": "ar_oneshot", "nvls": "ar_nvls",
                  "staged": "ar_staged", "push": "ar_push", "hybrid": "ar_hybrid",
                  "twoshot_ll": "ar_twoshot_ll"},
    "reducescatter": {"pull": "rs_pull", "staged": "rs_staged", "nvls": "rs_nvls", "push": "rs_push",
                      "hybrid": "rs_hybrid", "ll": "rs_ll"},
    "allgather": {"pull": "ag_pull", "nvls": "ag_nvls", "push": "ag_push", "ll": "ag_ll"},
    "broadcast": {"pull": "bc_pull", "scatter": "bc_scatter", "chain": "bc_chain", "nvls": "bc_nvls",
                  "ring": "bc_ring", "ll": "bc_ll"},
}
SWITCH_ROUTES = {"ar_nvls", "bc_nvls", "ag_nvls", "rs_nvls", "ar_hybrid", "rs_hybrid"}
ALGO_IDS = ["fallback", "ar_twoshot", "ar_nvls", "rs_pull", "ag_pull", "bc_pull", "bc_scatter",
            "ar_staged", "rs_staged", "bc_chain", "bc_nvls", "ag_nvls", "rs_nvls", "ag_push", "bc_ring",
            "rs_push", "ar_push", "ar_hybrid", "ar_oneshot", "rs_hybrid", "ar_twoshot_ll", "rs_ll",
            "ag_ll", "bc_ll"]


def parse_size(s: str | None) -> int | None:
    if s is None or s == "":
        return None
    t = s.strip()
    mul = {"K": KIB, "M": MIB, "G": GIB}.get(t[-1:].upper(), 1)
    if mul > 1:
        t = t[:-1]
    try:
        return int(t) * mul
    except ValueError:
        return None


def parse_bool(s: str | None) -> bool | None:
    if s is None:
        return None
    if s in ("1", "true", "on", "yes"):
        return True
    if s in ("0", "false", "off", "no"):
        return False
    return None


class Rules:
    """The routing policy as the environment sets it."""

    def __init__(self, env: dict | None = None):
        env = dict(os.environ if env is None else env)
        g = env.get
        self.enabled = not parse_bool(g("NCCL_B200_DISABLE"))
        self.kind_enabled = {k: parse_bool(g("NCCL_B200_" + v)) is not False for k, v in KIND_ENV.items()}
        self.min_set = {k: parse_size(g(f"NCCL_B200_{v}_MIN")) is not None for k, v in KEYS.items()}
        self.min_bytes = {k: parse_size(g(f"NCCL_B200_{v}_MIN")) or 32 * MIB for k, v in KEYS.items()}
        self.max_bytes = parse_size(g("NCCL_B200_MAX_BYTES")) or 8 * GIB
        nv = g("NCCL_B200_NVLS", "auto")
        self.nvls = "off" if nv in ("0", "off") else ("on" if nv in ("1", "on") else "auto")
        self.nvls_min_ranks = int(g("NCCL_B200_NVLS_MIN_RANKS", "4"))
        self.forced = {}
        for item in (g("NCCL_B200_ALGO") or "").split(","):
            if "=" not in item:
                continue
            k, a = item.split("=", 1)
            kind = {"ar": "allreduce", "ag": "allgather", "rs": "reducescatter", "bc": "broadcast"}.get(k, k)
            if kind in FORCE_NAMES and a in FORCE_NAMES[kind]:
                self.forced[kind] = FORCE_NAMES[kind][a]
            elif kind in FORCE_NAMES and a in ("nccl", "fallback"):
                self.forced.pop(kind, None)


def logical_bytes(kind: str, dtype: str, count: int, n: int) -> int:
    b = count * ELEM.get(dtype, 0)
    return b * n if kind in ("allgather", "reducescatter") else b


def gate_message(kind: str, dtype: str, op: str, count: int, n: int, rules: Rules) -> str:
    """The fallback reason of the message gate, or "None"."""
    es = ELEM.get(dtype, 0)
    if es == 0:
        return "UnsupportedType"
    red = kind in ("allreduce", "reducescatter")
    if red and dtype not in REDUCIBLE:
        return "UnsupportedType"
    if red and not (op in ("sum", "prod", "max", "min", "avg") or (op == "premulsum" and dtype in FLOATS)):
        return "UnsupportedOp"
    if count > ((1 << 64) - 1) // 4 // es // max(1, n):
        return "SizeOverflow"
    logical = logical_bytes(kind, dtype, count, n)
    if logical > rules.max_bytes:
        return "AboveLimit"
    if not rules.enabled:
        return "Disabled"
    if not rules.kind_enabled[kind]:
        return "PolicyFallback"
    if logical < rules.min_bytes[kind] or count == 0:
        return "BelowThreshold"
    if kind == "reducescatter" and (count * es) % 16:
        return "BadSlot"
    return "None"


def valid(route: str, kind: str, n: int, dtype: str, op: str, nvls: bool) -> bool:
    switch_op = op in ("sum", "avg", "premulsum")
    table = {
        "ar_twoshot": kind == "allreduce",
        "ar_oneshot": kind == "allreduce" and n >= 2 and dtype in SWITCH_TYPES,
        "ar_twoshot_ll": kind == "allreduce" and n >= 2 and dtype in SWITCH_TYPES,
        "rs_ll": kind == "reducescatter" and n >= 2 and dtype in SWITCH_TYPES,
        "ag_ll": kind == "allgather" and n >= 2,
        "bc_ll": kind == "broadcast" and n >= 2,
        "ar_nvls": kind == "allreduce" and nvls and n >= 2 and dtype in SWITCH_TYPES and switch_op,
        "ar_hybrid": False,  # refused by the library (wrong data at 4 GiB, measured)
        "ar_staged": kind == "allreduce",
        "ar_push": kind == "allreduce" and n >= 2 and dtype in SWITCH_TYPES,
        "rs_pull": kind == "reducescatter",
        "rs_staged": kind == "reducescatter",
        "rs_push": kind == "reducescatter" and n >= 2 and dtype in SWITCH_TYPES,
        "rs_nvls": kind == "reducescatter" and nvls and n >= 2 and dtype in SWITCH_TYPES and switch_op,
        "rs_hybrid": False,
        "ag_pull": kind == "allgather",
        "ag_push": kind == "allgather",
        "ag_nvls": kind == "allgather" and nvls and n >= 2,
        "bc_pull": kind == "broadcast",
        "bc_scatter": kind == "broadcast" and n >= 3,
        "bc_chain": kind == "broadcast",
        "bc_ring": kind == "broadcast" and n >= 2,
        "bc_nvls": kind == "broadcast" and nvls and n >= 2,
    }
    return table.get(route, False)


def static_route(kind: str, n: int, dtype: str, op: str, nvls: bool, rules: Rules) -> str:
    if kind == "allreduce":
        use = rules.nvls != "off" and (rules.nvls == "on" or n >= rules.nvls_min_ranks) and \
            valid("ar_nvls", kind, n, dtype, op, nvls)
        return "ar_nvls" if use else "ar_twoshot"
    if kind == "reducescatter":
        return "rs_pull"
    if kind == "allgather":
        return "ag_pull"
    return "bc_scatter" if n >= 3 else "bc_pull"


def tuned_route(calib: dict | None, kind: str, logical: int) -> str | None:
    """The tuned route for a message of `logical` bytes from a calibration
    cache record (the JSON the library writes), by size band."""
    if not calib:
        return None
    k = KIND_INDEX[kind]
    tiny = int(calib.get("tiny_below_kib", 0))
    small = int(calib.get("small_below_mib", 0))
    pick = 0
    if tiny > 0 and logical < tiny * KIB and int(calib.get(f"tpref{k}", 0)):
        pick = int(calib[f"tpref{k}"])
    elif small > 0 and logical < small * MIB and int(calib.get(f"spref{k}", 0)):
        pick = int(calib[f"spref{k}"])
    else:
        pick = int(calib.get(f"pref{k}", 0))
    return ALGO_IDS[pick] if 0 < pick < len(ALGO_IDS) else None


def load_calib(path: str | None, key_hint: str = "") -> dict | None:
    """The last calibration record in a cache file (one JSON object per line)."""
    if not path or not os.path.exists(path):
        return None
    rec = None
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line.startswith("{") and key_hint in line:
                try:
                    rec = json.loads(line)
                except ValueError:
                    continue
    return rec


def expected_route(kind: str, dtype: str, op: str, count: int, n: int, *, inplace: bool = False,
                   aligned: bool = True, uniform_scalar: bool = True, nvls: bool = False,
                   rules: Rules | None = None, calib: dict | None = None) -> str:
    """"nccl" when the call falls back, else the route that runs it."""
    rules = rules or Rules()
    engage = int((calib or {}).get(f"engage{KIND_INDEX[kind]}", 0))
    if engage > 0 and not rules.min_set[kind] and n > 1:
        # The measured crossover with NCCL lowers an unset threshold.
        import copy
        rules = copy.copy(rules)
        rules.min_bytes = dict(rules.min_bytes)
        rules.min_bytes[kind] = min(rules.min_bytes[kind], engage * KIB)
    if gate_message(kind, dtype, op, count, n, rules) != "None":
        return "nccl"
    logical = logical_bytes(kind, dtype, count, n)
    route = None
    forced = rules.forced.get(kind)
    if forced and valid(forced, kind, n, dtype, op, nvls):
        route = forced
    if route is None:
        t = tuned_route(calib, kind, logical)
        if t and valid(t, kind, n, dtype, op, nvls):
            route = t
    if route is None:
        route = static_route(kind, n, dtype, op, nvls, rules)
    # The multimem kernels move whole 16-byte vectors: every buffer and every
    # rank's payload must be 16-byte aligned.
    aligned = aligned and (count * ELEM[dtype]) % 16 == 0
    if route in SWITCH_ROUTES and (not aligned or (op == "premulsum" and not uniform_scalar)):
        route = static_route(kind, n, dtype, op, False, rules)
    # So do the low-latency AllGather and Broadcast copies.
    if route in ("ag_ll", "bc_ll") and not aligned:
        route = static_route(kind, n, dtype, op, False, rules)
    if route == "ar_oneshot" and inplace and n > 1:
        route = "ar_twoshot_ll"
    return route
