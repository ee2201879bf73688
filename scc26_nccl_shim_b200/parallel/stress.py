"""Back-to-back stress, differential and boundary harness for the interposer.

Every iteration of a back-to-back loop is checked, with no host
synchronization until the end of a case: per iteration and per GPU stream,
inputs are regenerated (exactly-summable hashed values that depend on rank,
index and iteration), the grouped collective runs through the interposed NCCL
ABI, and the output is compared bit for bit on the device, accumulating a
mismatch count. If the interposer let a rank return while a peer still read
its send buffer or wrote its receive buffer, the next iteration's input
regeneration or this iteration's check sees it.

Guards: every send and receive buffer sits between two 4096-byte guard
regions filled with 0xA5 inside one allocation; they are checked after the
case, so a write one element past an odd tail or before a slot fails it.

Differential mode (--diff): adversarial bit patterns (every exponent,
subnormals, signed zeros, infinities, the largest binade, near-negations
across ranks; NaNs for copy collectives). Each iteration first runs the same
collective through libnccl's own entry points (the real library handle,
bypassing the interposer) into shadow buffers, then through the interposer,
and compares bitwise. For reductions the interposer folds in rank order in
fp32 while NCCL's order is its own, so reductions are compared with a
tolerance in differential mode (exact data stays bitwise); positions where
both are NaN are skipped for reductions, never for copies.

Mutation self-test (--corrupt-shift K): rank 0's output is displaced by K
elements before the check; every affected case must FAIL, proving that the
checker can fail.

Ordering controls: --delay-input-device D holds rank D's caller stream
(a bounded sleep kernel) before every call, so a rank that read a peer's
input without waiting for it would see stale data; --overwrite-after
overwrites every input on its caller stream right after the call, which is
safe only if the call's side streams were joined back into the caller
streams; --fresh-streams issues every iteration on new caller streams.

Route oracle: every case also states the route an independent restatement
of the routing rules predicts (parallel/oracle.py); the route the library
reports running must match it, or the case FAILs with status ROUTE.
--oracle-drop VAR hides one variable from the oracle only (the library still
reads it), which must turn affected cases into ROUTE failures: the route
check's own mutation test.

Case sets: the standard cases (every kind, fp32/bf16/fp16, in and out of
place, odd tails, int types, every reduction op including avg and
PreMulSum); boundary cases (-1/0/+1 element around each kind's threshold);
--edges: the pipeline edges of the engines (NVLS round, push-reduce piece
round, push-chain step, host-lane piece) at -1/0/+1 vector; --big: the
2 GiB, 4 GiB and 8 GiB logical-size edges, the last at the message cap and
one element above it (which must fall back). Data for the large cases are
generated and checked in chunks.

Output: one TSV row per case:
  case iters bytes mismatches status guard_bad route expect kind mode
Parity: tests/stress_check.cu of the reference (two GPUs, fixed thresholds).
"""
from __future__ import annotations

import argparse
import os
import sys
from dataclasses import dataclass

import torch

from .._core import ALGO, policy_value
from ..utils.data import adversarial, exact
from . import oracle
from .nccl import Nccl, collective

GUARD = 4096
PATTERN = 0xA5
CHUNK = 64 << 20  # elements generated / checked at a time
DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16,
          "int32": torch.int32, "int8": torch.int8}


@dataclass
class Case:
    name: str
    kind: str
    dtype: str
    count: int          # AG send count / RS recv count / element count
    inplace: bool = False
    root: int = 0
    op: str = "sum"


def standard_cases(n: int, scale: int = 1) -> list[Case]:
    M = 1 << 20
    base = (48 * M) // 4 // scale
    cases = []
    for kind in ("allreduce", "allgather", "reducescatter", "broadcast"):
        for dt in ("float32", "bfloat16", "float16"):
            for inplace in (False, True):
                c = base if kind in ("allreduce", "broadcast") else base // n
                if kind == "reducescatter":
                    c -= c % 8
                cases.append(Case(f"{kind}_{dt}_{'ip' if inplace else 'oop'}", kind, dt, c, inplace,
                                  root=n - 1))
        # odd element counts (tails that fill no vector)
        odd = (base + 7) if kind != "reducescatter" else base // n - (base // n) % 8 + 8
        cases.append(Case(f"{kind}_float32_odd", kind, "float32", odd if kind != "allgather" else odd // n + 3))
    cases.append(Case("allreduce_int32", "allreduce", "int32", base + 3))
    cases.append(Case("allgather_int8", "allgather", "int8", base // n + 1))
    cases.append(Case("broadcast_root0_int8", "broadcast", "int8", base * 4 + 5, root=0))
    cases.append(Case("allreduce_max", "allreduce", "float32", base, op="max"))
    # Every reduction op, and PreMulSum with one host scalar per rank.
    for op in ("prod", "min", "avg", "premulsum"):
        cases.append(Case(f"allreduce_{op}", "allreduce", "float32", base + 5, op=op))
        cases.append(Case(f"allreduce_{op}_bf16", "allreduce", "bfloat16", base, op=op))
        rc = base // n - (base // n) % 8
        cases.append(Case(f"reducescatter_{op}", "reducescatter", "float32", rc, op=op))
    cases.append(Case("allreduce_avg_int32", "allreduce", "int32", base, op="avg"))
    return cases


def pipeline_cases(n: int, env: dict, sms: int) -> list[Case]:
    """-1/0/+1 vector (32 bytes of fp32) around the edges of the engines'
    pipelines: the NVLS round (AllReduce message, and the 4R start of the
    ramped round schedule; per-slot part of a round
    for ReduceScatter/AllGather), the push-reduce round of 256 KiB pieces per
    block (per segment), the push chain's step (chunk x blocks) and the
    host-lane piece. Each case runs on whatever route the environment picks;
    force routes to aim them."""
    out = []
    R = int(policy_value(env, "nvls_round"))
    part = (R // n) & ~31
    step = int(policy_value(env, "ring_chunk")) * sms
    push_round = 262144 * sms
    piece = int(policy_value(env, "host_piece"))

    def add(name, kind, nbytes):
        for d in (-8, 0, 8):  # fp32 elements: one 32-byte vector
            c = nbytes // 4 + d
            if kind == "reducescatter":
                c -= c % 4
            if c > 0:
                out.append(Case(f"edge_{name}_{d:+d}", kind, "float32", c))
    add("nvls_round_ar", "allreduce", R)
    add("nvls_round2_ar", "allreduce", 2 * R)
    # Ramped AllReduce schedule (first and last rounds R/8 .. R/2) from 4R on,
    # and a partial uniform round between the ramps.
    add("nvls_ramp_ar", "allreduce", 4 * R)
    add("nvls_ramp_part_ar", "allreduce", 5 * R + R // 16)
    add("nvls_part_rs", "reducescatter", part)
    add("nvls_part_ag", "allgather", part)
    add("ring_step_bc", "broadcast", step)
    add("ring_step2_bc", "broadcast", 2 * step)
    add("push_round_ar", "allreduce", push_round * n)
    add("push_round_rs", "reducescatter", push_round)
    add("host_piece_ar", "allreduce", piece * n)
    add("host_piece_rs", "reducescatter", piece)
    return out


def big_cases(n: int) -> list[Case]:
    """The 2 GiB and 4 GiB logical-size edges (-1/0/+1 element), and the
    8 GiB message cap: at the cap (custom) and one element above it (must
    fall back to NCCL)."""
    G = 1 << 30
    out = []
    for size, tag in ((2 * G, "2g"), (4 * G, "4g")):
        for d in (-1, 0, 1):
            out.append(Case(f"big_{tag}_allreduce_{d:+d}", "allreduce", "float32", size // 4 + d))
        rc = size // 4 // n
        out.append(Case(f"big_{tag}_reducescatter", "reducescatter", "float32", rc - rc % 4))
        out.append(Case(f"big_{tag}_allgather_+1", "allgather", "float32", size // 4 // n + 1))
    out.append(Case("cap_allreduce_at", "allreduce", "float32", 8 * G // 4))
    out.append(Case("cap_allreduce_above", "allreduce", "float32", 8 * G // 4 + 1))
    out.append(Case("cap_broadcast_at", "broadcast", "float32", 8 * G // 4, root=n - 1))
    out.append(Case("cap_broadcast_above", "broadcast", "float32", 8 * G // 4 + 1))
    return out


def boundary_cases(n: int, thresholds: dict) -> list[Case]:
    """Element counts at -1, 0, +1 around each kind's routing threshold
    (AllGather's applies to the whole output, so to n slots)."""
    out = []
    for kind in ("allreduce", "broadcast", "allgather"):
        for d in (-1, 0, 1):
            if kind == "allgather":
                c = thresholds[kind] // 4 // n + d
            else:
                c = thresholds[kind] // 4 + d
            out.append(Case(f"bnd_{kind}_{d:+d}", kind, "float32", c))
    return out


class Buffers:
    """Send/recv tensors of one rank, each inside a guarded allocation."""

    def __init__(self, nbytes_send: int, nbytes_recv: int, dtype, device, inplace_view=None):
        self.es = torch.tensor([], dtype=dtype).element_size()
        self.dtype = dtype
        self.device = device
        self.send_raw = torch.full((nbytes_send + 2 * GUARD,), PATTERN, dtype=torch.uint8, device=device)
        self.recv_raw = torch.full((nbytes_recv + 2 * GUARD,), PATTERN, dtype=torch.uint8, device=device)

    def send(self):
        return self.send_raw[GUARD:-GUARD].view(self.dtype)

    def recv(self):
        return self.recv_raw[GUARD:-GUARD].view(self.dtype)

    def guard_bad(self) -> torch.Tensor:
        bad = torch.zeros((), dtype=torch.int64, device=self.device)
        for raw in (self.send_raw, self.recv_raw):
            bad += (raw[:GUARD] != PATTERN).sum() + (raw[-GUARD:] != PATTERN).sum()
        return bad


def custom_total(nc: Nccl) -> int:
    return sum(nc.custom_calls(a) or 0 for a in range(1, len(ALGO)))


def route_counts(nc: Nccl) -> dict:
    return {a: nc.custom_calls(a) or 0 for a in range(1, len(ALGO))}


ALGO_NAME = {v: k for k, v in ALGO.items()}


def fill_exact(t: torch.Tensor, rank: int, it: int, seed: int, n: int):
    """exact(...) written into `t` chunk by chunk (large buffers)."""
    total = t.numel()
    for lo in range(0, total, CHUNK):
        hi = min(total, lo + CHUNK)
        t[lo:hi].copy_(exact(rank, hi - lo, it, seed, t.dtype, n, t.device, offset=lo))


def thresholds() -> dict:
    """Per-kind routing thresholds (bytes) as the library's policy parser
    reads them from this process's environment."""
    env = {k: v for k, v in os.environ.items() if k.startswith("NCCL_B200_")}
    return {kind: int(policy_value(env, f"{key}_min"))
            for kind, key in (("allreduce", "ar"), ("allgather", "ag"), ("broadcast", "bc"))}


def fold_ref(vals: list, op: str, dtype, n: int, scalar: float) -> torch.Tensor:
    """The library's fold of `vals` (rank order), restated with torch: fp32
    accumulation for floating types (exact data make a float64 sum equal),
    the integer type's own width otherwise."""
    if op == "sum":
        if dtype.is_floating_point:
            acc = vals[0].to(torch.float64)
            for x in vals[1:]:
                acc = acc + x.to(torch.float64)
        else:
            acc = vals[0].to(torch.int64)
            for x in vals[1:]:
                acc = acc + x.to(torch.int64)
        return acc.to(dtype)
    if not dtype.is_floating_point:
        acc = vals[0].to(torch.int64)
        for x in vals[1:]:
            acc = {"max": torch.maximum, "min": torch.minimum}.get(op, torch.add)(acc, x.to(torch.int64))
        if op == "avg":
            acc = torch.div(acc, n, rounding_mode="trunc")
        return acc.to(dtype)
    acc = vals[0].float() * scalar if op == "premulsum" else vals[0].float()
    for x in vals[1:]:
        xf = x.float()
        if op == "prod":
            acc = acc * xf
        elif op == "max":
            acc = torch.maximum(acc, xf)
        elif op == "min":
            acc = torch.minimum(acc, xf)
        elif op == "premulsum":
            acc = acc + xf * scalar  # exact data and a power-of-two scalar: no rounding
        else:
            acc = acc + xf
    if op == "avg":  # a true division, as the kernels do
        acc = torch.div(acc, torch.full_like(acc, float(n)))
    return acc.to(dtype)


PREMUL_SCALAR = 0.5  # exact in every floating type


def want_chunk(case: Case, r: int, n: int, it: int, seed: int, dtype, device, lo: int, hi: int):
    """Expected output elements [lo, hi) of rank r, regenerated from the
    hashed inputs (no copies of the inputs are kept)."""
    c = case.count
    gen = lambda q, off, m: exact(q, m, it, seed, dtype, n, device, offset=off)  # noqa: E731
    if case.kind == "allreduce":
        return fold_ref([gen(q, lo, hi - lo) for q in range(n)], case.op, dtype, n, PREMUL_SCALAR)
    if case.kind == "reducescatter":
        return fold_ref([gen(q, r * c + lo, hi - lo) for q in range(n)], case.op, dtype, n, PREMUL_SCALAR)
    if case.kind == "broadcast":
        return gen(case.root, lo, hi - lo)
    parts, i = [], lo  # allgather: slot q of the output is rank q's input
    while i < hi:
        q, off = divmod(i, c)
        m = min(hi - i, c - off)
        parts.append(gen(q, off, m))
        i += m
    return torch.cat(parts)


def run_case(nc: Nccl, ref: Nccl | None, comms, devs, case: Case, iters: int, seed: int,
             diff: bool, corrupt_shift: int, delay_device: int = -1, delay_ms: float = 0.0,
             overwrite_after: bool = False, fresh_streams: bool = False, expect: str = "") -> dict:
    n = len(devs)
    dtype = DTYPES[case.dtype]
    es = torch.tensor([], dtype=dtype).element_size()
    c = case.count
    send_elems = {"reducescatter": c * n}.get(case.kind, c)
    recv_elems = {"allgather": c * n}.get(case.kind, c)
    bufs = []
    for r, d in enumerate(devs):
        b = Buffers(send_elems * es, recv_elems * es, dtype, f"cuda:{d}")
        bufs.append(b)
    home = [torch.cuda.current_stream(d) for d in devs]
    streams = [h.cuda_stream for h in home]

    def views(r):
        b = bufs[r]
        if not case.inplace:
            return b.send(), b.recv()
        if case.kind == "allgather":
            rv = b.recv()
            return rv[r * c:(r + 1) * c], rv
        if case.kind == "reducescatter":
            sv = b.send()
            return sv, sv[r * c:(r + 1) * c]
        return b.send(), b.send()

    ops = case.op
    if case.op == "premulsum":
        ops = [nc.premul_sum(PREMUL_SCALAR, case.dtype, comm) for comm in comms]
    mism = [torch.zeros((), dtype=torch.int64, device=f"cuda:{d}") for d in devs]
    before = route_counts(nc)
    shadows = None
    if diff and ref is not None:
        shadows = [torch.empty(recv_elems, dtype=dtype, device=f"cuda:{d}") for d in devs]
    reduces = case.kind in ("allreduce", "reducescatter")
    overwrite = overwrite_after and not case.inplace
    for it in range(iters):
        if fresh_streams:
            # New caller streams every iteration, ordered after the previous ones.
            fresh = [torch.cuda.Stream(device=d) for d in devs]
            for i, d in enumerate(devs):
                fresh[i].wait_stream(torch.cuda.current_stream(d))
                torch.cuda.set_stream(fresh[i])
            streams = [f.cuda_stream for f in fresh]
        sends, recvs = [], []
        for r, d in enumerate(devs):
            s, v = views(r)
            with torch.cuda.device(d):
                if diff and dtype.is_floating_point:
                    s.copy_(adversarial(r, s.numel(), seed + it, dtype, f"cuda:{d}", nans=not reduces))
                else:
                    fill_exact(s, r, it, seed, n)
            sends.append(s)
            recvs.append(v)
        if shadows is not None:
            # Stock NCCL first, into shadow buffers, through the real library.
            shadow_sends = [x.clone() for x in sends]
            collective(ref, case.kind, shadow_sends, shadows, comms, streams, op=case.op, root=case.root)
        if 0 <= delay_device < len(devs):
            # Hold one GPU's caller stream before the call: every other rank
            # must wait for its input, not read it early.
            with torch.cuda.device(devs[delay_device]):
                torch.cuda._sleep(int(delay_ms * 1.9e6))
        collective(nc, case.kind, sends, recvs, comms, streams, op=ops, root=case.root)
        if overwrite:
            # Stream-ordered reuse of the inputs right after the call: safe
            # only if the call's side streams joined the caller streams.
            for r, d in enumerate(devs):
                with torch.cuda.device(d):
                    sends[r].view(torch.uint8).fill_(0x5A)
        for r, d in enumerate(devs):
            with torch.cuda.device(d):
                got = recvs[r]
                if corrupt_shift and r == 0:
                    got = torch.roll(got, corrupt_shift)
                if shadows is not None:
                    want = shadows[r]
                    if reduces and dtype.is_floating_point:
                        gf, wf = got.float(), want.float()
                        both_nan = torch.isnan(gf) & torch.isnan(wf)
                        close = torch.isclose(gf, wf, rtol=1e-2, atol=1e-6, equal_nan=True)
                        mism[r] += (~(close | both_nan)).sum()
                    else:
                        mism[r] += (got.view(torch.uint8) != want.view(torch.uint8)).sum()
                else:
                    total = got.numel()
                    for lo in range(0, total, CHUNK):
                        hi = min(total, lo + CHUNK)
                        want = want_chunk(case, r, n, it, seed, dtype, f"cuda:{d}", lo, hi)
                        mism[r] += (got[lo:hi].view(torch.uint8) != want.view(torch.uint8)).sum()
        if fresh_streams:
            for i, d in enumerate(devs):
                home[i].wait_stream(torch.cuda.current_stream(d))
                torch.cuda.set_stream(home[i])
            streams = [h.cuda_stream for h in home]
    for d in devs:
        torch.cuda.synchronize(d)
    if case.op == "premulsum":
        for o, comm in zip(ops, comms):
            nc.redop_destroy(o, comm)
    total = int(sum(m.item() for m in mism))
    guard = int(sum(b.guard_bad().item() for b in bufs))
    after = route_counts(nc)
    ran = sorted(ALGO_NAME[a] for a in after if after[a] > before.get(a, 0))
    route = ",".join(ran) if ran else "nccl"
    status = "PASS" if total == 0 and guard == 0 else "FAIL"
    if status == "PASS" and expect and not route_matches(route, expect):
        status = "ROUTE"
    return {"case": case.name, "iters": iters, "bytes": c * es, "mismatches": total,
            "status": status, "guard_bad": guard, "route": route, "expect": expect or "-",
            "kind": case.kind, "mode": "diff" if diff else "check"}


def route_matches(route: str, expect: str) -> bool:
    if expect == "custom":
        return route != "nccl"
    return route == expect


def oracle_route(case: Case, n: int, nvls: bool, calib: dict | None, tuned: bool,
                 rules: oracle.Rules | None = None) -> str:
    """The independent oracle's route for a case ("custom" when tuned routes
    are in force but no calibration record is available to restate them)."""
    r = oracle.expected_route(case.kind, case.dtype, case.op, case.count, n, inplace=case.inplace,
                              nvls=nvls, rules=rules or oracle.Rules(), calib=calib)
    if tuned and calib is None and r != "nccl":
        return "custom"
    return r


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=min(2, torch.cuda.device_count()))
    p.add_argument("--iters", type=int, default=6)
    p.add_argument("--seed", type=int, default=1)
    p.add_argument("--scale", type=int, default=1, help="divide the standard case sizes")
    p.add_argument("--diff", action="store_true")
    p.add_argument("--corrupt-shift", type=int, default=0)
    p.add_argument("--filter", default="")
    p.add_argument("--no-boundary", action="store_true")
    p.add_argument("--no-standard", action="store_true")
    p.add_argument("--edges", action="store_true", help="the engines' pipeline edges")
    p.add_argument("--big", action="store_true", help="2/4 GiB edges and the 8 GiB message cap")
    p.add_argument("--no-oracle", action="store_true", help="do not check routes against the oracle")
    p.add_argument("--oracle-drop", default="",
                   help="hide this variable from the oracle (mutation self-test of the route check)")
    p.add_argument("--delay-input-device", type=int, default=-1,
                   help="hold this rank's caller stream before every call")
    p.add_argument("--delay-ms", type=float, default=20.0)
    p.add_argument("--overwrite-after", action="store_true",
                   help="overwrite the inputs on the caller streams right after every call")
    p.add_argument("--fresh-streams", action="store_true", help="new caller streams every iteration")
    p.add_argument("--algo", default="", help="force routes, e.g. ar=push,rs=push,ag=push,bc=ring "
                   "(the library reads it once, when it loads)")
    a = p.parse_args(argv)
    if a.algo:
        os.environ["NCCL_B200_ALGO"] = a.algo
    devs = list(range(a.gpus))
    n = len(devs)
    nc = Nccl("interposer")
    ref = Nccl("nccl") if a.diff else None
    comms = nc.comm_init_all(devs)
    env = {k: v for k, v in os.environ.items() if k.startswith("NCCL_B200_")}
    cases = [] if a.no_standard else standard_cases(n, a.scale)
    if not a.no_boundary:
        cases += boundary_cases(n, thresholds())
    if a.edges:
        cases += pipeline_cases(n, env, torch.cuda.get_device_properties(0).multi_processor_count)
    if a.big:
        cases += big_cases(n)
    if a.filter:
        cases = [c for c in cases if a.filter in c.name]
    import ctypes as C
    arr = (C.c_int * n)(*devs)
    nvls = bool(nc.shim.nb_nvls_supported(arr, n)) and oracle.Rules().nvls != "off"
    tuned = oracle.parse_bool(os.environ.get("NCCL_B200_TUNE")) is not False and n > 1
    calib = oracle.load_calib(os.environ.get("NCCL_B200_CALIB_CACHE"))
    rules = oracle.Rules({k: v for k, v in os.environ.items() if k != a.oracle_drop})
    # Warm-up: the first eligible call of the process always runs on NCCL.
    run_case(nc, None, comms, devs, Case("warmup", "allreduce", "float32", (64 << 20) // 4), 1, 0, False, 0)
    print("case\titers\tbytes\tmismatches\tstatus\tguard_bad\troute\texpect\tkind\tmode", flush=True)
    bad = 0
    for case in cases:
        expect = "" if a.no_oracle or a.diff else oracle_route(case, n, nvls, calib, tuned, rules)
        res = run_case(nc, ref, comms, devs, case, a.iters, a.seed, a.diff, a.corrupt_shift,
                       a.delay_input_device, a.delay_ms, a.overwrite_after, a.fresh_streams, expect)
        bad += res["status"] != "PASS"
        print("\t".join(str(res[k]) for k in ("case", "iters", "bytes", "mismatches", "status",
                                                "guard_bad", "route", "expect", "kind", "mode")), flush=True)
        torch.cuda.empty_cache()
    sys.stderr.write(nc.summary_text())
    for c in comms:
        nc.comm_destroy(c)
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
