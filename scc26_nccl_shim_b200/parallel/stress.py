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

Output: one TSV row per case:
  case iters bytes mismatches status guard_bad route kind mode
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
from .nccl import Nccl, collective

GUARD = 4096
PATTERN = 0xA5
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
    return cases


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


def thresholds() -> dict:
    """Per-kind routing thresholds (bytes) as the library's policy parser
    reads them from this process's environment."""
    env = {k: v for k, v in os.environ.items() if k.startswith("NCCL_B200_")}
    return {kind: int(policy_value(env, f"{key}_min"))
            for kind, key in (("allreduce", "ar"), ("allgather", "ag"), ("broadcast", "bc"))}


def run_case(nc: Nccl, ref: Nccl | None, comms, devs, case: Case, iters: int, seed: int,
             diff: bool, corrupt_shift: int, delay_device: int = -1, delay_ms: float = 0.0,
             overwrite_after: bool = False, fresh_streams: bool = False) -> dict:
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

    mism = [torch.zeros((), dtype=torch.int64, device=f"cuda:{d}") for d in devs]
    custom_before = custom_total(nc)
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
                if diff:
                    s.copy_(adversarial(r, s.numel(), seed + it, dtype, f"cuda:{d}", nans=not reduces)
                            if dtype.is_floating_point else exact(r, s.numel(), it, seed, dtype, n, f"cuda:{d}"))
                else:
                    s.copy_(exact(r, s.numel(), it, seed, dtype, n, f"cuda:{d}"))
            sends.append(s)
            recvs.append(v)
        inputs = [s.clone() for s in sends] if (diff or case.inplace or overwrite) else sends
        if shadows is not None:
            # Stock NCCL first, into shadow buffers, through the real library.
            shadow_sends = [x.clone() for x in inputs]
            collective(ref, case.kind, shadow_sends, shadows, comms, streams, op=case.op, root=case.root)
        if 0 <= delay_device < len(devs):
            # Hold one GPU's caller stream before the call: every other rank
            # must wait for its input, not read it early.
            with torch.cuda.device(devs[delay_device]):
                torch.cuda._sleep(int(delay_ms * 1.9e6))
        collective(nc, case.kind, sends, recvs, comms, streams, op=case.op, root=case.root)
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
                    want = expected(case, r, n, it, seed, dtype, f"cuda:{d}", [x.to(f"cuda:{d}") for x in inputs]
                                    if case.kind in ("allgather", "broadcast") or case.op != "sum" else None)
                    mism[r] += (got.view(torch.uint8) != want.view(torch.uint8)).sum()
        if fresh_streams:
            for i, d in enumerate(devs):
                home[i].wait_stream(torch.cuda.current_stream(d))
                torch.cuda.set_stream(home[i])
            streams = [h.cuda_stream for h in home]
    for d in devs:
        torch.cuda.synchronize(d)
    total = int(sum(m.item() for m in mism))
    guard = int(sum(b.guard_bad().item() for b in bufs))
    custom = custom_total(nc) > custom_before
    return {"case": case.name, "iters": iters, "bytes": c * es, "mismatches": total,
            "status": "PASS" if total == 0 and guard == 0 else "FAIL", "guard_bad": guard,
            "route": "custom" if custom else "nccl", "kind": case.kind,
            "mode": "diff" if diff else "check"}


def expected(case: Case, r: int, n: int, it: int, seed: int, dtype, device, inputs):
    c = case.count
    if case.kind == "allreduce":
        if case.op != "sum":
            acc = inputs[0].float()
            for x in inputs[1:]:
                acc = torch.maximum(acc, x.float()) if case.op == "max" else acc + x.float()
            return acc.to(dtype)
        acc = None
        for q in range(n):
            x = exact(q, c, it, seed, dtype, n, device).to(torch.float64)
            acc = x if acc is None else acc + x
        return acc.to(dtype)
    if case.kind == "reducescatter":
        acc = None
        for q in range(n):
            x = exact(q, c, it, seed, dtype, n, device, offset=r * c).to(torch.float64)
            acc = x if acc is None else acc + x
        return acc.to(dtype)
    if case.kind == "allgather":
        return torch.cat(inputs)
    return inputs[case.root]


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
    nc = Nccl("interposer")
    ref = Nccl("nccl") if a.diff else None
    comms = nc.comm_init_all(devs)
    cases = standard_cases(len(devs), a.scale)
    if not a.no_boundary:
        cases += boundary_cases(len(devs), thresholds())
    if a.filter:
        cases = [c for c in cases if a.filter in c.name]
    # Warm-up: the first eligible call of the process always runs on NCCL.
    run_case(nc, None, comms, devs, Case("warmup", "allreduce", "float32", (64 << 20) // 4), 1, 0, False, 0)
    print("case\titers\tbytes\tmismatches\tstatus\tguard_bad\troute\tkind\tmode", flush=True)
    bad = 0
    for case in cases:
        res = run_case(nc, ref, comms, devs, case, a.iters, a.seed, a.diff, a.corrupt_shift,
                       a.delay_input_device, a.delay_ms, a.overwrite_after, a.fresh_streams)
        bad += res["status"] != "PASS"
        print("\t".join(str(res[k]) for k in ("case", "iters", "bytes", "mismatches", "status",
                                                "guard_bad", "route", "kind", "mode")), flush=True)
    sys.stderr.write(nc.summary_text())
    for c in comms:
        nc.comm_destroy(c)
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
