"""Mixed-group and back-to-back-group workloads (one process, N GPUs).

--mode mixed: ONE ncclGroupStart/End batch of --calls seeded calls per rank
  with log-uniform sizes (--min..--max bytes) and collectives, dtypes and
  reduce ops drawn uniformly, including an operation the interposer never
  handles (a self send/recv pair). The interposer must forward the whole
  group to libnccl, in order, and run none of it itself; every result is
  checked against a torch reference. Prints the group's aggregate device
  time (max over GPUs).

--mode eligible: --calls back-to-back groups, each one clique call of a
  random kind and size at or above the thresholds, issued without host
  synchronization, with the host lane optionally forced on
  (NCCL_B200_HOST_SHARE_PPM), so the pinned-host lanes are reused across
  calls under stream ordering only. Every result is checked after the run;
  prints the aggregate device time and the routes that ran.

Counterpart: the reference's two-thread and mixed AllGather+Broadcast cases
(tests/stress_check.cu:622-692); the mixed configuration is this
repository's benchmark configuration for group fallback.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import random
import sys

import torch

from .._core import ALGO
from ..utils.data import exact
from .nccl import Nccl

KINDS = ["allreduce", "allgather", "reducescatter", "broadcast"]
DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "int32": torch.int32}
ALGO_NAME = {v: k for k, v in ALGO.items()}


def parse_size(s: str) -> int:
    s = s.strip().upper().rstrip("B").rstrip("I")
    mul = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}.get(s[-1:], 1)
    return int(float(s[:-1] if mul > 1 else s) * mul)


def draw_calls(rng: random.Random, calls: int, n: int, lo: int, hi: int, unsupported: bool):
    out = []
    for _ in range(calls):
        kinds = KINDS + (["send_recv"] if unsupported else [])
        kind = rng.choice(kinds)
        dtype = rng.choice(list(DTYPES))
        op = rng.choice(["sum", "max", "min"]) if kind in ("allreduce", "reducescatter") else "sum"
        nbytes = int(math.exp(rng.uniform(math.log(lo), math.log(hi))))
        count = max(8, nbytes // 4 // 8 * 8)
        if kind in ("allgather", "reducescatter"):
            count = max(8, (count // n) // 8 * 8)
        out.append((kind, dtype, op, count))
    if unsupported and not any(k == "send_recv" for k, *_ in out):
        out[rng.randrange(len(out))] = ("send_recv", "float32", "sum", 1024)
    return out


def issue(nc: Nccl, kind, s, v, comm, stream, op, rank, count):
    if kind == "allreduce":
        return nc.all_reduce(s, v, comm, stream, op)
    if kind == "allgather":
        return nc.all_gather(s, v, comm, stream)
    if kind == "reducescatter":
        return nc.reduce_scatter(s, v, comm, stream, op)
    if kind == "broadcast":
        return nc.broadcast(s, v, 0, comm, stream)
    dt = Nccl._dt(s)  # an operation the interposer never handles
    r = nc._fn("ncclSend")(C.c_void_p(s.data_ptr()), C.c_size_t(count), dt, rank, C.c_void_p(comm),
                           C.c_void_p(stream))
    return r or nc._fn("ncclRecv")(C.c_void_p(v.data_ptr()), C.c_size_t(count), dt, rank, C.c_void_p(comm),
                                   C.c_void_p(stream))


def buffers(calls, devs, seed):
    n = len(devs)
    bufs = []
    for i, (kind, dtype, op, count) in enumerate(calls):
        per = []
        for r, d in enumerate(devs):
            send_n = count * n if kind == "reducescatter" else count
            recv_n = count * n if kind == "allgather" else count
            s = exact(r, send_n, i, seed, DTYPES[dtype], n, f"cuda:{d}")
            v = torch.zeros(recv_n, dtype=DTYPES[dtype], device=f"cuda:{d}")
            per.append((s, v))
        bufs.append(per)
    return bufs


def check(calls, bufs, n) -> int:
    bad = 0
    for (kind, dtype, op, count), per in zip(calls, bufs):
        dev = per[0][0].device
        ins = [p[0].to(dev) for p in per]
        for r in range(n):
            got = per[r][1].to(dev)
            if kind in ("allreduce", "reducescatter"):
                parts = ins if kind == "allreduce" else [x[r * count:(r + 1) * count] for x in ins]
                acc = parts[0].double()
                for x in parts[1:]:
                    acc = acc + x.double() if op == "sum" else \
                        (torch.maximum(acc, x.double()) if op == "max" else torch.minimum(acc, x.double()))
                want = acc.to(got.dtype)
            elif kind == "allgather":
                want = torch.cat(ins)
            elif kind == "broadcast":
                want = ins[0]
            else:
                want = ins[r]
            bad += 0 if torch.equal(got, want) else 1
    return bad


def routes(nc: Nccl) -> dict:
    return {a: nc.custom_calls(a) for a in range(1, len(ALGO))}


def timed(devs, fn):
    for d in devs:
        torch.cuda.synchronize(d)
    starts = [torch.cuda.Event(enable_timing=True) for _ in devs]
    stops = [torch.cuda.Event(enable_timing=True) for _ in devs]
    for i, d in enumerate(devs):
        with torch.cuda.device(d):
            starts[i].record(torch.cuda.current_stream(d))
    fn()
    for i, d in enumerate(devs):
        with torch.cuda.device(d):
            stops[i].record(torch.cuda.current_stream(d))
    for d in devs:
        torch.cuda.synchronize(d)
    return max(a.elapsed_time(b) for a, b in zip(starts, stops))


def run(mode: str, n: int, calls: int, lo: int, hi: int, seed: int, impl: str = "interposer") -> dict:
    devs = list(range(n))
    nc = Nccl(impl)
    comms = nc.comm_init_all(devs)
    streams = [torch.cuda.current_stream(d).cuda_stream for d in devs]
    rng = random.Random(seed)
    plan = draw_calls(rng, calls, n, lo, hi, unsupported=(mode == "mixed"))
    if mode == "eligible":
        # Warm-up: the first eligible call of a process runs on NCCL.
        w = buffers([("allreduce", "float32", "sum", (64 << 20) // 4)], devs, seed + 1)
        with nc.group():
            for r, comm in enumerate(comms):
                issue(nc, "allreduce", w[0][r][0], w[0][r][1], comm, streams[r], "sum", r, 0)
    bufs = buffers(plan, devs, seed)
    before = routes(nc) if nc.shim is not None else {}

    def mixed():
        with nc.group():
            for (kind, dtype, op, count), per in zip(plan, bufs):
                for r, comm in enumerate(comms):
                    issue(nc, kind, per[r][0], per[r][1], comm, streams[r], op, r, count)

    def eligible():
        for (kind, dtype, op, count), per in zip(plan, bufs):
            with nc.group():
                for r, comm in enumerate(comms):
                    issue(nc, kind, per[r][0], per[r][1], comm, streams[r], op, r, count)

    ms = timed(devs, mixed if mode == "mixed" else eligible)
    after = routes(nc) if nc.shim is not None else {}
    ran = {ALGO_NAME[a]: after[a] - before.get(a, 0) for a in after if after[a] > before.get(a, 0)}
    bad = check(plan, bufs, n)
    total = sum(per[0][0].numel() * per[0][0].element_size() for per in bufs)
    out = {"mode": mode, "impl": impl, "n_gpus": n, "calls": len(plan), "device_ms": round(ms, 3),
           "bytes_per_rank": total, "mismatches": bad, "custom_routes": ran,
           "kinds": {k: sum(1 for c in plan if c[0] == k) for k in KINDS + ["send_recv"]}}
    if nc.shim is not None:
        out["summary"] = [l for l in nc.summary_text().splitlines() if "host_bytes" in l or "lane" in l]
    for c in comms:
        nc.comm_destroy(c)
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--mode", choices=["mixed", "eligible"], default="mixed")
    p.add_argument("--gpus", type=int, default=torch.cuda.device_count())
    p.add_argument("--calls", type=int, default=64)
    p.add_argument("--min", default="4K")
    p.add_argument("--max", default="1G")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--impl", choices=["interposer", "nccl"], default="interposer")
    a = p.parse_args(argv)
    res = run(a.mode, a.gpus, a.calls, parse_size(a.min), parse_size(a.max), a.seed, a.impl)
    print(json.dumps(res), flush=True)
    return 0 if res["mismatches"] == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
