"""Device-timed collective size sweep (nccl-tests style) through the
interposer, stock libnccl, or whatever library is preloaded.

For each size (min..max by a factor): `--warmup` untimed calls, then
`--iters` timed calls bracketed by CUDA events on every GPU's caller stream;
the time is the MAX over GPUs. busbw follows nccl-tests: AllReduce
2(n-1)/n x algbw, AllGather/ReduceScatter (n-1)/n x algbw of the whole
(n-slot) buffer, Broadcast = algbw. Sizes are the logical message bytes
(AllReduce/Broadcast buffer; the n-slot buffer of AllGather/ReduceScatter).
Data are seeded: uniform[-1,1] (or N(0,1) with --normal) in the element
type; --check compares the last result with a torch fp32 reference.

One TSV row per size:
  bytes count dtype op inplace ms algbw_gbs busbw_gbs route max_abs_err

`route` is the interposer's route that ran the timed calls ("nccl" when
they fell back), read from its per-route counters.

Counterpart: the reference quotes nccl-tests all_reduce_perf -b 8 -e 8G -f 2
(README.md:41-47); this is the same measurement driven through the NCCL ABI
from one process.
"""
from __future__ import annotations

import argparse
import sys

import torch

from .._core import ALGO
from .nccl import DT, OPS, Nccl, collective

TORCH = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}
ALGO_NAME = {v: k for k, v in ALGO.items()}


def parse_size(s: str) -> int:
    s = s.strip().upper().rstrip("B").rstrip("I")
    mul = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}.get(s[-1:], 1)
    return int(s[:-1] if mul > 1 else s) * mul


def busbw(kind: str, nbytes: int, seconds: float, n: int) -> float:
    alg = nbytes / seconds / 1e9
    if n == 1:
        return alg
    return alg * {"allreduce": 2 * (n - 1) / n, "broadcast": 1.0}.get(kind, (n - 1) / n)


def routes(nc: Nccl) -> dict:
    if nc.shim is None:
        return {}
    return {a: nc.custom_calls(a) for a in range(1, len(ALGO))}


def premul(nc: Nccl, comms, dtype: str, n: int) -> list[int]:
    return [nc.premul_sum(1.0 / n, dtype, c) for c in comms]


def run_size(nc, comms, devs, kind, nbytes, dtype, op, inplace, warmup, iters, check, normal, seed):
    n = len(devs)
    tdt = TORCH[dtype]
    es = torch.tensor([], dtype=tdt).element_size()
    count = max(1, nbytes // es)
    slot = count // n if kind in ("allgather", "reducescatter") else count
    if slot == 0:
        return None
    sends, recvs = [], []
    for r, d in enumerate(devs):
        g = torch.Generator(device=f"cuda:{d}").manual_seed(seed + 7919 * r)
        big = slot * n if kind in ("allgather", "reducescatter") else slot
        if normal:
            x = torch.randn(big if kind != "allgather" else slot, device=f"cuda:{d}", generator=g)
        else:
            x = torch.rand(big if kind != "allgather" else slot, device=f"cuda:{d}", generator=g) * 2 - 1
        x = x.to(tdt)
        if kind == "allgather":
            recv = torch.empty(slot * n, dtype=tdt, device=f"cuda:{d}")
            if inplace:
                recv[r * slot:(r + 1) * slot].copy_(x)
                x = recv[r * slot:(r + 1) * slot]
        elif kind == "reducescatter":
            recv = x[r * slot:(r + 1) * slot] if inplace else torch.empty(slot, dtype=tdt, device=f"cuda:{d}")
        else:
            recv = x if inplace else torch.empty(slot, dtype=tdt, device=f"cuda:{d}")
        sends.append(x)
        recvs.append(recv)
    inputs = [s.float().to("cuda:0") for s in sends] if check else None
    streams = [torch.cuda.current_stream(d).cuda_stream for d in devs]
    ops = None
    if op == "premulsum":
        ops = premul(nc, comms, dtype, n)
    def one():
        if ops is None:
            collective(nc, kind, sends, recvs, comms, streams, op=op)
        else:
            with nc.group():
                for i, comm in enumerate(comms):
                    if kind == "allreduce":
                        nc.all_reduce(sends[i], recvs[i], comm, streams[i], ops[i])
                    else:
                        nc.reduce_scatter(sends[i], recvs[i], comm, streams[i], ops[i])
    for _ in range(warmup):
        one()
    for d in devs:
        torch.cuda.synchronize(d)
    before = routes(nc)
    starts = [torch.cuda.Event(enable_timing=True) for _ in devs]
    stops = [torch.cuda.Event(enable_timing=True) for _ in devs]
    for i, d in enumerate(devs):
        with torch.cuda.device(d):
            starts[i].record(torch.cuda.current_stream(d))
    for _ in range(iters):
        one()
    for i, d in enumerate(devs):
        with torch.cuda.device(d):
            stops[i].record(torch.cuda.current_stream(d))
    for d in devs:
        torch.cuda.synchronize(d)
    ms = max(starts[i].elapsed_time(stops[i]) for i in range(n)) / iters
    after = routes(nc)
    ran = [ALGO_NAME[a] for a in after if after[a] > before.get(a, 0)]
    route = ",".join(ran) if ran else ("nccl" if nc.shim is not None else "n/a")
    err = float("nan")
    if check and not inplace:
        err = 0.0
        for r in range(n):
            got = recvs[r].float().to("cuda:0")
            if kind == "allreduce":
                want = sum(inputs)
                if op == "avg" or op == "premulsum":
                    want = want / n
            elif kind == "reducescatter":
                want = sum(x[r * slot:(r + 1) * slot] for x in inputs)
                if op == "avg" or op == "premulsum":
                    want = want / n
            elif kind == "allgather":
                want = torch.cat(inputs)
            else:
                want = inputs[0]
            err = max(err, (got - want).abs().max().item())
    if ops is not None:
        for o, c in zip(ops, comms):
            nc.redop_destroy(o, c)
    logical = slot * es * (n if kind in ("allgather", "reducescatter") else 1)
    return {"bytes": logical, "count": slot, "ms": ms,
            "algbw": logical / (ms / 1e3) / 1e9, "busbw": busbw(kind, logical, ms / 1e3, n),
            "route": route, "err": err}


def sizes(lo: int, hi: int, factor: int):
    s = lo
    while s <= hi:
        yield s
        s *= factor


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=max(1, min(2, torch.cuda.device_count())))
    p.add_argument("--kind", default="allreduce",
                   choices=["allreduce", "allgather", "reducescatter", "broadcast"])
    p.add_argument("--dtype", default="float32", choices=list(TORCH))
    p.add_argument("--op", default="sum", choices=["sum", "prod", "max", "min", "avg", "premulsum"])
    p.add_argument("--min", default="8")
    p.add_argument("--max", default="8G")
    p.add_argument("--factor", type=int, default=2)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--inplace", action="store_true")
    p.add_argument("--check", action="store_true")
    p.add_argument("--normal", action="store_true", help="N(0,1) data instead of uniform[-1,1]")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--mode", default="interposer", choices=["interposer", "nccl", "preload"])
    a = p.parse_args(argv)
    nc = Nccl(a.mode)
    devs = list(range(a.gpus))
    comms = nc.comm_init_all(devs)
    assert a.op in OPS or a.op == "premulsum"
    assert a.dtype in DT
    print("bytes\tcount\tdtype\top\tinplace\tms\talgbw_gbs\tbusbw_gbs\troute\tmax_abs_err", flush=True)
    for s in sizes(parse_size(a.min), parse_size(a.max), a.factor):
        row = run_size(nc, comms, devs, a.kind, s, a.dtype, a.op, a.inplace, a.warmup, a.iters,
                       a.check, a.normal, a.seed)
        if row is None:
            continue
        print(f"{row['bytes']}\t{row['count']}\t{a.dtype}\t{a.op}\t{int(a.inplace)}\t{row['ms']:.4f}\t"
              f"{row['algbw']:.2f}\t{row['busbw']:.2f}\t{row['route']}\t{row['err']:.3g}", flush=True)
        torch.cuda.empty_cache()
    if nc.shim is not None:
        sys.stderr.write(nc.summary_text())
    for c in comms:
        nc.comm_destroy(c)
    return 0


if __name__ == "__main__":
    sys.exit(main())
