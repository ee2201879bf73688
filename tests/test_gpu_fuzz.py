"""The mixed-group benchmark configuration (scaled): one ncclGroupStart/End batch of 64 seeded
calls with log-uniform sizes and random collectives, dtypes and reduce ops,
including operations the interposer does not handle. The mixed group must
fall back to libnccl as a whole, in order, with correct results, and the
interposer must run none of it on its own routes."""
import math
import random

import pytest
import torch

from conftest import gpu_count, need_gpus

pytestmark = pytest.mark.gpu


def test_mixed_64_call_group_falls_back_in_order():
    need_gpus(1)
    from scc26_nccl_shim_b200._core import ALGO
    from scc26_nccl_shim_b200.parallel.nccl import Nccl
    n = min(2, gpu_count())
    devs = list(range(n))
    nc = Nccl("interposer")
    comms = nc.comm_init_all(devs)
    rng = random.Random(0)
    streams = [torch.cuda.current_stream(d).cuda_stream for d in devs]
    calls = []
    for i in range(64 // n):
        kind = rng.choice(["allreduce", "allgather", "reducescatter", "broadcast", "send_recv"])
        dtype = rng.choice([torch.float32, torch.bfloat16, torch.int32])
        op = rng.choice(["sum", "max", "min"]) if kind in ("allreduce", "reducescatter") else "sum"
        nbytes = int(math.exp(rng.uniform(math.log(4096), math.log(64 << 20))))
        count = max(8, nbytes // 4 // 8 * 8)
        if kind in ("allgather", "reducescatter"):
            count //= n
            count -= count % 8
        calls.append((kind, dtype, op, max(8, count)))
    assert any(k == "send_recv" for k, *_ in calls)
    bufs = []
    for kind, dtype, op, count in calls:
        per = []
        for r, d in enumerate(devs):
            send_n = count * n if kind == "reducescatter" else count
            recv_n = count * n if kind == "allgather" else count
            s = torch.randint(-50, 50, (send_n,), device=f"cuda:{d}").to(dtype)
            v = torch.zeros(recv_n, dtype=dtype, device=f"cuda:{d}")
            per.append((s, v))
        bufs.append(per)
    before = sum(nc.custom_calls(a) for a in ALGO.values() if a)
    for d in devs:
        torch.cuda.synchronize(d)
    starts = [torch.cuda.Event(enable_timing=True) for _ in devs]
    stops = [torch.cuda.Event(enable_timing=True) for _ in devs]
    for i, d in enumerate(devs):
        with torch.cuda.device(d):
            starts[i].record(torch.cuda.current_stream(d))
    with nc.group():
        for (kind, dtype, op, count), per in zip(calls, bufs):
            for r, comm in enumerate(comms):
                s, v = per[r]
                if kind == "allreduce":
                    nc.all_reduce(s, v, comm, streams[r], op)
                elif kind == "allgather":
                    nc.all_gather(s, v, comm, streams[r])
                elif kind == "reducescatter":
                    nc.reduce_scatter(s, v, comm, streams[r], op)
                elif kind == "broadcast":
                    nc.broadcast(s, v, 0, comm, streams[r])
                else:  # an operation the interposer never handles: a self send/recv pair
                    import ctypes as C
                    dt = Nccl._dt(s)
                    nc._fn("ncclSend")(C.c_void_p(s.data_ptr()), C.c_size_t(count), dt, r,
                                       C.c_void_p(comm), C.c_void_p(streams[r]))
                    nc._fn("ncclRecv")(C.c_void_p(v.data_ptr()), C.c_size_t(count), dt, r,
                                       C.c_void_p(comm), C.c_void_p(streams[r]))
    for i, d in enumerate(devs):
        with torch.cuda.device(d):
            stops[i].record(torch.cuda.current_stream(d))
    for d in devs:
        torch.cuda.synchronize(d)
    # Aggregate device time of the whole group (max over GPUs), for the log.
    print("mixed group of", len(calls), "calls per rank:",
          round(max(a.elapsed_time(b) for a, b in zip(starts, stops)), 3), "ms")
    assert sum(nc.custom_calls(a) for a in ALGO.values() if a) == before
    for (kind, dtype, op, count), per in zip(calls, bufs):
        ins = [p[0].to("cuda:0") for p in per]
        for r in range(n):
            got = per[r][1].to("cuda:0")
            if kind == "allreduce":
                acc = ins[0].double()
                for x in ins[1:]:
                    acc = acc + x.double() if op == "sum" else (torch.maximum(acc, x.double()) if op == "max" else torch.minimum(acc, x.double()))
                want = acc.to(dtype)
            elif kind == "reducescatter":
                parts = [x[r * count:(r + 1) * count].double() for x in ins]
                acc = parts[0]
                for x in parts[1:]:
                    acc = acc + x if op == "sum" else (torch.maximum(acc, x) if op == "max" else torch.minimum(acc, x))
                want = acc.to(dtype)
            elif kind == "allgather":
                want = torch.cat(ins)
            elif kind == "broadcast":
                want = ins[0]
            else:
                want = ins[r]
            assert torch.equal(got, want), (kind, dtype, op, count, r)
    for c in comms:
        nc.comm_destroy(c)
