#!/usr/bin/env python
"""Out-of-place busbw at 8 GiB fp32 per collective, one process driving N GPUs.

Arms (--impl):
  ours       LD_PRELOAD=scc26_nccl_shim_b200/lib/libnccl_b200.so (this repo)
  reference  LD_PRELOAD=baseline/_ref/libnccl_ce.so, the unmodified reference
             shim built from its own source with its README's nvcc line, with
             the reference's tuned-NCCL settings (Ring/Simple/MIN_CTAS=32/
             BUFFSIZE=1M); it forwards every call it does not handle to NCCL
  nccl       the real libnccl alone, default settings

The product is a single-process multi-GPU NCCL interposer, so the measuring
process is ONE process that calls ncclCommInitAll over GPUs 0..N-1 and issues
grouped collectives, as nccl-tests `-g N` does. Under torchrun (WORLD_SIZE>1)
rank 0 runs that process and the other ranks wait on a gloo barrier without
touching a GPU.

Timing: W untimed warm-up steps, then K timed steps bracketed by a device
synchronize on every GPU; CUDA events on every GPU's stream, max over GPUs.
Every input is 8 GiB (larger than the 126 MB L2), so no L2 flush is needed.
busbw follows nccl-tests: AllReduce algbw*2(N-1)/N, AllGather and
ReduceScatter algbw*(N-1)/N over the N-slot buffer, Broadcast algbw. At N=1
busbw is undefined (zero bus traffic); the 1-GPU point is the algbw of the
1-rank AllReduce, i.e. the device copy bandwidth.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "out-of-place busbw GB/s @8 GiB fp32 per collective at 2/4/8 B200 vs tuned NCCL"
# Reference shim, 2x H100 NVL (README.md of the reference, "Results").
PUBLISHED_SHIM = {"allreduce": 301.60, "allgather": 303.75, "reducescatter": 295.44,
                  "broadcast": 316.68}
REF_LIB = os.path.join(REPO, "baseline", "_ref", "libnccl_ce.so")
REF_TUNED_ENV = {"NCCL_ALGO": "Ring", "NCCL_PROTO": "Simple", "NCCL_MIN_CTAS": "32",
                 "NCCL_BUFFSIZE": "1048576"}
COLLS = ["allreduce", "allgather", "reducescatter", "broadcast"]


def parse_size(s: str) -> int:
    s = s.strip().upper().rstrip("B").rstrip("I")
    mul = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}.get(s[-1:], 1)
    return int(float(s[:-1] if s[-1:] in "KMG" else s) * mul)


def args_parser():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference", "nccl"], default="ours")
    p.add_argument("--colls", default=",".join(COLLS))
    p.add_argument("--bytes", default="8G", help="per-GPU buffer (AllReduce/Broadcast) or N-slot buffer")
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--worker", action="store_true", help=argparse.SUPPRESS)
    p.add_argument("--timeout", type=int, default=1500)
    return p


# --------------------------------------------------------------------------
# Parent: torchrun plumbing and the child process
# --------------------------------------------------------------------------

def reference_source() -> str | None:
    """The reference shim's source file, under BASELINE.json's reference_path."""
    try:
        with open(os.path.join(REPO, "BASELINE.json")) as f:
            root = json.load(f).get("reference_path")
    except (OSError, ValueError):
        return None
    return os.path.join(root, "shim", "nccl_collectives_shim.cu") if root else None


def ensure_reference() -> str | None:
    """Build the unmodified reference shim (its README's nvcc line) if missing."""
    if os.path.exists(REF_LIB):
        return None
    src = reference_source()
    if not src or not os.path.exists(src):
        return "reference source not present on this machine and baseline/_ref not built"
    import hashlib
    import nvidia.nccl  # type: ignore
    nccl = list(nvidia.nccl.__path__)[0]
    sha = hashlib.sha256(open(src, "rb").read()).hexdigest()
    os.makedirs(os.path.dirname(REF_LIB), exist_ok=True)
    cmd = ["nvcc", "-O3", "-std=c++17", "-arch=sm_90", "--cudart", "shared", "-include", "cstring",
           "-I", f"{nccl}/include", "-shared", "-Xcompiler", "-fPIC",
           f'-DNCCL_SHIM_SOURCE_SHA256="{sha}"', src, "-L", f"{nccl}/lib", "-L",
           "/usr/local/cuda/lib64/stubs", "-l:libnccl.so.2", "-lcuda", "-ldl", "-Xcompiler",
           "-pthread", "-o", REF_LIB]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return None if r.returncode == 0 else "reference build failed: " + r.stderr[-300:]


def child_env(impl: str) -> dict:
    from scc26_nccl_shim_b200 import LIB_PATH
    from scc26_nccl_shim_b200.parallel.nccl import preload_env
    if impl == "ours":
        return preload_env(LIB_PATH)
    if impl == "reference":
        return preload_env(REF_LIB, REF_TUNED_ENV)
    env = dict(os.environ)
    env.pop("LD_PRELOAD", None)
    return env


def run_child(args) -> str:
    if args.impl == "reference":
        why = ensure_reference()
        if why:
            return json.dumps({"impl": "reference", "unavailable": why})
    if args.impl == "ours":
        from scc26_nccl_shim_b200 import LIB_PATH
        if not os.path.exists(LIB_PATH):
            subprocess.run(["make", "-C", REPO, "-j8"], check=True, capture_output=True)
    cmd = [sys.executable, os.path.abspath(__file__), "--worker", "--gpus", str(args.gpus),
           "--steps", str(args.steps), "--warmup", str(args.warmup), "--impl", args.impl,
           "--colls", args.colls, "--bytes", args.bytes, "--e2e-steps", str(args.e2e_steps)]
    if args.no_e2e:
        cmd.append("--no-e2e")
    env = child_env(args.impl)
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK",
              "TORCHELASTIC_RUN_ID"):
        env.pop(k, None)
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=args.timeout)
    sys.stderr.write(r.stderr[-20000:])
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    if r.returncode != 0 or not lines:
        return json.dumps({"impl": args.impl, "metric": METRIC, "error":
                           f"worker exit {r.returncode}: {r.stderr[-400:]}"})
    return lines[-1]


def main():
    args = args_parser().parse_args()
    if args.worker:
        return worker(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import torch.distributed as dist
        rank = int(os.environ["RANK"])
        addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
        port = os.environ.get("MASTER_PORT", "29500")
        dist.init_process_group("gloo", init_method=f"tcp://{addr}:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=args.timeout + 300))
        line = run_child(args) if rank == 0 else None
        dist.barrier()
        dist.destroy_process_group()
        if rank == 0:
            print(line, flush=True)
        return 0
    print(run_child(args), flush=True)
    return 0


# --------------------------------------------------------------------------
# Worker: one process, N GPUs, grouped NCCL calls through the public ABI
# --------------------------------------------------------------------------

def busbw(kind: str, nbytes: int, seconds: float, n: int) -> float:
    algbw = nbytes / seconds / 1e9
    if n == 1:
        return algbw
    if kind == "allreduce":
        return algbw * 2 * (n - 1) / n
    if kind in ("allgather", "reducescatter"):
        return algbw * (n - 1) / n
    return algbw


def worker(args) -> int:
    import torch
    from scc26_nccl_shim_b200.parallel.nccl import Nccl, collective
    from scc26_nccl_shim_b200.utils.clocks import ClockSampler

    n = args.gpus
    if torch.cuda.device_count() < n:
        print(json.dumps({"impl": args.impl, "unavailable": f"need {n} GPUs, have {torch.cuda.device_count()}"}))
        return 0
    mode = "nccl" if args.impl == "nccl" else "preload"
    nc = Nccl(mode)
    devs = list(range(n))
    comms = nc.comm_init_all(devs)
    total = parse_size(args.bytes)
    colls = [c for c in args.colls.split(",") if c]
    streams = [torch.cuda.current_stream(d).cuda_stream for d in devs]
    results, checks = {}, {}
    clocks = None
    launches = None
    e2e = None

    def sync_all():
        for d in devs:
            torch.cuda.synchronize(d)

    for kind in colls:
        count = total // 4
        if kind in ("allgather", "reducescatter"):
            count = (total // 4) // n // 4 * 4  # per-rank slot, 16-byte multiple
        sends, recvs = [], []
        for d in devs:
            g = torch.Generator(device=f"cuda:{d}").manual_seed(1234 + d)
            if kind == "reducescatter":
                s = torch.rand(count * n, device=f"cuda:{d}", generator=g) * 2 - 1
                r = torch.empty(count, device=f"cuda:{d}")
            elif kind == "allgather":
                s = torch.rand(count, device=f"cuda:{d}", generator=g) * 2 - 1
                r = torch.empty(count * n, device=f"cuda:{d}")
            else:
                s = torch.rand(count, device=f"cuda:{d}", generator=g) * 2 - 1
                r = torch.empty(count, device=f"cuda:{d}")
            sends.append(s)
            recvs.append(r)
        nbytes = {"allreduce": count * 4, "broadcast": count * 4}.get(kind, count * 4 * n)
        for _ in range(args.warmup):
            collective(nc, kind, sends, recvs, comms, streams)
        sync_all()
        nvls_trace(nc, devs, kind, reset_only=True)
        l0 = nc.kernel_launches()
        starts = [torch.cuda.Event(enable_timing=True) for _ in devs]
        stops = [torch.cuda.Event(enable_timing=True) for _ in devs]
        sampler = ClockSampler(devs).start() if kind == "allreduce" else None
        time.sleep(0.3 if sampler else 0)
        for i, d in enumerate(devs):
            with torch.cuda.device(d):
                starts[i].record(torch.cuda.current_stream(d))
        for _ in range(args.steps):
            collective(nc, kind, sends, recvs, comms, streams)
        for i, d in enumerate(devs):
            with torch.cuda.device(d):
                stops[i].record(torch.cuda.current_stream(d))
        sync_all()
        if sampler:
            clocks = sampler.stop()
        ms = max(starts[i].elapsed_time(stops[i]) for i in range(n)) / args.steps
        nvls_trace(nc, devs, kind, steps=args.steps)
        l1 = nc.kernel_launches()
        if kind == "allreduce" and l0 is not None:
            launches = l1 - l0
        results[kind] = {"busbw_gbs": round(busbw(kind, nbytes, ms / 1e3, n), 2),
                         "algbw_gbs": round(nbytes / (ms / 1e3) / 1e9, 2), "ms": round(ms, 4),
                         "bytes": nbytes}
        # Check the last result against a torch fp32 reference on a sample.
        k = min(count, 1 << 20)
        idx = [slice(0, k), slice(count - k, count)]
        err = 0.0
        for sl in idx:
            if kind == "allreduce":
                ref = sum(sends[q][sl].to("cuda:0") for q in range(n))
                got = recvs[n - 1][sl].to("cuda:0")
            elif kind == "broadcast":
                ref = sends[0][sl].to("cuda:0")
                got = recvs[n - 1][sl].to("cuda:0")
            elif kind == "allgather":
                ref = sends[n - 1][sl].to("cuda:0")
                got = recvs[0][(n - 1) * count:][sl].to("cuda:0")
            else:
                ref = sum(sends[q][(n - 1) * count:][sl].to("cuda:0") for q in range(n))
                got = recvs[n - 1][sl].to("cuda:0")
            err = max(err, (ref - got).abs().max().item())
        checks[kind] = err
        if kind == "allreduce" and not args.no_e2e:
            e2e = end_to_end(torch, nc, comms, sends, recvs, streams, devs, count, args)
        del sends, recvs
        torch.cuda.empty_cache()

    head = "allreduce" if "allreduce" in results else colls[0]
    value = results[head]["busbw_gbs"]
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": n,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": results[head]["ms"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": round(value / PUBLISHED_SHIM[head], 4) if n > 1 else None,
        "dtype": "float32",
        "data": "synthetic: seeded uniform[-1,1] fp32 buffers (torch.rand, seed 1234+gpu)",
        "impl": args.impl,
        "config": {"model": f"{head} {total >> 30} GiB fp32 out-of-place (nccl-tests busbw)",
                   "global_batch": 1, "seq_len": results[head]["bytes"] // 4,
                   "parallelism": f"single-process clique of {n} GPU(s), ncclCommInitAll",
                   "l2": "inputs larger than L2 (8 GiB per buffer); no flush",
                   "n1_point": "algbw of the 1-rank AllReduce (device copy)" if n == 1 else None,
                   "nccl_version": nc.version()},
        "per_collective": results,
        "check_max_abs_err": checks,
        "clocks": clocks,
        "e2e": e2e,
        "gpu_launches": launches,
    }
    for c in comms:
        try:
            nc.comm_destroy(c)
        except Exception:
            pass
    if nc.shim is not None:
        sys.stderr.write(nc.summary_text())
    print(json.dumps(line), flush=True)
    return 0


def nvls_trace(nc, devs, kind, reset_only=False, steps=1):
    """With NCCL_B200_NVLS_TRACE=1: the in-kernel-synchronized engines'
    per-block phase times (mean over blocks, per call) of every rank, to
    stderr: the NVLS kernels, the push-reduce kernel and the Broadcast push
    chain. Read outside the timed region (it synchronizes the devices)."""
    import ctypes as C
    if not os.environ.get("NCCL_B200_NVLS_TRACE") or nc.shim is None or \
            not hasattr(nc.shim, "nb_nvls_trace"):
        return
    n = len(devs)
    arr = (C.c_int * n)(*devs)
    for r in range(n):
        out = (C.c_double * 6)()
        blocks = nc.shim.nb_nvls_trace(arr, n, r, out, 1)
        if not reset_only and blocks > 0:
            ms = [v / 1e6 / steps for v in out]
            sys.stderr.write(f"nvls_trace {kind} rank={r} blocks={blocks} per_call_ms mover_busy={ms[0]:.3f} "
                             f"mover_wait={ms[1]:.3f} copier_busy={ms[2]:.3f} copier_wait={ms[3]:.3f} "
                             f"mover_total={ms[4]:.3f} copier_total={ms[5]:.3f}\n")
        out4 = (C.c_double * 4)()
        blocks = nc.shim.nb_pushred_trace(arr, n, r, out4, 1)
        if not reset_only and blocks > 0:
            ms = [v / 1e6 / steps for v in out4]
            sys.stderr.write(f"pushred_trace {kind} rank={r} blocks={blocks} per_call_ms sender_wait={ms[0]:.3f} "
                             f"sender_total={ms[1]:.3f} reducer_wait={ms[2]:.3f} reducer_total={ms[3]:.3f}\n")
        out2 = (C.c_double * 2)()
        blocks = nc.shim.nb_ring_trace(arr, n, r, out2, 1)
        if not reset_only and blocks > 0:
            ms = [v / 1e6 / steps for v in out2]
            sys.stderr.write(f"ring_trace {kind} rank={r} blocks={blocks} per_call_ms wait={ms[0]:.3f} "
                             f"total={ms[1]:.3f}\n")


def end_to_end(torch, nc, comms, sends, recvs, streams, devs, count, args):
    """The same AllReduce through the public API with host I/O every step:
    H2D of every GPU's input from pinned host memory, the collective, and a
    D2H read of a result sample, with a host synchronize per step."""
    from scc26_nccl_shim_b200.parallel.nccl import collective
    n = len(devs)
    host = torch.empty(count, dtype=torch.float32, pin_memory=True)
    host.uniform_(-1, 1)
    sample = 1 << 18  # 1 MiB of fp32 read back per GPU
    outs = [torch.empty(sample, dtype=torch.float32, pin_memory=True) for _ in devs]
    bi = count * 4 * n
    bo = sample * 4 * n

    def step():
        for i, d in enumerate(devs):
            with torch.cuda.device(d):
                sends[i].copy_(host, non_blocking=True)
        collective(nc, "allreduce", sends, recvs, comms, streams)
        for i, d in enumerate(devs):
            with torch.cuda.device(d):
                outs[i].copy_(recvs[i][:sample], non_blocking=True)
        for d in devs:
            torch.cuda.synchronize(d)

    step()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        step()
    sec = (time.perf_counter() - t0) / args.e2e_steps
    return {"value": round(busbw("allreduce", count * 4, sec, n), 2), "unit": "GB/s",
            "ms_per_step": round(sec * 1e3, 3), "steps": args.e2e_steps,
            "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
            "note": "AllReduce busbw over the whole step incl. H2D of inputs and D2H of a result sample"}


if __name__ == "__main__":
    sys.exit(main())
