"""Routes forced through the environment, in child processes, against a
torch reference: the AllGather push route and the Broadcast push chain
(in-kernel progress words), out of place and in place, every root, odd
sizes and bf16; and the chain's bounded wait (a progress target nothing
reaches: the waiting kernels give up, record the status and return)."""
import os
import subprocess
import sys

import pytest

from conftest import REPO, need_gpus

pytestmark = pytest.mark.gpu

CHILD = r"""
import sys, torch
sys.path.insert(0, {repo!r}); sys.path.insert(0, {repo!r} + "/tests")
from scc26_nccl_shim_b200.parallel.nccl import Nccl
from scc26_nccl_shim_b200._core import ALGO
from test_gpu_abi import run_kind
n = {n}
devs = list(range(n))
nc = Nccl("interposer")
comms = nc.comm_init_all(devs)
for c in ((24 << 20) // 4, (24 << 20) // 4 + 3, 1000003):
    for inplace in (False, True):
        run_kind(nc, "allgather", comms, devs, c, inplace=inplace)
    for root in sorted({{0, n - 1, n // 2}}):
        run_kind(nc, "broadcast", comms, devs, c * 2 + 1, root=root)
        run_kind(nc, "broadcast", comms, devs, c, inplace=True, root=root)
run_kind(nc, "allgather", comms, devs, (24 << 20) // 4, dtype=torch.bfloat16)
run_kind(nc, "broadcast", comms, devs, (24 << 20) // 4, dtype=torch.bfloat16, root=n - 1)
print("RESULT", nc.custom_calls(ALGO["ag_push"]), nc.custom_calls(ALGO["bc_ring"]))
for c in comms:
    nc.comm_destroy(c)
"""


@pytest.mark.parametrize("n", [2, 3, 4, 8])
def test_forced_push_routes(n):
    need_gpus(n)
    env = dict(os.environ, NCCL_B200_ALGO="ag=push,bc=ring", NCCL_B200_TUNE="0",
               NCCL_B200_FIRST_PASS="0", NCCL_B200_AG_MIN="1K", NCCL_B200_BC_MIN="1K",
               NCCL_B200_RING_CHUNK="64K")
    r = subprocess.run([sys.executable, "-c", CHILD.format(repo=REPO, n=n)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    assert int(line[1]) >= 7 and int(line[2]) >= 8, line


PR_CHILD = r"""
import sys, torch
sys.path.insert(0, {repo!r}); sys.path.insert(0, {repo!r} + "/tests")
from scc26_nccl_shim_b200.parallel.nccl import Nccl
from scc26_nccl_shim_b200._core import ALGO
from test_gpu_abi import run_kind
n = {n}
devs = list(range(n))
nc = Nccl("interposer")
comms = nc.comm_init_all(devs)
for c in ((40 << 20) // 4, (40 << 20) // 4 + 5, 3000011):
    for inplace in (False, True):
        run_kind(nc, "allreduce", comms, devs, c, inplace=inplace)
    rs = c - c % 4
    run_kind(nc, "reducescatter", comms, devs, rs // n - (rs // n) % 4)
    run_kind(nc, "reducescatter", comms, devs, rs // n - (rs // n) % 4, inplace=True)
for dt in (torch.bfloat16, torch.float16):
    run_kind(nc, "allreduce", comms, devs, (24 << 20) // 4, dtype=dt)
    run_kind(nc, "reducescatter", comms, devs, (24 << 20) // 4 // n // 8 * 8, dtype=dt)
for op in ("avg", "max", "min", "prod"):
    run_kind(nc, "allreduce", comms, devs, (16 << 20) // 4 + 7, op=op)
print("RESULT", nc.custom_calls(ALGO["ar_push"]), nc.custom_calls(ALGO["rs_push"]))
for c in comms:
    nc.comm_destroy(c)
"""


@pytest.mark.parametrize("n", [2, 3, 4, 8])
def test_forced_push_reduce(n):
    need_gpus(n)
    env = dict(os.environ, NCCL_B200_ALGO="ar=push,rs=push", NCCL_B200_TUNE="0",
               NCCL_B200_FIRST_PASS="0", NCCL_B200_AR_MIN="1K", NCCL_B200_RS_MIN="1K")
    r = subprocess.run([sys.executable, "-c", PR_CHILD.format(repo=REPO, n=n)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    assert int(line[1]) >= 12 and int(line[2]) >= 8, line


TIMEOUT_CHILD = r"""
import sys, ctypes as C, torch
sys.path.insert(0, {repo!r})
from scc26_nccl_shim_b200.parallel.nccl import Nccl, collective, NcclError
nc = Nccl("interposer")
devs = [0, 1, 2]
arr = (C.c_int * 3)(*devs)
comms = nc.comm_init_all(devs)
xs = [torch.full((16 << 20,), float(d + 1), device=f"cuda:{{d}}") for d in devs]
ys = [torch.empty_like(x) for x in xs]
s = [torch.cuda.current_stream(d).cuda_stream for d in devs]
out = []
for i in range(3):
    try:
        collective(nc, "broadcast", xs, ys, comms, s, root=0)
        for d in devs: torch.cuda.synchronize(d)
        out.append("ok" if all(torch.equal(y, xs[0].to(y.device)) for y in ys) else "stale")
    except NcclError as e:
        for d in devs: torch.cuda.synchronize(d)
        out.append("err%d" % e.code)
    out.append("s%d" % nc.shim.nb_ring_status(arr, 3))
print("RESULT", ",".join(out), nc.shim.nb_poisoned())
"""


def test_ring_bounded_wait_reports_timeout():
    """Three GPUs (the middle rank of the chain waits): with a progress target
    nothing reaches, the middle rank's kernel gives up after 200 ms and sets
    the status word; the next call reports ncclUnhandledCudaError and
    poisons the custom paths; the call after runs on NCCL. No GPU faults."""
    need_gpus(3)
    env = dict(os.environ, NCCL_B200_ALGO="bc=ring", NCCL_B200_TUNE="0", NCCL_B200_FIRST_PASS="0",
               NCCL_B200_TEST_NVLS_SKEW="1000", NCCL_B200_TIMEOUT_MS="200")
    r = subprocess.run([sys.executable, "-c", TIMEOUT_CHILD.format(repo=REPO)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    seq = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    calls = seq[1].split(",")
    # call 1: the middle rank's wait expires (status 1; its successor is stale)
    assert calls[1] == "s1", calls
    assert calls[2] == "err1", calls
    assert calls[4] == "ok", calls
    assert seq[2] == "1"


ORDER_CHILD = r"""
import sys, ctypes as C, torch
sys.path.insert(0, {repo!r})
from scc26_nccl_shim_b200.parallel.nccl import Nccl, collective
from scc26_nccl_shim_b200._core import ALGO
from scc26_nccl_shim_b200.utils.data import exact
n = {n}
devs = list(range(n))
nc = Nccl("interposer")
cliques = [nc.comm_init_all(devs), nc.comm_init_all(devs)]
# Two unordered streams per GPU (neither waits on the other).
streams = [[torch.cuda.Stream(device=d) for d in devs] for _ in range(2)]
count = (48 << 20) // 4  # 48 MiB per rank: long enough for calls to overlap
kinds = ["broadcast", "allreduce", "reducescatter"]
jobs = []
# (a) two cliques over the same GPUs, (b) one clique on two unordered streams;
# every call back to back, no host synchronization in between.
for it in range(6):
    for mode in ("two_cliques", "two_streams"):
        comms = cliques[it % 2] if mode == "two_cliques" else cliques[0]
        ss = streams[it % 2]
        kind = kinds[it % 3]
        slots = n if kind == "reducescatter" else 1
        rc = count // n // 8 * 8 if kind == "reducescatter" else count
        sends, recvs = [], []
        for r, d in enumerate(devs):
            with torch.cuda.stream(ss[r]):
                sends.append(exact(r, rc * slots, it, 7 + len(jobs), torch.float32, n, f"cuda:{{d}}"))
                recvs.append(torch.empty(rc, device=f"cuda:{{d}}"))
        collective(nc, kind, sends, recvs, comms, [s.cuda_stream for s in ss], root=it % n)
        jobs.append((kind, rc, sends, recvs, it % n))
for d in devs:
    torch.cuda.synchronize(d)
bad = 0
for kind, rc, sends, recvs, root in jobs:
    ins = [s.to("cuda:0") for s in sends]
    for r in range(n):
        if kind == "broadcast":
            ref = ins[root]
        elif kind == "allreduce":
            ref = ins[0].clone()
            for x in ins[1:]:
                ref = ref + x
        else:
            ref = ins[0][r * rc:(r + 1) * rc].clone()
            for x in ins[1:]:
                ref = ref + x[r * rc:(r + 1) * rc]
        bad += 0 if torch.equal(recvs[r].to("cuda:0"), ref) else 1
arr = (C.c_int * n)(*devs)
st = nc.shim.nb_ring_status(arr, n) | nc.shim.nb_pushred_status(arr, n) | nc.shim.nb_oneshot_status(arr, n)
print("RESULT", bad, st, nc.shim.nb_poisoned(), nc.custom_calls(ALGO["bc_ring"]),
      nc.custom_calls(ALGO["ar_push"]), nc.custom_calls(ALGO["rs_push"]),
      nc.custom_calls(ALGO["ar_oneshot"]) + nc.custom_calls(ALGO["ar_twoshot_ll"]),
      nc.custom_calls(ALGO["rs_ll"]) + nc.custom_calls(ALGO["bc_ll"]))
"""


@pytest.mark.parametrize("algo", ["bc=ring,ar=push,rs=push", "ar=oneshot", "bc=ll,ar=twoshot_ll,rs=ll"])
@pytest.mark.parametrize("n", [2, 3])
def test_gang_calls_ordered_across_streams_and_cliques(n, algo):
    """The push chain and the push-reduce engine keep scratch, progress words
    and an epoch per device set. Calls from two cliques over the same GPUs,
    and calls of one clique on two unordered streams, issued back to back
    without host synchronization, must not overlap on those engines: every
    result bit-exact, no wait expired, nothing poisoned."""
    need_gpus(n)
    env = dict(os.environ, NCCL_B200_ALGO=algo, NCCL_B200_TUNE="0",
               NCCL_B200_FIRST_PASS="0", NCCL_B200_AR_MIN="1K", NCCL_B200_RS_MIN="1K",
               NCCL_B200_BC_MIN="1K", NCCL_B200_TIMEOUT_MS="5000")
    r = subprocess.run([sys.executable, "-c", ORDER_CHILD.format(repo=REPO, n=n)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    bad, status, poisoned, ring, arp, rsp, one, ll = map(int, line[1:])
    assert (bad, status, poisoned) == (0, 0, 0), line
    if "ll" in algo:
        assert one >= 4 and ll >= 8, line
    elif "shot" in algo:
        assert one >= 4, line
    else:
        assert ring >= 4 and arp >= 4 and rsp >= 4, line


OS_CHILD = r"""
import sys, torch
sys.path.insert(0, {repo!r}); sys.path.insert(0, {repo!r} + "/tests")
from scc26_nccl_shim_b200.parallel.nccl import Nccl
from scc26_nccl_shim_b200._core import ALGO
from test_gpu_abi import run_kind
n = {n}
devs = list(range(n))
nc = Nccl("interposer")
comms = nc.comm_init_all(devs)
for c in (1, 7, 4096, 65536 + 3, (1 << 20) // 4, (8 << 20) // 4 + 5, (48 << 20) // 4):
    run_kind(nc, "allreduce", comms, devs, c)
for dt in (torch.bfloat16, torch.float16):
    run_kind(nc, "allreduce", comms, devs, (1 << 20) + 9, dtype=dt)
for op in ("avg", "max", "min", "prod"):
    run_kind(nc, "allreduce", comms, devs, (2 << 20) // 4 + 1, op=op)
run_kind(nc, "allreduce", comms, devs, (4 << 20) // 4, inplace=True)  # one-shot: planned as two-shot
print("RESULT", nc.custom_calls(ALGO["ar_oneshot"]), nc.custom_calls(ALGO["ar_twoshot_ll"]))
for c in comms:
    nc.comm_destroy(c)
"""


@pytest.mark.parametrize("algo", ["oneshot", "twoshot_ll"])
@pytest.mark.parametrize("n", [2, 3, 4, 8])
def test_forced_oneshot(n, algo):
    """The low-latency one-shot and two-shot AllReduce (in-kernel
    arrive/depart barriers) from 4 bytes up (slices of a few bytes, empty
    slices), odd tails, 16-bit types and every op, bit-exact against a torch
    fp32 fold in rank order; in place the one-shot runs the low-latency
    two-shot plan."""
    need_gpus(n)
    env = dict(os.environ, NCCL_B200_ALGO="ar=" + algo, NCCL_B200_TUNE="0", NCCL_B200_FIRST_PASS="0",
               NCCL_B200_AR_MIN="1")
    r = subprocess.run([sys.executable, "-c", OS_CHILD.format(repo=REPO, n=n)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    one, two = int(line[1]), int(line[2])
    if algo == "oneshot":
        assert one >= 13 and two >= 1, line
    else:
        assert one == 0 and two >= 14, line


OS_TIMEOUT_CHILD = r"""
import sys, ctypes as C, torch
sys.path.insert(0, {repo!r})
from scc26_nccl_shim_b200.parallel.nccl import Nccl, collective, NcclError
nc = Nccl("interposer")
devs = [0, 1]
arr = (C.c_int * 2)(*devs)
comms = nc.comm_init_all(devs)
xs = [torch.full((1 << 20,), float(d + 1), device=f"cuda:{{d}}") for d in devs]
ys = [torch.empty_like(x) for x in xs]
s = [torch.cuda.current_stream(d).cuda_stream for d in devs]
out = []
for i in range(3):
    try:
        collective(nc, "allreduce", xs, ys, comms, s)
        for d in devs: torch.cuda.synchronize(d)
        out.append("ok" if all(torch.equal(y, torch.full_like(y, 3.0)) for y in ys) else "stale")
    except NcclError as e:
        for d in devs: torch.cuda.synchronize(d)
        out.append("err%d" % e.code)
    out.append("s%d" % nc.shim.nb_oneshot_status(arr, 2))
print("RESULT", ",".join(out), nc.shim.nb_poisoned())
"""


def test_oneshot_bounded_wait_reports_timeout():
    """With a barrier target nothing reaches, every block gives up after
    200 ms and sets the status word; the next call reports
    ncclUnhandledCudaError and poisons the custom paths; the call after runs
    on NCCL. No GPU faults."""
    need_gpus(2)
    env = dict(os.environ, NCCL_B200_ALGO="ar=oneshot", NCCL_B200_TUNE="0", NCCL_B200_FIRST_PASS="0",
               NCCL_B200_AR_MIN="1K", NCCL_B200_TEST_NVLS_SKEW="1000", NCCL_B200_TIMEOUT_MS="200")
    r = subprocess.run([sys.executable, "-c", OS_TIMEOUT_CHILD.format(repo=REPO)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    seq = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    calls = seq[1].split(",")
    assert calls[1] == "s1", calls
    assert calls[2] == "err1", calls
    assert calls[4] == "ok", calls
    assert seq[2] == "1"
