"""NVLS (multimem) AllReduce on real GPUs, in child processes (the route is
forced through the environment, which the library reads once at load)."""
import os
import subprocess
import sys

import pytest

from conftest import REPO, gpu_count, need_gpus

pytestmark = pytest.mark.gpu

CHILD = r"""
import sys, ctypes as C, torch
sys.path.insert(0, {repo!r})
from scc26_nccl_shim_b200.parallel.nccl import Nccl, collective, NcclError
from scc26_nccl_shim_b200._core import ALGO
n = {n}
devs = list(range(n))
nc = Nccl("interposer")
arr = (C.c_int * n)(*devs)
supported = nc.shim.nb_nvls_supported(arr, n)
comms = nc.comm_init_all(devs)
streams = [torch.cuda.current_stream(d).cuda_stream for d in devs]
out = []
for dtype in (torch.float32, torch.bfloat16):
    for op in ("sum", "avg", "premulsum"):
        for count in ((16 << 20), (100 << 20) + 4 * 1024):
            lim = 15 if dtype == torch.bfloat16 else 1 << 18
            xs = [torch.randint(-lim, lim + 1, (count,), device=f"cuda:{{d}}").to(dtype) for d in devs]
            ys = [torch.empty_like(x) for x in xs]
            ops = None
            if op == "premulsum":  # one host scalar shared by every rank
                name = "float32" if dtype == torch.float32 else "bfloat16"
                ops = [nc.premul_sum(0.5, name, c) for c in comms]
            for it in range(2):
                if ops is None:
                    collective(nc, "allreduce", xs, ys, comms, streams, op=op)
                else:
                    with nc.group():
                        for i, c in enumerate(comms):
                            nc.all_reduce(xs[i], ys[i], c, streams[i], ops[i])
            for d in devs:
                torch.cuda.synchronize(d)
            if ops is not None:
                for o, c in zip(ops, comms):
                    nc.redop_destroy(o, c)
            ref = sum(x.to("cuda:0").float() for x in xs)
            if op == "avg":
                ref = ref / n
            if op == "premulsum":
                ref = ref * 0.5
            ok = all(torch.equal(y.to("cuda:0"), ref.to(dtype)) for y in ys)
            out.append("ok" if ok else "bad")
print("RESULT", supported, ",".join(out), nc.custom_calls(ALGO["ar_nvls"]))
print("\n".join(l for l in nc.summary_text().splitlines() if not l.endswith("calls=0")))
"""


def run_child(n, extra_env):
    env = dict(os.environ, NCCL_B200_NVLS="on", NCCL_B200_ALGO="ar=nvls", NCCL_B200_TUNE="0",
               NCCL_B200_SUMMARY="1", **extra_env)
    r = subprocess.run([sys.executable, "-c", CHILD.format(repo=REPO, n=n)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    return int(line[1]), line[2].split(","), int(line[3]), r.stdout


@pytest.mark.parametrize("n", [2, 4, 8])
def test_nvls_allreduce(n):
    need_gpus(n)
    supported, results, calls, log = run_child(n, {})
    assert all(r == "ok" for r in results), (results, log)
    if supported:
        assert calls >= len(results), "NVLS route did not run:\n" + log


KINDS_CHILD = r"""
import sys, ctypes as C, torch
sys.path.insert(0, {repo!r}); sys.path.insert(0, {repo!r} + "/tests")
from scc26_nccl_shim_b200.parallel.nccl import Nccl
from scc26_nccl_shim_b200._core import ALGO
from test_gpu_abi import run_kind
n = {n}
devs = list(range(n))
nc = Nccl("interposer")
comms = nc.comm_init_all(devs)
for kind in ("broadcast", "allgather", "reducescatter"):
    c = (48 << 20) // 4 // n if kind != "broadcast" else (300 << 20) // 4
    for inplace in (False, True):
        run_kind(nc, kind, comms, devs, c, inplace=inplace, root=n - 1)
    run_kind(nc, kind, comms, devs, c, dtype=torch.bfloat16)
print("RESULT", nc.custom_calls(ALGO["bc_nvls"]), nc.custom_calls(ALGO["ag_nvls"]),
      nc.custom_calls(ALGO["rs_nvls"]))
"""


@pytest.mark.parametrize("n", [2, 4, 8])
def test_nvls_broadcast_allgather_reducescatter(n):
    need_gpus(n)
    env = dict(os.environ, NCCL_B200_NVLS="on", NCCL_B200_ALGO="bc=nvls,ag=nvls,rs=nvls",
               NCCL_B200_TUNE="0", NCCL_B200_FIRST_PASS="0", NCCL_B200_RS_MIN="1K",
               NCCL_B200_AG_MIN="1K")
    r = subprocess.run([sys.executable, "-c", KINDS_CHILD.format(repo=REPO, n=n)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    assert all(int(x) >= 3 for x in line[1:]), line


TIMEOUT_CHILD = r"""
import sys, ctypes as C, torch
sys.path.insert(0, {repo!r})
from scc26_nccl_shim_b200.parallel.nccl import Nccl, collective, NcclError
nc = Nccl("interposer")
arr = (C.c_int * 2)(0, 1)
if not nc.shim.nb_nvls_supported(arr, 2):
    print("RESULT unsupported"); sys.exit(0)
comms = nc.comm_init_all([0, 1])
xs = [torch.ones(16 << 20, device=f"cuda:{{d}}") for d in (0, 1)]
ys = [torch.empty_like(x) for x in xs]
s = [torch.cuda.current_stream(d).cuda_stream for d in (0, 1)]
out = []
for i in range(4):
    try:
        collective(nc, "allreduce", xs, ys, comms, s)
        for d in (0, 1): torch.cuda.synchronize(d)
        out.append("ok" if all(torch.equal(y, 2 * x) for x, y in zip(xs, ys)) else "stale")
    except NcclError as e:
        for d in (0, 1): torch.cuda.synchronize(d)
        out.append("err%d" % e.code)
    out.append("s%d" % nc.shim.nb_nvls_status(arr, 2))
print("RESULT", ",".join(out), nc.shim.nb_poisoned())
"""


def test_nvls_bounded_wait_reports_timeout():
    """A barrier target nothing can reach, on a 2-GPU clique: every in-kernel
    wait runs out after 200 ms, the kernels record the status and return (the
    GPUs stay usable), the next call returns ncclUnhandledCudaError and later
    calls use NCCL. No rank dies and no GPU faults."""
    need_gpus(2)
    env = dict(os.environ, NCCL_B200_NVLS="on", NCCL_B200_ALGO="ar=nvls", NCCL_B200_TUNE="0",
               NCCL_B200_TEST_NVLS_SKEW="1000", NCCL_B200_TIMEOUT_MS="200")
    r = subprocess.run([sys.executable, "-c", TIMEOUT_CHILD.format(repo=REPO)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    if line[1] == "unsupported":
        pytest.skip("multicast objects unavailable on this GPU")
    seq = line[1].split(",")
    # call 1: first pass on NCCL; call 2: NVLS kernel times out (status 1);
    # call 3: reported as an error and the process is poisoned; call 4: NCCL.
    assert seq[0] == "ok" and seq[1] == "s0"
    assert seq[3] == "s1", seq
    assert seq[4] == "err1", seq
    assert seq[6] == "ok", seq
    assert line[2] == "1"


HYBRID_CHILD = r"""
import sys, torch
sys.path.insert(0, {repo!r}); sys.path.insert(0, {repo!r} + "/tests")
from scc26_nccl_shim_b200.parallel.nccl import Nccl
from scc26_nccl_shim_b200._core import ALGO
from test_gpu_abi import run_kind
n = {n}
devs = list(range(n))
nc = Nccl("interposer")
comms = nc.comm_init_all(devs)
for c in ((64 << 20) // 4, (100 << 20) // 4 + 4, (48 << 20) // 4):
    run_kind(nc, "allreduce", comms, devs, c)
    run_kind(nc, "allreduce", comms, devs, c, inplace=True)
run_kind(nc, "allreduce", comms, devs, (64 << 20) // 2, dtype=torch.bfloat16)
run_kind(nc, "allreduce", comms, devs, (64 << 20) // 4, op="avg")
print("RESULT", nc.custom_calls(ALGO["ar_hybrid"]))
"""


@pytest.mark.parametrize("n", [2, 4])
def test_forced_hybrid_takes_the_static_route(n):
    """The hybrid routes are refused (wrong data at 4 GiB, measured): forcing
    ar=hybrid runs the static route and the result is exact."""
    need_gpus(n)
    env = dict(os.environ, NCCL_B200_NVLS="on", NCCL_B200_ALGO="ar=hybrid", NCCL_B200_TUNE="0",
               NCCL_B200_FIRST_PASS="0")
    r = subprocess.run([sys.executable, "-c", HYBRID_CHILD.format(repo=REPO, n=n)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    assert int(line[1]) == 0, line
