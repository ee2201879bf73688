"""The interposer through its public NCCL ABI on real GPUs.

One-GPU cases use a one-rank clique (ncclCommInitAll over [0]); the
multi-GPU cases run when the process sees two or more GPUs. Results are
compared with a torch fp32 reference; the interposer's own counters show
which calls ran on its kernels and which fell back to libnccl.
"""
import os
import subprocess
import sys

import pytest
import torch

from conftest import REPO, gpu_count, need_gpus

pytestmark = pytest.mark.gpu

from scc26_nccl_shim_b200._core import ALGO  # noqa: E402


@pytest.fixture(scope="module")
def nc():
    need_gpus(1)
    from scc26_nccl_shim_b200.parallel.nccl import Nccl
    return Nccl("interposer")


def run_kind(nc, kind, comms, devs, count, dtype=torch.float32, op="sum", inplace=False, root=0):
    from scc26_nccl_shim_b200.parallel.nccl import collective
    n = len(devs)
    streams = [torch.cuda.current_stream(d).cuda_stream for d in devs]
    gens = [torch.Generator(device=f"cuda:{d}").manual_seed(100 + d) for d in devs]
    # Every partial sum must be exact in the element type, so any reduction
    # order (the NVSwitch's included) gives the same bits: |sum| <= 256 for
    # bf16 (8-bit significand), <= 2048 for fp16.
    lim = {torch.bfloat16: 256 // n, torch.float16: 2048 // n}.get(dtype, 1023)
    def data(d, c):
        return torch.randint(-lim, lim + 1, (c,), device=f"cuda:{d}", generator=gens[devs.index(d)]).to(dtype)
    if kind == "reducescatter":
        sends = [data(d, count * n) for d in devs]
        recvs = [s[r * count:(r + 1) * count] if inplace else torch.empty(count, dtype=dtype, device=f"cuda:{d}")
                 for r, (d, s) in enumerate(zip(devs, sends))]
    elif kind == "allgather":
        recvs = [torch.empty(count * n, dtype=dtype, device=f"cuda:{d}") for d in devs]
        if inplace:
            sends = [recvs[r][r * count:(r + 1) * count] for r in range(n)]
            for r, d in enumerate(devs):
                sends[r].copy_(data(d, count))
        else:
            sends = [data(d, count) for d in devs]
    else:
        sends = [data(d, count) for d in devs]
        recvs = sends if inplace else [torch.empty(count, dtype=dtype, device=f"cuda:{d}") for d in devs]
    inputs = [s.to("cuda:0").clone() for s in sends]
    collective(nc, kind, sends, recvs, comms, streams, op=op, root=root)
    for d in devs:
        torch.cuda.synchronize(d)
    for r in range(n):
        if kind == "allreduce":
            ref = inputs[0].float()
            for x in inputs[1:]:  # rank order, fp32, like the fused fold
                ref = {"max": torch.maximum, "min": torch.minimum,
                       "prod": torch.mul}.get(op, torch.add)(ref, x.float())
            if op == "avg":  # a true division (torch's tensor / scalar multiplies by 1/n)
                ref = torch.div(ref, torch.full_like(ref, float(n)))
            ref = ref.to(dtype)
        elif kind == "reducescatter":
            ref = inputs[0][r * count:(r + 1) * count].float()
            for x in inputs[1:]:
                ref = ref + x[r * count:(r + 1) * count].float()
            ref = ref.to(dtype)
        elif kind == "allgather":
            ref = torch.cat(inputs)
        else:
            ref = inputs[root]
        got = recvs[r].to("cuda:0")
        assert torch.equal(got, ref), (kind, r)


def test_one_rank_clique(nc):
    devs = [0]
    comms = nc.comm_init_all(devs)
    count = (32 << 20) // 4 + 12  # at the 32 MiB threshold
    for kind in ("allreduce", "allgather", "reducescatter", "broadcast"):
        c = count if kind != "reducescatter" else count - count % 4
        before = sum(nc.custom_calls(a) for a in ALGO.values() if a)
        run_kind(nc, kind, comms, devs, c)
        run_kind(nc, kind, comms, devs, c, inplace=True)
        after = sum(nc.custom_calls(a) for a in ALGO.values() if a)
        assert after > before, kind
    # A length that ends inside a 16-byte unit (the bulk copy's byte tail).
    run_kind(nc, "allreduce", comms, devs, count + 1, dtype=torch.bfloat16)
    run_kind(nc, "broadcast", comms, devs, (48 << 20) // 4 + 3, dtype=torch.bfloat16)
    nc.comm_destroy(comms[0])


def test_one_rank_below_threshold_falls_back(nc):
    comms = nc.comm_init_all([0])
    before = nc.fallbacks(6)  # BelowThreshold
    run_kind(nc, "allreduce", comms, [0], 1000)
    assert nc.fallbacks(6) > before
    nc.comm_destroy(comms[0])


def test_capture_falls_back(nc):
    """A capturing caller stream is never run on the custom path."""
    from scc26_nccl_shim_b200.parallel.nccl import collective
    comms = nc.comm_init_all([0])
    x = torch.ones(16 << 20, device="cuda:0")
    y = torch.empty_like(x)
    s = torch.cuda.Stream(0)
    collective(nc, "allreduce", [x], [y], comms, [s.cuda_stream])  # consume FirstPass
    torch.cuda.synchronize()
    before = nc.fallbacks(14)  # Capturing
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        collective(nc, "allreduce", [x], [y], comms, [s.cuda_stream])
    assert nc.fallbacks(14) > before
    y.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(x, y)
    del g
    nc.comm_destroy(comms[0])


@pytest.mark.parametrize("n", [2, 4, 8])
def test_multi_gpu_collectives(nc, n):
    need_gpus(n)
    devs = list(range(n))
    comms = nc.comm_init_all(devs)
    count = (64 << 20) // 4
    for kind in ("allreduce", "allgather", "reducescatter", "broadcast"):
        c = count // n if kind in ("allgather", "reducescatter") else count
        run_kind(nc, kind, comms, devs, c)  # the first eligible call may run on NCCL
        before = sum(nc.custom_calls(a) for a in ALGO.values() if a)
        run_kind(nc, kind, comms, devs, c, root=n - 1)
        run_kind(nc, kind, comms, devs, c, inplace=True)
        assert sum(nc.custom_calls(a) for a in ALGO.values() if a) >= before + 2, \
            (kind, nc.summary_text())
    run_kind(nc, "allreduce", comms, devs, count, dtype=torch.bfloat16)
    run_kind(nc, "allreduce", comms, devs, count, op="avg")
    for c in comms:
        nc.comm_destroy(c)


FAULT_CHILD = r"""
import sys, torch
sys.path.insert(0, {repo!r})
from scc26_nccl_shim_b200.parallel.nccl import Nccl, collective, NcclError
nc = Nccl("interposer")
comms = nc.comm_init_all([0])
x = torch.ones(16 << 20, device="cuda:0"); y = torch.empty_like(x)
s = [torch.cuda.current_stream(0).cuda_stream]
out = []
for i in range(3):
    try:
        collective(nc, "allreduce", [x], [y], comms, s)
        torch.cuda.synchronize(); out.append("ok" if torch.equal(x, y) else "bad")
    except NcclError as e:
        torch.cuda.synchronize(); out.append("err%d" % e.code)
print(",".join(out), nc.shim.nb_poisoned(), nc.fallbacks(16), nc.fallbacks(17), nc.fallbacks(18))
"""


@pytest.mark.parametrize("spec,expect", [
    # call 1 runs on NCCL (first pass); the injected fault hits call 2.
    ("setup", ("ok,ok,ok", "0")),        # falls back, later calls run custom
    ("op:0", ("ok,ok,ok", "0")),         # a record fails before any data op: falls back
    ("op:1", ("ok,err1,ok", "1")),       # the kernel launch fails: error + poison, later on NCCL
])
def test_host_fault_injection(spec, expect):
    """Error policy with host-side injected CUDA errors (nothing faults on the GPU)."""
    need_gpus(1)
    # No init-time tuning: the one-rank plan is then [record, copy kernel, ...],
    # so op 1 is the kernel launch.
    env = dict(os.environ, NCCL_B200_FAULT=spec, NCCL_B200_TUNE="0")
    r = subprocess.run([sys.executable, "-c", FAULT_CHILD.format(repo=REPO)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    words = r.stdout.strip().splitlines()[-1].split()
    assert words[0] == expect[0], r.stdout + r.stderr[-1000:]
    assert words[1] == expect[1]
