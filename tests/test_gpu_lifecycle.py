"""Communicator lifecycle and host-side concurrency through the interposer,
each case in a fresh child process (the interposer's state is per process):

- grouped ncclCommInitRank calls with one unique id form a clique;
- a lifecycle call (ncclCommRegister) forgets the clique, so the next
  collective falls back with NotClique;
- a reversed device list ({1,0}) forms a clique with rank 0 on device 1;
- the caller's current device survives ncclGroupEnd;
- two host threads, each with its own one-GPU clique, run back-to-back
  AllReduces at the same time (the exec lock and the per-thread group state);
- buffers from ncclMemAlloc (VMM) give correct results.

Counterparts in the reference: shim.cu:1472-1505 (grouped InitRank pairing),
:1434-1444 (forget on lifecycle calls), stress.cu:887 (reversed devlist),
:1003-1007 (current device), :622-639 (two threads), :597-604 (ncclMemAlloc).
"""
import json
import os
import subprocess
import sys
import textwrap

import pytest

from conftest import REPO, need_gpus

pytestmark = pytest.mark.gpu

PRELUDE = textwrap.dedent("""
    import ctypes as C, json, os, sys, threading
    import torch
    from scc26_nccl_shim_b200._core import ALGO, REASON
    from scc26_nccl_shim_b200.parallel.nccl import Nccl, collective
    nc = Nccl("interposer")
    nc.shim.nb_custom_calls.restype = C.c_int
    def custom():
        return sum(nc.custom_calls(a) for a in range(1, len(ALGO)))
    def ar(comms, devs, count=(64 << 20) // 4, fill=None):
        sends = [torch.full((count,), float(i + 1), device=f"cuda:{d}") for i, d in enumerate(devs)]
        recvs = [torch.empty(count, device=f"cuda:{d}") for d in devs]
        streams = [torch.cuda.current_stream(d).cuda_stream for d in devs]
        collective(nc, "allreduce", sends, recvs, comms, streams)
        for d in devs:
            torch.cuda.synchronize(d)
        want = float(sum(range(1, len(devs) + 1)))
        return all(bool((r == want).all()) for r in recvs)
""")


def child(body: str, timeout=600):
    code = PRELUDE + textwrap.dedent(body)
    env = dict(os.environ, NCCL_B200_TUNE="0")
    r = subprocess.run([sys.executable, "-c", code], cwd=REPO, env=env, capture_output=True,
                       text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    return json.loads(line)


def test_grouped_initrank_forms_clique_and_register_forgets_it():
    need_gpus(2)
    out = child("""
        devs = [0, 1]
        class UniqueId(C.Structure):  # ncclUniqueId, passed by value to InitRank
            _fields_ = [("internal", C.c_char * 128)]
        uid = UniqueId()
        assert nc._fn("ncclGetUniqueId")(C.byref(uid)) == 0
        comms = [C.c_void_p() for _ in devs]
        assert nc.group_start() == 0
        for r, d in enumerate(devs):
            torch.cuda.set_device(d)
            assert nc._fn("ncclCommInitRank")(C.byref(comms[r]), len(devs), uid, r) == 0
        assert nc.group_end() == 0
        comms = [c.value for c in comms]
        ok1 = ar(comms, devs)            # the first eligible call runs on NCCL
        c0 = custom()
        ok2 = ar(comms, devs)            # a clique from grouped InitRank: custom
        c1 = custom()
        torch.cuda.set_device(0)
        buf = torch.empty(1 << 20, device="cuda:0")
        handle = C.c_void_p()
        rc = nc._fn("ncclCommRegister")(C.c_void_p(comms[0]), C.c_void_p(buf.data_ptr()),
                                        C.c_size_t(buf.numel() * 4), C.byref(handle))
        nc_before = nc.fallbacks(REASON["NotClique"])
        ok3 = ar(comms, devs)            # clique forgotten: falls back
        c2 = custom()
        nc_after = nc.fallbacks(REASON["NotClique"])
        if rc == 0:
            nc._fn("ncclCommDeregister")(C.c_void_p(comms[0]), handle)
        for c in comms:
            nc.comm_destroy(c)
        print(json.dumps(dict(ok=[ok1, ok2, ok3], custom=[c0, c1, c2], register_rc=rc,
                              notclique=[nc_before, nc_after])))
    """)
    assert out["ok"] == [True, True, True]
    c0, c1, c2 = out["custom"]
    assert c1 == c0 + 1, out
    assert c2 == c1, out
    assert out["notclique"][1] > out["notclique"][0], out


def test_reversed_devlist_and_current_device_restored():
    need_gpus(2)
    out = child("""
        devs = [1, 0]
        comms = nc.comm_init_all(devs)
        ar(comms, devs)
        c0 = custom()
        torch.cuda.set_device(1)
        ok = ar(comms, devs)
        cur = torch.cuda.current_device()
        # reversed call order inside the group as well
        count = (64 << 20) // 4
        sends = [torch.full((count,), float(i + 1), device=f"cuda:{d}") for i, d in enumerate(devs)]
        recvs = [torch.empty(count, device=f"cuda:{d}") for d in devs]
        streams = [torch.cuda.current_stream(d).cuda_stream for d in devs]
        torch.cuda.set_device(0)
        with nc.group():
            for i in (1, 0):
                nc.all_reduce(sends[i], recvs[i], comms[i], streams[i])
        cur2 = torch.cuda.current_device()
        for d in devs:
            torch.cuda.synchronize(d)
        ok2 = all(bool((r == 3.0).all()) for r in recvs)
        c1 = custom()
        for c in comms:
            nc.comm_destroy(c)
        print(json.dumps(dict(ok=[ok, ok2], cur=[cur, cur2], custom=[c0, c1])))
    """)
    assert out["ok"] == [True, True]
    assert out["cur"] == [1, 0]
    assert out["custom"][1] == out["custom"][0] + 2


def test_two_threads_with_their_own_cliques():
    need_gpus(2)
    out = child("""
        results = {}
        barrier = threading.Barrier(2)
        def work(dev):
            torch.cuda.set_device(dev)
            comms = nc.comm_init_all([dev])
            barrier.wait()
            ok = True
            for it in range(6):
                ok &= ar(comms, [dev])
            results[dev] = ok
            barrier.wait()
            nc.comm_destroy(comms[0])
        ts = [threading.Thread(target=work, args=(d,)) for d in (0, 1)]
        for t in ts: t.start()
        for t in ts: t.join()
        print(json.dumps(dict(ok=[results.get(0), results.get(1)], custom=custom())))
    """)
    assert out["ok"] == [True, True]
    assert out["custom"] >= 10  # all but the process's first eligible call


def test_ncclmemalloc_buffers():
    need_gpus(2)
    out = child("""
        devs = [0, 1]
        comms = nc.comm_init_all(devs)
        count = (64 << 20) // 4
        nbytes = count * 4
        ptrs = []
        for d in devs:
            torch.cuda.set_device(d)
            p = C.c_void_p()
            assert nc._fn("ncclMemAlloc")(C.byref(p), C.c_size_t(2 * nbytes)) == 0
            ptrs.append(p.value)
        streams = [torch.cuda.current_stream(d).cuda_stream for d in devs]
        cudart = C.CDLL("libcudart.so.12")
        cudart.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
        D2D = 3
        oks = []
        for it in range(3):
            for r, d in enumerate(devs):
                with torch.cuda.device(d):
                    t = torch.full((count,), float(r + 1 + it), device=f"cuda:{d}")
                    torch.cuda.synchronize(d)
                    assert cudart.cudaMemcpy(ptrs[r], t.data_ptr(), nbytes, D2D) == 0
            dt = 7  # ncclFloat32
            assert nc.group_start() == 0
            for r, d in enumerate(devs):
                nc._fn("ncclAllReduce")(C.c_void_p(ptrs[r]), C.c_void_p(ptrs[r] + nbytes),
                                        C.c_size_t(count), dt, 0, C.c_void_p(comms[r]),
                                        C.c_void_p(streams[r]))
            assert nc.group_end() == 0
            ok = True
            for r, d in enumerate(devs):
                torch.cuda.synchronize(d)
                with torch.cuda.device(d):
                    out = torch.empty(count, device=f"cuda:{d}")
                    assert cudart.cudaMemcpy(out.data_ptr(), ptrs[r] + nbytes, nbytes, D2D) == 0
                    torch.cuda.synchronize(d)
                    ok &= bool((out == float(3 + 2 * it)).all())
            oks.append(ok)
        for r, d in enumerate(devs):
            torch.cuda.set_device(d)
            nc._fn("ncclMemFree")(C.c_void_p(ptrs[r]))
        for c in comms:
            nc.comm_destroy(c)
        print(json.dumps(dict(ok=oks, custom=custom())))
    """)
    assert out["ok"] == [True, True, True]
