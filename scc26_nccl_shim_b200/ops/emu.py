"""Run the sm_100a kernels on one GPU with virtual ranks (torch tensors).

These call the interposer library's test entry points: `reduce` and `copy`
launch one kernel directly; `plan` runs a complete collective plan for N
virtual ranks whose buffers all live on the current device (the ops run one
after another on one stream, so no kernel waits on another).
"""
from __future__ import annotations

import ctypes as C
import functools

from .. import LIB_PATH, real_nccl_path, require
from .._core import ALGO, DTYPE, KIND, OP

TORCH_TO_DTYPE = {"torch.float32": "float32", "torch.float16": "float16",
                  "torch.bfloat16": "bfloat16", "torch.float64": "float64", "torch.int8": "int8",
                  "torch.uint8": "uint8", "torch.int32": "int32", "torch.int64": "int64"}


@functools.lru_cache(maxsize=1)
def lib() -> C.CDLL:
    C.CDLL(real_nccl_path(), mode=C.RTLD_GLOBAL)
    L = C.CDLL(require(LIB_PATH), mode=C.RTLD_GLOBAL)
    L.nb_emu_reduce.argtypes = [C.POINTER(C.c_void_p), C.c_int, C.POINTER(C.c_void_p), C.c_int,
                                C.c_uint64, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double),
                                C.c_void_p]
    L.nb_emu_copy.argtypes = [C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.POINTER(C.c_uint64),
                              C.c_int, C.c_void_p]
    L.nb_emu_plan.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_int,
                              C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                              C.POINTER(C.c_double), C.c_void_p]
    L.nb_kernel_launches.restype = C.c_uint64
    return L


def _ptrs(ts):
    return (C.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _stream(t):
    import torch
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def reduce(srcs, dsts, op="sum", nranks=None, scalars=None, nbytes=None):
    t = srcs[0]
    dt = DTYPE[TORCH_TO_DTYPE[str(t.dtype)]]
    nb = t.numel() * t.element_size() if nbytes is None else nbytes
    sc = (C.c_double * 8)(*(list(scalars) + [1.0] * (8 - len(scalars)))) if scalars else None
    rc = lib().nb_emu_reduce(_ptrs(srcs), len(srcs), _ptrs(dsts), len(dsts), nb, dt, OP[op],
                             nranks or len(srcs), sc, _stream(t))
    if rc:
        raise RuntimeError(f"nb_emu_reduce failed: CUDA error {rc}")


def copy(srcs, dsts, lens):
    lens_arr = (C.c_uint64 * len(lens))(*lens)
    rc = lib().nb_emu_copy(_ptrs(srcs), _ptrs(dsts), lens_arr, len(srcs), _stream(srcs[0]))
    if rc:
        raise RuntimeError(f"nb_emu_copy failed: CUDA error {rc}")


def plan(algo, kind, sends, recvs, op="sum", root=0, ce_ppm=0, scalars=None, count=None):
    t = recvs[0]
    dt = DTYPE[TORCH_TO_DTYPE[str(t.dtype)]]
    n = len(recvs)
    if count is None:
        count = {"allgather": sends[0].numel(), "reducescatter": recvs[0].numel()}.get(kind, t.numel())
    sc = (C.c_double * 8)(*(list(scalars) + [1.0] * (8 - len(scalars)))) if scalars else None
    send_ptrs = (C.c_void_p * n)(*[(s.data_ptr() if s is not None else recvs[i].data_ptr())
                                   for i, s in enumerate(sends)])
    rc = lib().nb_emu_plan(ALGO[algo], KIND[kind], dt, OP[op], n, count, root, ce_ppm, send_ptrs,
                           _ptrs(recvs), sc, _stream(t))
    if rc:
        raise RuntimeError(f"nb_emu_plan failed: {rc}")


def kernel_launches() -> int:
    return int(lib().nb_kernel_launches())


def bench(kernel: str, n: int, mib: int, dtype: str = "float32", ndst: int = 1, iters: int = 20,
          warmup: int = 3) -> dict:
    """Time one kernel on virtual-rank buffers of the current device with CUDA
    events: `reduce` folds n sources of `mib` MiB into ndst destinations;
    `copy` moves n segments of `mib` MiB. Total sources exceed the 126 MB L2
    for the default sizes, so every launch streams from HBM."""
    import torch
    dt = getattr(torch, dtype)
    es = torch.tensor([], dtype=dt).element_size()
    count = (mib << 20) // es
    srcs = [torch.randn(count, device="cuda").to(dt) for _ in range(n)]
    if kernel == "reduce":
        dsts = [torch.empty_like(srcs[0]) for _ in range(ndst)]
        run = lambda: reduce(srcs, dsts)  # noqa: E731
        moved = (n + ndst) * count * es
    elif kernel == "copy":
        dsts = [torch.empty_like(s) for s in srcs]
        run = lambda: copy(srcs, dsts, [count * es] * n)  # noqa: E731
        moved = 2 * n * count * es
    else:
        raise ValueError(kernel)
    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        run()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    return {"kernel": kernel, "n": n, "mib": mib, "dtype": dtype, "ndst": ndst,
            "ms": round(ms, 4), "hbm_gbs": round(moved / ms / 1e6, 1)}


if __name__ == "__main__":
    import argparse
    import json
    p = argparse.ArgumentParser(description="time one sm_100a collective kernel on one GPU")
    p.add_argument("--kernel", choices=["reduce", "copy"], default="reduce")
    p.add_argument("--n", type=int, default=8)
    p.add_argument("--mib", type=int, default=64)
    p.add_argument("--dtype", default="float32")
    p.add_argument("--ndst", type=int, default=1)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    a = p.parse_args()
    print(json.dumps(bench(a.kernel, a.n, a.mib, a.dtype, a.ndst, a.iters, a.warmup)))
