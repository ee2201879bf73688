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
