"""A small client of the NCCL C ABI (ctypes), for single-process multi-GPU use.

Three ways to reach the collectives:

* ``mode="interposer"``: load ``libnccl_b200.so`` directly and call its
  exported NCCL symbols (the interposer forwards what it does not handle to
  the real libnccl, which is loaded RTLD_GLOBAL first).
* ``mode="preload"``: the process was started with ``LD_PRELOAD=<shim>``;
  symbols are looked up in the global scope, so the preloaded shim (ours or
  the reference's) wins, exactly as for any NCCL application.
* ``mode="nccl"``: the real libnccl only (the baseline).

Buffers are torch tensors; streams are torch CUDA streams.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import os

from .. import LIB_PATH, real_nccl_path, require

ncclSuccess = 0
DT = {"int8": 0, "uint8": 1, "int32": 2, "uint32": 3, "int64": 4, "uint64": 5,
      "float16": 6, "float32": 7, "float64": 8, "bfloat16": 9}
OPS = {"sum": 0, "prod": 1, "max": 2, "min": 3, "avg": 4}
TORCH_DT = {"torch.int8": "int8", "torch.uint8": "uint8", "torch.int32": "int32",
            "torch.int64": "int64", "torch.float16": "float16", "torch.float32": "float32",
            "torch.float64": "float64", "torch.bfloat16": "bfloat16"}


class NcclError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} returned {code}")
        self.code = code


class Nccl:
    def __init__(self, mode: str = "interposer"):
        self.mode = mode
        self.real = C.CDLL(real_nccl_path(), mode=C.RTLD_GLOBAL)
        if mode == "interposer":
            self.api = C.CDLL(require(LIB_PATH), mode=C.RTLD_GLOBAL)
        elif mode == "preload":
            self.api = C.CDLL(None)
        elif mode == "nccl":
            self.api = self.real
        else:
            raise ValueError(mode)
        self.shim = None
        if mode == "interposer":
            self.shim = self.api
        elif mode == "preload" and hasattr(C.CDLL(None), "nb_custom_calls"):
            self.shim = C.CDLL(None)

    def _fn(self, name):
        try:
            return getattr(self.api, name)
        except AttributeError:
            return getattr(self.real, name)

    def _ck(self, name, *args):
        r = self._fn(name)(*args)
        if r != ncclSuccess:
            raise NcclError(name, r)
        return r

    def version(self) -> int:
        v = C.c_int(0)
        self._ck("ncclGetVersion", C.byref(v))
        return v.value

    def comm_init_all(self, devices: list[int]) -> list[int]:
        n = len(devices)
        comms = (C.c_void_p * n)()
        devs = (C.c_int * n)(*devices)
        self._ck("ncclCommInitAll", comms, n, devs)
        return [comms[i] for i in range(n)]

    def comm_destroy(self, comm) -> None:
        self._ck("ncclCommDestroy", C.c_void_p(comm))

    def group_start(self):
        return self._fn("ncclGroupStart")()

    def group_end(self):
        return self._fn("ncclGroupEnd")()

    @contextlib.contextmanager
    def group(self):
        r = self.group_start()
        if r != ncclSuccess:
            raise NcclError("ncclGroupStart", r)
        err = None
        try:
            yield
        finally:
            r = self.group_end()
            if r != ncclSuccess:
                err = NcclError("ncclGroupEnd", r)
        if err:
            raise err

    @staticmethod
    def _dt(t) -> int:
        return DT[TORCH_DT[str(t.dtype)]]

    def all_reduce(self, send, recv, comm, stream, op="sum", count=None):
        count = send.numel() if count is None else count
        opv = OPS[op] if isinstance(op, str) else int(op)
        return self._fn("ncclAllReduce")(C.c_void_p(send.data_ptr()), C.c_void_p(recv.data_ptr()),
                                         C.c_size_t(count), self._dt(send), opv, C.c_void_p(comm),
                                         C.c_void_p(stream))

    def all_gather(self, send, recv, comm, stream, count=None):
        count = send.numel() if count is None else count
        return self._fn("ncclAllGather")(C.c_void_p(send.data_ptr()), C.c_void_p(recv.data_ptr()),
                                         C.c_size_t(count), self._dt(send), C.c_void_p(comm),
                                         C.c_void_p(stream))

    def reduce_scatter(self, send, recv, comm, stream, op="sum", count=None):
        count = recv.numel() if count is None else count
        opv = OPS[op] if isinstance(op, str) else int(op)
        return self._fn("ncclReduceScatter")(C.c_void_p(send.data_ptr()), C.c_void_p(recv.data_ptr()),
                                             C.c_size_t(count), self._dt(send), opv,
                                             C.c_void_p(comm), C.c_void_p(stream))

    def broadcast(self, send, recv, root, comm, stream, count=None):
        count = recv.numel() if count is None else count
        sp = send.data_ptr() if send is not None else recv.data_ptr()
        return self._fn("ncclBroadcast")(C.c_void_p(sp), C.c_void_p(recv.data_ptr()),
                                         C.c_size_t(count), self._dt(recv), int(root),
                                         C.c_void_p(comm), C.c_void_p(stream))

    def premul_sum(self, scalar: float, dtype: str, comm) -> int:
        op = C.c_int(0)
        if dtype == "float32":
            s = C.c_float(scalar)
        elif dtype == "float64":
            s = C.c_double(scalar)
        else:
            import struct
            import numpy as np
            h = np.array([scalar], dtype=np.float32)
            if dtype == "float16":
                v = h.astype(np.float16).view(np.uint16)[0]
            else:
                v = (h.view(np.uint32)[0] + 0x7FFF + ((h.view(np.uint32)[0] >> 16) & 1)) >> 16
            s = C.c_uint16(int(v))
            del struct
        self._ck("ncclRedOpCreatePreMulSum", C.byref(op), C.byref(s), DT[dtype], 1, C.c_void_p(comm))
        return op.value

    def redop_destroy(self, op: int, comm) -> None:
        self._ck("ncclRedOpDestroy", int(op), C.c_void_p(comm))

    # Interposer introspection (None when running on the real NCCL only).
    def custom_calls(self, algo: int) -> int | None:
        return None if self.shim is None else self.shim.nb_custom_calls(algo)

    def fallbacks(self, reason: int) -> int | None:
        return None if self.shim is None else self.shim.nb_fallbacks(reason)

    def kernel_launches(self) -> int | None:
        if self.shim is None or not hasattr(self.shim, "nb_kernel_launches"):
            return None
        self.shim.nb_kernel_launches.restype = C.c_uint64
        return int(self.shim.nb_kernel_launches())

    def summary_text(self) -> str:
        if self.shim is None:
            return ""
        buf = C.create_string_buffer(1 << 16)
        self.shim.nb_summary_text(buf, 1 << 16)
        return buf.value.decode()


def collective(nc: Nccl, kind: str, sends, recvs, comms, streams, op="sum", root=0):
    """One grouped collective over every rank of a clique (rank i = comms[i]).
    `op` is one op for every rank (a name or an ncclRedOp_t value), or a list
    with one per rank (PreMulSum ops are created per communicator)."""
    with nc.group():
        for i, comm in enumerate(comms):
            s = streams[i]
            o = op[i] if isinstance(op, (list, tuple)) else op
            if kind == "allreduce":
                r = nc.all_reduce(sends[i], recvs[i], comm, s, o)
            elif kind == "allgather":
                r = nc.all_gather(sends[i], recvs[i], comm, s)
            elif kind == "reducescatter":
                r = nc.reduce_scatter(sends[i], recvs[i], comm, s, o)
            elif kind == "broadcast":
                r = nc.broadcast(sends[i], recvs[i], root, comm, s)
            else:
                raise ValueError(kind)
            if r != ncclSuccess:
                raise NcclError(kind, r)


def preload_env(lib: str, extra: dict | None = None) -> dict:
    """Environment for a child process that preloads `lib` over torch's libnccl."""
    env = dict(os.environ)
    nccl_dir = os.path.dirname(real_nccl_path())
    env["LD_PRELOAD"] = lib
    env["LD_LIBRARY_PATH"] = nccl_dir + (":" + env["LD_LIBRARY_PATH"] if env.get("LD_LIBRARY_PATH") else "")
    env.update(extra or {})
    return env
