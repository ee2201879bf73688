"""The allocation-free staged AllReduce entry point, called through its exported
C symbol, against the library's existing staged AllReduce (the virtual-rank
plan runner, whose scratch the executor allocates) and against a torch fp32
fold in rank order. The dtype argument is an ncclDataType_t value. Callers that cannot
allocate device memory (allocator hooks, capture-sensitive code, hosts that
own all device memory) use this entry point; it stages through a fixed
file-scope device array instead. Two calls in a row must both match, which
also shows the shared array carries nothing wrong from one call to the next.

This file is collected last on purpose (its name), so a failing run that
stops at the first failure has already run every other test."""
import ctypes as C

import pytest
import torch

from conftest import need_gpus

pytestmark = pytest.mark.gpu


def entry():
    from scc26_nccl_shim_b200.ops import emu
    L = emu.lib()  # libnccl_b200.so, loaded from the repository tree
    fn = L.nb_staged_allreduce_noalloc
    fn.argtypes = [C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_int, C.c_uint64, C.c_int,
                   C.c_void_p, C.c_char_p, C.c_size_t]
    fn.restype = C.c_int
    L.nb_noalloc_scratch_bytes.restype = C.c_uint64
    return fn, int(L.nb_noalloc_scratch_bytes())


# ncclDataType_t values (nccl.h): ncclFloat16 = 6, ncclFloat32 = 7, ncclBfloat16 = 9.
DTYPE_CODE = {torch.float32: 7, torch.float16: 6, torch.bfloat16: 9}
NCCL_FLOAT64 = 8


def data(n, count, dtype, seed):
    g = torch.Generator(device="cuda:0").manual_seed(seed)
    lim = {torch.float32: 1 << 16, torch.float16: 2048 // n, torch.bfloat16: 256 // n}[dtype]
    return [torch.randint(-lim, lim + 1, (count,), device="cuda:0", generator=g).to(dtype)
            for _ in range(n)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [2, 3, 8])
def test_noalloc_matches_staged_route(dtype, n):
    need_gpus(1)
    from scc26_nccl_shim_b200.ops import emu
    fn, cap = entry()
    count = (1 << 20) + 5
    stream = torch.cuda.current_stream(0).cuda_stream
    err = C.create_string_buffer(256)
    for call in range(2):  # two calls in a row
        sends = data(n, count, dtype, seed=10 * n + call)
        ours = [torch.full_like(sends[0], 7) for _ in range(n)]
        ptrs = lambda ts: (C.c_void_p * n)(*[t.data_ptr() for t in ts])  # noqa: E731
        rc = fn(ptrs(sends), ptrs(ours), n, count, DTYPE_CODE[dtype], C.c_void_p(stream), err, 256)
        assert rc == 0, (rc, err.value)
        ref = [torch.empty_like(sends[0]) for _ in range(n)]
        emu.plan("ar_staged", "allreduce", sends, ref)
        fold = sends[0].float()
        for q in range(1, n):
            fold = fold + sends[q].float()
        fold = fold.to(dtype)
        torch.cuda.synchronize()
        for r in range(n):
            assert torch.equal(ours[r], ref[r]), (call, r)
            assert torch.equal(ours[r], fold), (call, r)


def test_noalloc_rejects_oversized_messages():
    need_gpus(1)
    fn, cap = entry()
    n = 2
    count = cap // 4 + 1024  # fp32: one slice alone is larger than half the scratch... and more
    count *= 2
    x = [torch.zeros(8, device="cuda:0") for _ in range(n)]
    err = C.create_string_buffer(256)
    ptrs = (C.c_void_p * n)(*[t.data_ptr() for t in x])
    rc = fn(ptrs, ptrs, n, count, DTYPE_CODE[torch.float32], C.c_void_p(0), err, 256)
    assert rc == -2
    assert b"static scratch holds" in err.value


def test_noalloc_rejects_bad_dtype_and_overflowing_count():
    need_gpus(1)
    fn, cap = entry()
    n = 2
    x = [torch.zeros(8, device="cuda:0") for _ in range(n)]
    err = C.create_string_buffer(256)
    ptrs = (C.c_void_p * n)(*[t.data_ptr() for t in x])
    # ncclFloat64 is not one of the entry point's types.
    assert fn(ptrs, ptrs, n, 8, NCCL_FLOAT64, C.c_void_p(0), err, 256) == -1
    assert b"ncclFloat32" in err.value
    # A count whose byte size wraps 64 bits is refused before any arithmetic.
    assert fn(ptrs, ptrs, n, (1 << 63) + 1, DTYPE_CODE[torch.float32], C.c_void_p(0), err, 256) == -1
    assert b"overflows" in err.value
