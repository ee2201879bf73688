"""The buffer classification table (core/bufclass.h) on facts built by hand:
which caller buffers the clique kernels may address from every GPU. The
executor gathers the same facts from the CUDA driver on a GPU box."""
import ctypes as C

import pytest

from scc26_nccl_shim_b200 import _core

NO_MAPPING, NO_FLAGS, READ_WRITE, OTHER, FAILED = range(5)
REFUSED, ORDINARY, MAPPED = 0, 1, 2


class Facts(C.Structure):
    _fields_ = [("known", C.c_int), ("device_memory", C.c_int), ("device", C.c_int),
                ("from_pool", C.c_int), ("legacy_ipc", C.c_int), ("ndev", C.c_int),
                ("range_start", C.c_uint64), ("range_size", C.c_uint64),
                ("mapping_start", C.c_uint64), ("mapping_size", C.c_uint64),
                ("access", C.c_int * 8)]


BASE, SIZE = 1 << 40, 1 << 30


def facts(**kw):
    f = Facts(known=1, device_memory=1, device=0, from_pool=0, legacy_ipc=1, ndev=2,
              range_start=BASE, range_size=SIZE, mapping_start=BASE, mapping_size=SIZE)
    acc = kw.pop("access", [NO_MAPPING, NO_MAPPING])
    for i, a in enumerate(acc):
        f.access[i] = a
    for k, v in kw.items():
        setattr(f, k, v)
    return f


def classify(first, last=None, addr=BASE, nbytes=1 << 20, device=0):
    L = _core.lib()
    fn = L.nb_classify_buffer
    fn.argtypes = [C.POINTER(Facts), C.POINTER(Facts), C.c_uint64, C.c_uint64, C.c_int, C.c_char_p,
                   C.c_size_t]
    rule = C.create_string_buffer(64)
    cls = fn(C.byref(first), C.byref(last if last is not None else first), addr, nbytes, device, rule, 64)
    return cls, rule.value.decode()


def test_ordinary_cudamalloc_buffer():
    for acc in ([NO_MAPPING, NO_MAPPING], [NO_FLAGS, READ_WRITE]):
        assert classify(facts(access=acc))[0] == ORDINARY


def test_vmm_buffer_mapped_everywhere():
    f = facts(legacy_ipc=0, access=[READ_WRITE, READ_WRITE])
    assert classify(f) == (MAPPED, "mapped-read-write-everywhere")


@pytest.mark.parametrize("change,rule", [
    (dict(known=0), "known-to-driver"),
    (dict(device_memory=0), "device-memory"),
    (dict(device=1), "on-expected-device"),
    (dict(from_pool=1), "not-pool-memory"),
    (dict(access=[READ_WRITE, FAILED]), "access-queries-answered"),
    (dict(legacy_ipc=0, access=[READ_WRITE, NO_MAPPING]), "neither-ordinary-nor-mapped"),
    (dict(legacy_ipc=1, access=[OTHER, NO_MAPPING]), "neither-ordinary-nor-mapped"),
    (dict(legacy_ipc=-1), "neither-ordinary-nor-mapped"),
])
def test_refusals_name_their_rule(change, rule):
    assert classify(facts(**change)) == (REFUSED, rule)


def test_range_must_stay_in_one_allocation():
    f = facts()
    assert classify(f, addr=BASE + SIZE - 16, nbytes=32) == (REFUSED, "one-allocation")
    assert classify(f, addr=BASE - 16, nbytes=32) == (REFUSED, "one-allocation")
    assert classify(f, nbytes=0) == (REFUSED, "non-empty")
    assert classify(f, addr=(1 << 64) - 8, nbytes=16) == (REFUSED, "non-empty")
    other = facts(range_start=BASE + SIZE)
    assert classify(f, other) == (REFUSED, "one-allocation")


def test_vmm_ends_in_different_mappings_refused():
    a = facts(legacy_ipc=0, access=[READ_WRITE, READ_WRITE])
    b = facts(legacy_ipc=0, access=[READ_WRITE, READ_WRITE], mapping_start=BASE + SIZE // 2)
    assert classify(a, b) == (REFUSED, "one-mapping")
    # Ordinary memory is one allocation whatever mapping the driver reports.
    c = facts(mapping_start=BASE + SIZE // 2)
    assert classify(facts(), c)[0] == ORDINARY


def test_ends_disagreeing_on_access_refused():
    a = facts(legacy_ipc=0, access=[READ_WRITE, READ_WRITE])
    b = facts(legacy_ipc=0, access=[READ_WRITE, NO_FLAGS])
    assert classify(a, b) == (REFUSED, "neither-ordinary-nor-mapped")
