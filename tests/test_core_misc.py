"""CPU tests of the CUDA-free core helpers: the host-lane fold against numpy,
the library's own half/bf16 conversions, the calibrated share model and its
JSON cache, the clique registry and grouped-init detection, the per-op fault
policy and the exit-summary format."""
import ctypes as C

import numpy as np
import pytest
import torch

from scc26_nccl_shim_b200 import _core as c


def fold(dtype, op, arrays, nranks=None, scalars=None, threads=3):
    L = c.lib()
    srcs = (C.c_void_p * len(arrays))(*[a.ctypes.data for a in arrays])
    out = np.empty_like(arrays[0])
    sc = (C.c_double * 8)(*(list(scalars) + [1.0] * (8 - len(scalars)))) if scalars else None
    L.nb_host_fold(c.DTYPE[dtype], c.OP[op], nranks or len(arrays), srcs, len(arrays),
                   out.ctypes.data, out.nbytes, sc, threads)
    return out


def rng_f32(seed, n):
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


@pytest.mark.parametrize("nsrc", [2, 3, 8])
def test_fold_f32_sum_is_rank_ordered_fp32(nsrc):
    xs = [rng_f32(i, 100003) for i in range(nsrc)]
    want = xs[0].copy()
    for x in xs[1:]:
        want = want + x  # fp32 adds in rank order
    assert np.array_equal(fold("float32", "sum", xs).view(np.uint32), want.view(np.uint32))


def test_fold_f32_avg_prod_max_min():
    xs = [rng_f32(10 + i, 4099) for i in range(4)]
    xs[1][:3] = [np.nan, 0.0, -0.0]
    xs[2][:3] = [1.0, -0.0, 0.0]
    s = xs[0] + xs[1] + xs[2] + xs[3]
    assert np.array_equal(fold("float32", "avg", xs)[3:], (s / np.float32(4))[3:])
    p = xs[0] * xs[1] * xs[2] * xs[3]
    assert np.array_equal(fold("float32", "prod", xs)[3:], p[3:])
    mx = fold("float32", "max", xs)
    mn = fold("float32", "min", xs)
    assert np.array_equal(mx[3:], np.maximum.reduce(xs)[3:])
    assert np.array_equal(mn[3:], np.minimum.reduce(xs)[3:])
    # NaN loses to a number (IEEE maxNum); +0 beats -0 for max and loses for min
    assert not np.isnan(mx[0]) and not np.isnan(mn[0])
    assert not np.signbit(mx[1]) and not np.signbit(mx[2])
    assert np.signbit(mn[1]) and np.signbit(mn[2])


def test_fold_premulsum_scales_each_rank():
    xs = [np.arange(1000, dtype=np.float32) * (i + 1) for i in range(3)]
    sc = [0.5, 2.0, 0.25]
    want = xs[0] * np.float32(0.5) + xs[1] * np.float32(2.0) + xs[2] * np.float32(0.25)
    assert np.array_equal(fold("float32", "premulsum", xs, scalars=sc), want)


@pytest.mark.parametrize("dtype,npdt,tdt", [("float16", np.float16, torch.float16),
                                            ("bfloat16", np.uint16, torch.bfloat16)])
def test_fold_half_types_accumulate_in_fp32(dtype, npdt, tdt):
    xs32 = [rng_f32(20 + i, 8191) for i in range(5)]
    xs = [torch.from_numpy(x).to(tdt) for x in xs32]
    arrays = [x.view(torch.int16).numpy().view(np.uint16).copy() for x in xs]
    acc = xs[0].float()
    for x in xs[1:]:
        acc = acc + x.float()
    want = acc.to(tdt).view(torch.int16).numpy().view(np.uint16)
    got = fold(dtype, "sum", arrays)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("dtype,npdt", [("int32", np.int32), ("int8", np.int8), ("uint8", np.uint8),
                                        ("int64", np.int64)])
def test_fold_integers_wrap(dtype, npdt):
    info = np.iinfo(npdt)
    xs = [np.random.default_rng(i).integers(info.min, info.max, 5000, dtype=npdt, endpoint=True)
          for i in range(4)]
    with np.errstate(over="ignore"):
        s = xs[0] + xs[1] + xs[2] + xs[3]
        p = xs[0] * xs[1] * xs[2] * xs[3]
    assert np.array_equal(fold(dtype, "sum", xs), s)
    assert np.array_equal(fold(dtype, "prod", xs), p)
    assert np.array_equal(fold(dtype, "max", xs), np.maximum.reduce(xs))
    assert np.array_equal(fold(dtype, "min", xs), np.minimum.reduce(xs))


def test_half_to_float_exhaustive():
    L = c.lib()
    bits = np.arange(1 << 16, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([L.nb_half_to_float(int(b)) for b in bits], dtype=np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_float_to_half_rounds_to_nearest_even():
    L = c.lib()
    r = np.random.default_rng(5)
    bits = r.integers(0, 1 << 32, 40000, dtype=np.uint64).astype(np.uint32)
    # plus the halfway cases, subnormals, overflow edge and specials
    extra = np.array([65504.0, 65520.0, 65519.996, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26,
                      2.0 ** -14, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11, np.inf, -np.inf, 0.0,
                      -0.0], dtype=np.float32)
    xs = np.concatenate([bits.view(np.float32), extra])
    xs = xs[~np.isnan(xs)]
    with np.errstate(over="ignore"):
        want = xs.astype(np.float16).view(np.uint16)
    got = np.array([L.nb_float_to_half(float(x)) for x in xs], dtype=np.uint16)
    assert np.array_equal(got, want)
    assert np.isnan(np.uint16(L.nb_float_to_half(float("nan"))).view(np.float16))


def test_bf16_conversions_match_torch():
    L = c.lib()
    r = np.random.default_rng(6)
    xs = r.integers(0, 1 << 32, 40000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    xs = xs[~np.isnan(xs)]
    want = torch.from_numpy(xs.copy()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = np.array([L.nb_float_to_bf16(float(x)) for x in xs], dtype=np.uint16)
    assert np.array_equal(got, want)
    for b in (0x0000, 0x8000, 0x3f80, 0x7f7f, 0x0001, 0xff80):
        assert np.float32(L.nb_bf16_to_float(b)).view(np.uint32) == np.uint32(b << 16)
    assert np.isnan(L.nb_bf16_to_float(L.nb_float_to_bf16(float("nan"))))


def shares(sm, ce, mix, ce_frac, d2h, h2d, fold_gbs, algo, n):
    h, e = C.c_int(-1), C.c_int(-1)
    c.lib().nb_shares_from(sm, ce, mix, ce_frac, d2h, h2d, fold_gbs, c.ALGO[algo], n,
                           C.byref(h), C.byref(e))
    return h.value, e.value


def test_share_model():
    # A fast host path earns a host share, capped at a quarter.
    h, e = shares(700, 700, 700, 0, 55, 55, 400, "ar_twoshot", 2)
    assert 0 < h <= 2500 and e == 0
    # A slow host path earns nothing (predicted gain under 3 %).
    assert shares(700, 700, 700, 0, 5, 5, 20, "ar_twoshot", 8)[0] == 0
    # More ranks move more NVLink bytes per byte of share: larger host share for AG.
    assert shares(700, 700, 700, 0, 55, 55, 400, "ag_pull", 8)[0] <= 2500
    # Copy engines beside SM pulls pay when the mix beats SM-only by 3 %.
    assert shares(700, 770, 760, 0.4, 1, 1, 1, "ar_twoshot", 4)[1] == 4000
    assert shares(700, 770, 710, 0.4, 1, 1, 1, "ar_twoshot", 4)[1] == 0
    assert shares(700, 770, 760, 0.9, 1, 1, 1, "bc_scatter", 4)[1] == 5000
    # Reductions that the host cannot fold cheaply never see a CE share.
    assert shares(700, 770, 760, 0.4, 1, 1, 1, "rs_pull", 4)[1] == 0
    # No calibration, no shares.
    assert shares(0, 0, 0, 0, 0, 0, 0, "ar_twoshot", 4) == (0, 0)


def test_calibration_cache_roundtrip_and_key():
    back = C.c_double(0)
    rc = c.lib().nb_calib_roundtrip(712.125, b"GPU-abc,GPU-def|580.159|nccl22809", C.byref(back))
    assert rc == 1  # read back under its key, refused under another key
    assert abs(back.value - 712.125) < 1e-3


def test_size_aware_route_choice():
    L = c.lib()
    L.nb_calib_small.argtypes = [C.c_int, C.c_int, C.c_int, C.c_uint64, C.POINTER(C.c_int)]
    ce = C.c_int(-5)
    staged, twoshot = c.ALGO["ar_staged"], c.ALGO["ar_twoshot"]
    # Below the crossover the small-size winner, with its own shares...
    assert L.nb_calib_small(staged, twoshot, 512, 32 << 20, C.byref(ce)) == twoshot
    assert ce.value == 2222
    # ...at and above it the large-size winner.
    assert L.nb_calib_small(staged, twoshot, 512, 512 << 20, C.byref(ce)) == staged
    assert L.nb_calib_small(staged, twoshot, 512, 8 << 30, C.byref(ce)) == staged
    # No small-size tuning: always the large-size winner.
    assert L.nb_calib_small(staged, 0, 0, 32 << 20, C.byref(ce)) == staged


def u64s(*v):
    return (C.c_uint64 * len(v))(*v)


def ints(*v):
    return (C.c_int * len(v))(*v)


def test_clique_registry():
    L = c.lib()
    base = L.nb_clique_count()
    a = L.nb_clique_add(u64s(0x10, 0x20, 0x30), ints(0, 1, 2), 3)
    assert a >= 0 and L.nb_clique_count() == base + 1
    assert L.nb_clique_same(u64s(0x30, 0x10, 0x20), 3) == 1  # any order
    assert L.nb_clique_same(u64s(0x10, 0x20), 2) == 0        # a strict subset is no clique
    assert L.nb_clique_same(u64s(0x10, 0x10, 0x20), 3) == 0  # a repeated comm is no clique
    assert L.nb_clique_add(u64s(0x40, 0x50), ints(3, 3), 2) == -1  # two comms on one device
    assert L.nb_clique_add(u64s(0x40, 0x40), ints(3, 4), 2) == -1
    # Re-registering a member replaces its old clique.
    b = L.nb_clique_add(u64s(0x10, 0x60), ints(0, 5), 2)
    assert b > a and L.nb_clique_same(u64s(0x10, 0x60), 2) == 1
    assert L.nb_clique_same(u64s(0x20, 0x30, 0x10), 3) == 0
    L.nb_clique_forget(0x10)
    assert L.nb_clique_same(u64s(0x10, 0x60), 2) == 0


@pytest.mark.parametrize("ranks,nranks,ids,ok", [
    ([0, 1, 2, 3], [4] * 4, [7] * 4, 1),
    ([3, 1, 0, 2], [4] * 4, [7] * 4, 1),      # any issue order
    ([0, 1, 1, 3], [4] * 4, [7] * 4, 0),      # repeated rank
    ([0, 1, 2], [4] * 3, [7] * 3, 0),         # incomplete
    ([0, 1], [2, 3], [7, 7], 0),              # nranks disagree
    ([0, 1], [2, 2], [7, 8], 0),              # two different unique ids
    ([0], [1], [9], 1),                       # a one-rank communicator
])
def test_grouped_inits_form_clique(ranks, nranks, ids, ok):
    n = len(ranks)
    assert c.lib().nb_inits_form_clique(ints(*ranks), ints(*nranks), ints(*ids), n) == ok


def fault(spec, n=4, nbytes=1 << 30):
    at, first = C.c_uint64(0), C.c_uint64(0)
    rc = c.lib().nb_fault_policy(spec.encode(), n, nbytes, C.byref(at), C.byref(first))
    return rc, at.value, first.value


def test_fault_policy():
    assert fault("")[0] == 0
    assert fault("setup")[0] == 3
    rc, at, first = fault("op:0")
    assert rc == 1 and at == 0  # before any data op: nothing started, NCCL may take the call
    rc, at, first = fault(f"op:{first}")
    assert rc == 2 and at == first  # the first data op was attempted: the call fails
    rc, at, first = fault("op:999999")
    assert rc == 0  # past the end: never fires
    assert fault("bogus")[0] == -1
    assert fault("op:x")[0] == -1


def test_summary_format():
    buf = C.create_string_buffer(1 << 14)
    c.lib().nb_summary_sample(buf, 1 << 14)
    lines = buf.value.decode().splitlines()
    assert lines[0] == "build=test"
    assert "route=ar_twoshot custom_calls=1 logical_bytes=8589934592" in lines
    assert "route=ar_nvls custom_calls=0 logical_bytes=0" in lines
    assert "nranks=2 custom_calls=1" in lines
    assert "path sm_nvlink_bytes=100 ce_nvlink_bytes=10 host_bytes=1" in lines
    assert "device_timeouts=0" in lines
    assert "fallback_reason=FirstPass calls=1" in lines
    assert "fallback_reason=BelowThreshold calls=2" in lines
    assert "clique nranks=2 devices=0,1" in lines
    assert "staging_numa target=0 placed=0 method=mbind device=0 lane=1" in lines
    routes = [l for l in lines if l.startswith("route=")]
    reasons = [l for l in lines if l.startswith("fallback_reason=")]
    assert len(routes) == len(c.ALGO) - 1 and len(reasons) == len(c.REASONS) - 1
