"""Numerics of the sm_100a kernels on one GPU, against a plain torch fp32
reference of the same op (fold in rank order in fp32, then cast)."""
import pytest
import torch

from conftest import need_gpus

pytestmark = pytest.mark.gpu

FLOATS = [torch.float32, torch.float16, torch.bfloat16, torch.float64]
INTS = [torch.int32, torch.int8, torch.uint8, torch.int64]


def exact_data(n, count, dtype, seed, lim=None):
    g = torch.Generator(device="cuda:0").manual_seed(seed)
    if dtype.is_floating_point:
        lim = lim or {torch.float32: 1 << 20, torch.float64: 1 << 40, torch.float16: 255,
                      torch.bfloat16: 15}[dtype]
        return [torch.randint(-lim, lim + 1, (count,), device="cuda:0", generator=g).to(dtype)
                for _ in range(n)]
    info = torch.iinfo(dtype)
    return [torch.randint(info.min, info.max, (count,), device="cuda:0", generator=g, dtype=torch.int64).to(dtype)
            for _ in range(n)]


def ref_fold(srcs, op, scalars=None):
    dt = srcs[0].dtype
    acc_t = torch.float64 if dt == torch.float64 else (torch.float32 if dt.is_floating_point else torch.int64)
    xs = [s.to(acc_t) for s in srcs]
    if op == "premulsum":
        acc = xs[0] * scalars[0]
        for i, x in enumerate(xs[1:], 1):
            acc = torch.addcmul(acc, x, torch.full_like(x, scalars[i]))  # a + x*s (one rounding each)
        return acc.to(dt)
    acc = xs[0].clone()
    for x in xs[1:]:
        if op in ("sum", "avg"):
            acc = acc + x
        elif op == "prod":
            acc = acc * x
        elif op == "max":
            acc = torch.maximum(acc, x)
        elif op == "min":
            acc = torch.minimum(acc, x)
    if not dt.is_floating_point:
        # Integer sums wrap in the element type.
        acc = acc.to(dt)
        if op == "avg":
            acc = torch.div(acc.to(torch.int64), len(srcs), rounding_mode="trunc").to(dt)
        return acc
    if op == "avg":
        acc = acc / len(srcs)
    return acc.to(dt)


@pytest.mark.parametrize("dtype", FLOATS)
@pytest.mark.parametrize("nsrc", [1, 2, 3, 4, 8])
def test_reduce_sum_exact(dtype, nsrc):
    need_gpus(1)
    from scc26_nccl_shim_b200.ops import emu
    count = (1 << 20) + 7  # a tail that fills no 16-byte vector
    srcs = exact_data(nsrc, count, dtype, seed=nsrc)
    dsts = [torch.empty_like(srcs[0]) for _ in range(2)]
    emu.reduce(srcs, dsts, "sum")
    torch.cuda.synchronize()
    ref = ref_fold(srcs, "sum")
    for d in dsts:
        assert torch.equal(d, ref)


@pytest.mark.parametrize("op", ["prod", "max", "min", "avg"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_reduce_ops(op, dtype):
    need_gpus(1)
    from scc26_nccl_shim_b200.ops import emu
    count = 65536 + 3
    if op == "prod":
        srcs = exact_data(4, count, dtype, seed=7, lim=3)
    else:
        g = torch.Generator(device="cuda:0").manual_seed(3)
        srcs = [torch.randn(count, device="cuda:0", generator=g).to(dtype) for _ in range(4)]
    out = torch.empty_like(srcs[0])
    emu.reduce(srcs, [out], op)
    torch.cuda.synchronize()
    ref = ref_fold(srcs, op)
    if op == "avg":
        torch.testing.assert_close(out.float(), ref.float(), rtol=1e-6, atol=1e-6) if dtype == torch.float32 \
            else torch.testing.assert_close(out.float(), ref.float(), rtol=1e-2, atol=1e-2)
    else:
        assert torch.equal(out, ref)


def test_reduce_premulsum():
    need_gpus(1)
    from scc26_nccl_shim_b200.ops import emu
    g = torch.Generator(device="cuda:0").manual_seed(5)
    srcs = [torch.randn(100003, device="cuda:0", generator=g) for _ in range(3)]
    scalars = [0.5, -1.25, 3.0]
    out = torch.empty_like(srcs[0])
    emu.reduce(srcs, [out], "premulsum", scalars=scalars)
    torch.cuda.synchronize()
    ref = ref_fold(srcs, "premulsum", scalars)
    torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("dtype", INTS)
@pytest.mark.parametrize("op", ["sum", "max", "min", "prod"])
def test_reduce_ints(dtype, op):
    need_gpus(1)
    from scc26_nccl_shim_b200.ops import emu
    srcs = exact_data(3, 4099, dtype, seed=11)
    out = torch.empty_like(srcs[0])
    emu.reduce(srcs, [out], op)
    torch.cuda.synchronize()
    if op in ("sum", "prod") and dtype in (torch.int64,):
        # torch int64 arithmetic wraps the same way.
        ref = srcs[0].clone()
        for s in srcs[1:]:
            ref = ref + s if op == "sum" else ref * s
    else:
        ref = ref_fold(srcs, op)
    assert torch.equal(out, ref)


def test_copy_segments_alignment():
    need_gpus(1)
    from scc26_nccl_shim_b200.ops import emu
    base = torch.randint(0, 255, (5 << 20,), dtype=torch.uint8, device="cuda:0")
    out = torch.zeros_like(base)
    # aligned, misaligned-but-co-aligned, and fully misaligned segments
    segs = [(0, 0, (1 << 20) + 5), (1 << 21, (1 << 21) + 16, 70001), (3 << 20, (3 << 20) + 3, 99999),
            ((4 << 20) + 1, (4 << 20) + 7, 12345)]
    emu.copy([base[s:] for s, _, _ in segs], [out[d:] for _, d, _ in segs], [n for _, _, n in segs])
    torch.cuda.synchronize()
    for s, d, n in segs:
        assert torch.equal(out[d:d + n], base[s:s + n])


@pytest.mark.parametrize("nbytes,src_off,dst_off", [
    (4 << 20, 0, 0),                       # the smallest bulk copy
    ((64 << 20) + 5, 0, 256),              # a byte tail after the last 16-byte unit
    ((100 << 20) + 16, 16, 48),            # 16-byte aligned, not 32
    ((8 << 20) + 3, 1, 7),                 # misaligned: the SM copy loop instead
])
def test_single_local_copy(nbytes, src_off, dst_off):
    """One large copy within a GPU (the TMA bulk copy when both ends are
    16-byte aligned) against torch's copy, with guard bytes around it."""
    need_gpus(1)
    from scc26_nccl_shim_b200.ops import emu
    g = torch.Generator(device="cuda:0").manual_seed(nbytes % 1000)
    base = torch.randint(0, 256, (nbytes + src_off + 64,), dtype=torch.uint8, device="cuda:0",
                         generator=g)
    out = torch.full((nbytes + dst_off + 64,), 0xA5, dtype=torch.uint8, device="cuda:0")
    emu.copy([base[src_off:]], [out[dst_off:]], [nbytes])
    torch.cuda.synchronize()
    assert torch.equal(out[dst_off:dst_off + nbytes], base[src_off:src_off + nbytes])
    assert bool((out[:dst_off] == 0xA5).all()) and bool((out[dst_off + nbytes:] == 0xA5).all())


CASES = [("ar_twoshot", "allreduce"), ("rs_pull", "reducescatter"), ("ag_pull", "allgather"),
         ("bc_pull", "broadcast"), ("bc_scatter", "broadcast"), ("ar_staged", "allreduce"),
         ("rs_staged", "reducescatter"), ("bc_chain", "broadcast"), ("ag_push", "allgather")]


@pytest.mark.parametrize("algo,kind", CASES)
@pytest.mark.parametrize("n", [2, 3, 4, 8])
@pytest.mark.parametrize("inplace", [False, True])
def test_virtual_rank_plans(algo, kind, n, inplace):
    # (The gang engines -- NVLS, push chain, push-reduce, one-shot -- wait for
    # their counterparts on other GPUs inside the kernel; the virtual-rank
    # runner refuses them. Their GPU tests run on real cliques.)
    need_gpus(1)
    if algo == "bc_scatter" and n < 3:
        pytest.skip("scatter broadcast needs 3+ ranks")
    from scc26_nccl_shim_b200.ops import emu
    count = (1 << 18) + (0 if kind == "reducescatter" else 5)
    dt = torch.float32
    if kind == "reducescatter":
        sends = exact_data(n, count * n, dt, seed=n)
        recvs = [s[r * count:(r + 1) * count] if inplace else torch.empty(count, device="cuda:0")
                 for r, s in enumerate(sends)]
    elif kind == "allgather":
        recvs = [torch.empty(count * n, device="cuda:0") for _ in range(n)]
        data = exact_data(n, count, dt, seed=n)
        if inplace:
            sends = [recvs[r][r * count:(r + 1) * count] for r in range(n)]
            for r in range(n):
                sends[r].copy_(data[r])
        else:
            sends = data
    else:
        sends = exact_data(n, count, dt, seed=n)
        recvs = sends if inplace else [torch.empty(count, device="cuda:0") for _ in range(n)]
    inputs = [s.clone() for s in sends]
    root = n - 1
    ce = 3000 if algo in ("ar_twoshot", "ag_pull", "bc_pull") else \
        (10000 if algo in ("bc_scatter", "bc_chain") else 0)
    emu.plan(algo, kind, sends, recvs, root=root, ce_ppm=ce)
    torch.cuda.synchronize()
    for r in range(n):
        if kind == "allreduce":
            ref = ref_fold(inputs, "sum")
        elif kind == "reducescatter":
            ref = ref_fold([x[r * count:(r + 1) * count] for x in inputs], "sum")
        elif kind == "allgather":
            ref = torch.cat(inputs)
        else:
            ref = inputs[root]
        assert torch.equal(recvs[r], ref), (algo, n, r)
