"""Seeded test data for collectives.

`exact(...)`: a 64-bit hash of (rank, index, iteration, seed) mapped to a
signed integer small enough that every partial sum of N ranks is exactly
representable in the element type, so any reduction order (including the
NVSwitch's) gives the same bits and outputs can be compared bit for bit.
Neighbouring elements and iterations differ, so data displaced by any chunk
boundary is caught.

`adversarial(...)`: full-range bit patterns for differential runs against
stock NCCL: finite values of every exponent, subnormals, signed zeros,
infinities, the largest binade (sums overflow) and near-negations across
ranks (catastrophic cancellation); NaNs only for copy collectives.
"""
from __future__ import annotations

import torch

MASK64 = (1 << 64) - 1


def _mix64(z: torch.Tensor) -> torch.Tensor:
    # splitmix64 on int64 tensors (arithmetic wraps modulo 2^64).
    z = z + (0x9E3779B97F4A7C15 - (1 << 64))
    z = (z ^ (z >> 30) & 0x3FFFFFFFF) * (0xBF58476D1CE4E5B9 - (1 << 64))
    z = (z ^ (z >> 27) & 0x1FFFFFFFFF) * (0x94D049BB133111EB - (1 << 64))
    return z ^ (z >> 31) & 0x1FFFFFFFF


def exact_limit(dtype: torch.dtype, nranks: int) -> int:
    """Largest |v| whose N-rank partial sums are exact in `dtype`."""
    mant = {torch.float32: 24, torch.float16: 11, torch.bfloat16: 8, torch.float64: 53}
    if dtype in mant:
        return max(1, ((1 << mant[dtype]) - 1) // max(1, nranks))
    info = torch.iinfo(dtype)
    return max(1, info.max // max(1, nranks))


def exact(rank: int, count: int, iteration: int, seed: int, dtype: torch.dtype, nranks: int,
          device, offset: int = 0) -> torch.Tensor:
    idx = torch.arange(offset, offset + count, device=device, dtype=torch.int64)
    key = idx ^ ((iteration * 16 + rank) << 44)
    h = _mix64(key ^ seed)
    lim = exact_limit(dtype, nranks)
    v = torch.remainder(h, 2 * lim + 1) - lim
    return v.to(dtype)


def adversarial(rank: int, count: int, seed: int, dtype: torch.dtype, device, nans: bool) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed * 131 + rank)
    if dtype == torch.float32:
        bits = torch.randint(-(1 << 31), (1 << 31) - 1, (count,), device=device, generator=g,
                             dtype=torch.int64).to(torch.int32)
        x = bits.view(torch.float32).clone()
    else:
        bits = torch.randint(-(1 << 15), (1 << 15) - 1, (count,), device=device, generator=g,
                             dtype=torch.int64).to(torch.int16)
        x = bits.view(dtype).clone()
    specials = torch.tensor([0.0, -0.0, float("inf"), float("-inf")], device=device, dtype=dtype)
    if count >= 4:
        x[:4] = specials
    if rank % 2 == 1 and count >= 64:
        # near-negations of rank 0's pattern: catastrophic cancellation
        other = adversarial(0, count, seed, dtype, device, nans)
        x[8:64] = -other[8:64]
    if not nans:
        x = torch.where(torch.isnan(x), torch.zeros_like(x), x)
    return x
