// Host-side reduction: the fold the pinned-host lane applies to its share,
// and the oracle the CPU simulator and the tests use. The fold order is the
// rank order 0..N-1, accumulating in fp32 for 16-bit floats (fp64 for
// doubles, the type's own width with wrap-around for integers), so that the
// GPU kernels (which use the same order and the same per-element operations)
// agree bit for bit.
//
// Parity: the reference reduces only fp32/fp16/bf16 sums, on the GPU, two
// inputs at a time with half-precision adds for 16-bit types
// (shim/nccl_collectives_shim.cu:772-802); it has no host reduction.
#pragma once

#include <cstddef>
#include <cstdint>

#include "core/types.h"

namespace nb {

// IEEE binary16 / bfloat16 <-> binary32, round to nearest even.
float half_to_float(uint16_t h);
uint16_t float_to_half(float f);
float bf16_to_float(uint16_t b);
uint16_t float_to_bf16(float f);

// Reduction parameters shared by the kernels and the host fold.
struct FoldParams {
  DType dtype = DType::F32;
  RedOp op = RedOp::Sum;
  int nranks = 1;                 // Avg divides by this
  double scalars[kMaxRanks] = {1, 1, 1, 1, 1, 1, 1, 1};  // PreMulSum per source
};

// dst[0..bytes) := fold(srcs[0..nsrc)[0..bytes)). `bytes` is a multiple of
// the element size. dst may alias srcs[0].
void host_fold(const FoldParams& p, const void* const* srcs, int nsrc, void* dst, size_t bytes);

// The same fold split over `threads` CPU threads (contiguous element ranges).
void host_fold_parallel(const FoldParams& p, const void* const* srcs, int nsrc, void* dst,
                        size_t bytes, int threads);

}  // namespace nb
