// Host-visible interface of the sm_100a collective kernels.
//
// Every kernel reads and writes the caller's buffers directly, on this GPU
// and on peer GPUs (single-process UVA with peer access enabled), so the
// reduction, scaling and cast are fused with the NVLink transfer: one pass,
// no staging copy, no separate elementwise kernel.
//
// Parity: the reference's only kernels are a two-input elementwise add over a
// scratch buffer that a copy engine filled first, plus a scalar tail kernel
// (shim/nccl_collectives_shim.cu:772-851).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "core/hostreduce.h"
#include "core/types.h"

namespace nb {

struct ReduceLaunch {
  const void* src[kMaxRanks] = {};
  void* dst[kMaxRanks] = {};
  int nsrc = 0, ndst = 0;
  size_t bytes = 0;  // multiple of the element size
  FoldParams fold;
  // PreMulSum scalars that live in device memory (residence 0), per source;
  // null entries use fold.scalars.
  const void* dev_scalar[kMaxRanks] = {};
};

struct CopyLaunch {
  const void* src[kMaxRanks] = {};
  void* dst[kMaxRanks] = {};
  size_t len[kMaxRanks] = {};
  int nseg = 0;
  bool local = false;  // every buffer is in the launching GPU's own device memory
  bool prefer_tma = false;  // a large local copy runs on the TMA bulk engine
};

struct LaunchShape {
  int blocks = 0;
  int threads = 512;
};

// Launch on `stream` (the current device must be the stream's device).
// Returns the launch's own error (cudaLaunchKernel, not a stale one).
cudaError_t launch_reduce(const ReduceLaunch& a, LaunchShape shape, cudaStream_t stream);
cudaError_t launch_copy(const CopyLaunch& a, LaunchShape shape, cudaStream_t stream);

// Nonzero once a bounded wait of the TMA bulk copy expired (that copy is
// incomplete); the runner then stops using its own routes.
unsigned tma_copy_status();
// Allocates the status word (once); false when pinned host memory is unavailable.
bool tma_copy_prepare();

// Grid for `bytes` of work on a device with `sm_count` SMs.
LaunchShape shape_for(size_t bytes, int sm_count, int blocks_per_sm, int threads);

}  // namespace nb
