// Flag-synchronized push chain for Broadcast over peer memory (ring.cu).
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "core/plan.h"
#include "core/policy.h"
#include "exec/executor.h"

namespace nb {

// Per-device progress words and the status word for the clique's devices.
bool ring_ensure(const int* devices, int n, std::string* why);
// Submit one rank's share (op.stream.dev) of a chain Broadcast on stream s.
cudaError_t ring_launch(const PlanOp& op, const Plan& plan, const Binding& b, const Policy& p,
                        cudaStream_t s);
// Nonzero once a bounded wait expired.
unsigned ring_status(const int* devices, int n);
// With NCCL_B200_NVLS_TRACE=1: mean per-block ns since the last reset of rank
// `rank`'s kernel, {waiting for the predecessor, total}; returns the blocks
// that ran (0 for the last rank of the chain, which runs no kernel).
int ring_trace_read(const int* devices, int n, int rank, double out[2], bool reset);

}  // namespace nb
