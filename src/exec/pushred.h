// Push-reduce engine (pushred.cu): ReduceScatter and two-shot AllReduce
// whose NVLink traffic is stores only, synchronized by in-kernel progress
// words.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "core/plan.h"
#include "core/policy.h"
#include "exec/executor.h"

namespace nb {

// Whether the engine has kernels for this element type and rank count.
bool pushred_supported(DType t, int n);
// Scratch and progress words on every clique device.
bool pushred_ensure(const int* devices, int n, std::string* why);
// Submit one rank's share (op.stream.dev) on stream s.
cudaError_t pushred_launch(const PlanOp& op, const Plan& plan, const Binding& b, const Policy& p,
                           cudaStream_t s);
// Nonzero once a bounded wait expired.
unsigned pushred_status(const int* devices, int n);
// With NCCL_B200_NVLS_TRACE=1: mean per-block ns since the last reset of rank
// `rank`'s kernels, {sender waiting, sender total, reducer waiting, reducer
// total}; returns the blocks that ran, -1 on error.
int pushred_trace_read(const int* devices, int n, int rank, double out[4], bool reset);

}  // namespace nb
