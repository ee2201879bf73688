// Low-latency one-shot AllReduce with in-kernel barriers over peer memory
// (oneshot.cu).
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "core/plan.h"
#include "core/policy.h"
#include "exec/executor.h"

namespace nb {

// The element types and clique sizes the kernels are built for.
bool oneshot_supported(DType t, int n);
// Arrive/depart tables, the per-device events and the status word.
bool oneshot_ensure(const int* devices, int n, std::string* why);
// Submit one rank's kernel (op.stream.dev) on stream s.
cudaError_t oneshot_launch(const PlanOp& op, const Plan& plan, const Binding& b, const Policy& p,
                           cudaStream_t s);
// Nonzero once a bounded wait expired.
unsigned oneshot_status(const int* devices, int n);

}  // namespace nb
