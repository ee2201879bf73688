// NVLS (NVLink SHARP) support: multicast objects over the clique's GPUs and
// the multimem AllReduce gang kernel.
//
// User cudaMalloc buffers cannot be bound to a multicast object, so every
// GPU owns a multicast-bound scratch region (physical memory from
// cuMemCreate, bound into one multicast object that spans every clique
// device). The gang kernel copies its input into its own scratch, reduces its
// slice through the switch with multimem.ld_reduce, multicasts the result
// with multimem.st and copies its output out, in rounds, with bounded
// in-kernel barriers (multimem.red on a multicast flag word per block) between
// the phases. No TMA multicast is used anywhere.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "core/plan.h"
#include "exec/executor.h"

namespace nb {

// True when every device supports multicast objects and the driver entry
// points exist. Cheap after the first call per device set.
bool nvls_supported(const int* devices, int n);
// Create the multicast scratch for this device set: `nbuf` round buffers
// (at least 3) of `round_bytes` each, fixed at creation.
bool nvls_ensure(const int* devices, int n, size_t round_bytes, int nbuf, std::string* why);
cudaError_t nvls_launch(const PlanOp& op, const Plan& plan, const Binding& b, const Policy& p,
                        cudaStream_t s, int dev);
// Device-side status of the last NVLS gang on this device set: 0 ok,
// nonzero = a bounded wait expired. Reading it synchronizes nothing.
unsigned nvls_status(const int* devices, int n);
// The multicast scratch of this device set, once created: bytes bound per
// GPU, round buffers and round size. False when there is none.
bool nvls_scratch(const int* devices, int n, size_t* bytes, unsigned* buffers, size_t* round);
// Phase timing of one rank's NVLS kernels since the last reset (policy
// nvls_trace): out = mean over blocks of {mover busy, mover waiting, copier
// busy, copier waiting, mover total, copier total} in ns. Synchronizes that
// device. Returns the block count, or -1 without an NVLS context.
int nvls_trace_read(const int* devices, int n, int rank, double out[6], bool reset);

}  // namespace nb
