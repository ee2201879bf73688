// CPU execution and verification of plans.
//
// check_plan builds the happens-before graph of a plan exactly as CUDA
// orders its ops (stream order; a Wait orders after the most recent Record
// of its event submitted before it; the NVLS gang ops of one plan start
// together) and reports (a) any two data ops that touch overlapping bytes,
// at least one writing, with no happens-before path between them, and (b)
// any data op that does not happen before the end of every caller stream
// (a rank could return while a peer still touches its buffers).
//
// simulate_plan runs the data ops on host memory in a random topological
// order, using the host fold for every reduction.
//
// Parity: the reference relies on TLA+ (tla/*.tla) plus GPU stress runs; its
// planner layers are written to be CPU-testable (shim.cu:15-16) but no CPU
// test of them ships.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "core/hostreduce.h"
#include "core/plan.h"

namespace nb {

// Where each rank's send and receive buffers live inside that rank's memory
// arena (in-place layouts alias).
struct SimLayout {
  int nranks = 0;
  size_t arena_bytes[kMaxRanks] = {};
  size_t send_off[kMaxRanks] = {};
  size_t recv_off[kMaxRanks] = {};
  bool send_valid[kMaxRanks] = {};  // false for a Broadcast non-root's send
};

// Layout of a clique call with NCCL's in-place conventions.
SimLayout layout_for(const CliqueDesc& d);

// "" when the plan is race-free and fully joined; otherwise a description.
std::string check_plan(const Plan& plan, const SimLayout& layout);

// Executes the plan on `arenas` (one per rank, sized per layout).
std::string simulate_plan(const Plan& plan, const SimLayout& layout, const FoldParams& fp,
                          std::vector<std::vector<uint8_t>>& arenas, uint64_t seed);

}  // namespace nb
