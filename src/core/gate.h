// Pure eligibility decisions: per message, per call and per clique (the N
// calls of one collective, one per communicator of a clique).
//
// Parity: gate_message / gate_call / gate_pair of the reference
// (shim/nccl_collectives_shim.cu:178-269), generalized from a fixed device
// pair {0,1} to any clique of 1..8 distinct devices, and from sum-only fp
// reductions to every op and type the kernels implement. The rejection order
// of the reference is kept, so that the first failing check names the reason.
#pragma once

#include <vector>

#include "core/policy.h"
#include "core/types.h"

namespace nb {

// Pure message checks need no pointer queries (NCCL's nranks is known).
Reason gate_message(const CallDesc& c, const Policy& p);
// Full per-call eligibility; `device`, `rank` and `nranks` come from the
// communicator.
Reason gate_call(const CallDesc& c, const Policy& p);

// Process state the clique decision depends on, gathered by the interposer.
struct CliqueState {
  bool known_clique = false;   // the communicators were created together
  bool capturing = false;      // some stream is capturing (or unknown)
  bool first_pass_done = false;
  bool poisoned = false;
  bool nccl_supported = true;  // libnccl inside the supported version range
  bool nvls_available = false; // multicast objects usable on this clique
  // Per-kind algorithm the init-time calibration measured fastest on this
  // clique (Fallback = no preference).
  Algo preferred[size_t(Kind::Count)] = {Algo::Fallback, Algo::Fallback, Algo::Fallback,
                                         Algo::Fallback};
};

struct CliqueDecision {
  Algo algo;
  Reason reason;
};

// `calls` are the N buffered calls of one group in arrival order.
CliqueDecision gate_clique(const std::vector<CallDesc>& calls, const CliqueState& s,
                           const Policy& p);

// Algorithm choice for an eligible clique call.
Algo choose_algo(const CallDesc& c, int nranks, bool nvls_available, const Policy& p,
                 Algo preferred = Algo::Fallback);
bool algo_valid(Algo a, Kind k, int nranks, DType t, RedOp op, bool nvls_available);

// A gated clique as the planner sees it: no pointers, everything indexed by
// rank.
struct CliqueDesc {
  Kind kind = Kind::AllReduce;
  DType dtype = DType::Unsupported;
  RedOp op = RedOp::Sum;
  int nranks = 0;
  size_t bytes = 0;      // call_bytes (per-rank payload / slot)
  size_t count = 0;
  int root = -1;         // Broadcast only (a rank)
  bool in_place[kMaxRanks] = {};
  double scalar = 1.0;   // PreMulSum: the scalar every rank shares (NVLS routes)
};
CliqueDesc describe_clique(const std::vector<CallDesc>& calls);

}  // namespace nb
