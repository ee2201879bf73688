// NCCL group buffering state machine, generalized to cliques of N ranks,
// written as the transition system of tla/GroupFallbackN.tla (Receive, End).
//
// Inside an outer ncclGroupStart/End, up to N eligible calls of one kind are
// buffered (NCCL itself defers grouped calls, so returning success without
// touching the GPU is legal). At the outer GroupEnd an exact clique set (N
// calls) is handed to the clique runner; anything else is forwarded, in
// arrival order, into the real group that GroupStart already opened. The
// first call that cannot be buffered (wrong kind, failed gate, one call too
// many, an unsupported operation, a nested group) flushes the buffered prefix
// in order and makes the rest of the outer group sticky-passthrough. The real
// GroupStart/GroupEnd are each called exactly once per interposed call.
//
// Invariants (checked by the models and tests): forwarded calls are always a
// prefix of the calls seen, in order; at most N calls are pending; before the
// end, forwarded ++ pending == seen; at the end, either the clique ran
// (exactly one complete clique set and nothing else) or everything was
// forwarded.
//
// Parity: GroupState / shim_enqueue / replay_pending / ncclGroupStart /
// group_end_impl / force_passthrough / ncclGroupSimulateEnd of the reference
// (shim/nccl_collectives_shim.cu:1346-1427, 1451-1459, 1774-1794, 1943-1953)
// for two ranks, and the TLA+ model tla/GroupFallback.tla.
#pragma once

#include <cstdint>
#include <vector>

#include "core/gate.h"
#include "core/policy.h"
#include "core/types.h"

namespace nb {

struct Call {
  CallDesc desc;
  const void* sendbuff = nullptr;
  void* recvbuff = nullptr;
  int nccl_dtype = 0;
  int nccl_op = 0;
  void* comm = nullptr;
  void* stream = nullptr;
};

// A grouped ncclCommInitRank* call, registered as a clique at the outer end.
struct PendingInit {
  void** output = nullptr;
  uint8_t id[128] = {};
  int rank = -1;
  int nranks = -1;
};

struct GroupState {
  int depth = 0;
  bool passthrough = false;
  Reason passthrough_reason = Reason::GroupShape;
  bool init_only = true;
  std::vector<Call> pending;
  std::vector<PendingInit> inits;
};

enum class Outcome { Handled, Fallback, Error };

// What the state machine needs from the outside world: libnccl (real group
// calls, forwarding, communicator queries) and the clique runner.
class GroupBackend {
 public:
  virtual ~GroupBackend() = default;
  virtual int real_group_start() = 0;
  virtual int real_group_end() = 0;
  virtual int real_simulate_end(void* info) = 0;
  // Forward one call to libnccl and count the fallback reason.
  virtual int forward(const Call& c, Reason reason) = 0;
  // Fill desc.device / rank / nranks from the communicator.
  virtual bool query(Call& c) = 0;
  // The routing policy in force for cliques of `nranks` (thresholds may be
  // the measured crossover with NCCL for that size).
  virtual const Policy& policy(int nranks) = 0;
  // Gate, plan and execute a complete clique set.
  virtual Outcome run(std::vector<Call>& calls, Reason& reason) = 0;
};

class GroupMachine {
 public:
  explicit GroupMachine(GroupBackend& b) : b_(b) {}
  int enqueue(GroupState& g, Call c);
  int group_start(GroupState& g);
  int group_end(GroupState& g);
  int simulate_end(GroupState& g, void* info);
  // An unsupported operation arrives: flush the prefix, go sticky.
  int force_passthrough(GroupState& g, bool initialization = false);

 private:
  Reason decide_receive(const GroupState& g, Call& c);
  bool decide_end(const GroupState& g) const;
  int apply_flush(GroupState& g, Reason why, const Call* arriving);
  int forward_pending(GroupState& g, Reason why);
  int ungrouped(Call& c);
  GroupBackend& b_;
};

}  // namespace nb
