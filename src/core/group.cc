#include "core/group.h"

namespace nb {

int GroupMachine::replay(GroupState& g, Reason reason) {
  int first_error = nccl::Success;
  for (const Call& c : g.pending) {
    const int r = b_.forward(c, reason);
    if (first_error == nccl::Success && r != nccl::Success) first_error = r;
  }
  g.pending.clear();
  return first_error;
}

int GroupMachine::enqueue(GroupState& g, Call c) {
  if (g.depth > 0) g.init_only = false;
  if (g.depth == 0) {
    // A one-rank clique needs no grouping: run it at once.
    if (b_.query(c) && c.desc.nranks == 1 && gate_call(c.desc, b_.policy()) == Reason::None) {
      std::vector<Call> one{c};
      Reason reason = Reason::NotGrouped;
      const Outcome o = b_.run(one, reason);
      if (o == Outcome::Handled) return nccl::Success;
      if (o == Outcome::Error) return nccl::UnhandledCudaError;
      return b_.forward(c, reason);
    }
    return b_.forward(c, Reason::NotGrouped);
  }
  if (g.passthrough) return b_.forward(c, g.passthrough_reason);
  const bool same_kind = g.pending.empty() || g.pending[0].desc.kind == c.desc.kind;
  const size_t limit = g.pending.empty() ? size_t(kMaxRanks) : size_t(g.pending[0].desc.nranks);
  Reason reason = Reason::GroupShape;
  if (g.pending.size() < limit && same_kind) {
    reason = Reason::MetadataQuery;
    if (b_.query(c)) {
      reason = Reason::GroupShape;
      if (size_t(c.desc.nranks) > g.pending.size() &&
          (g.pending.empty() || c.desc.nranks == g.pending[0].desc.nranks))
        reason = gate_call(c.desc, b_.policy());
    }
    if (reason == Reason::None) {
      g.pending.push_back(c);
      return nccl::Success;  // deferred, as NCCL defers grouped calls
    }
  }
  // Flush the buffered prefix in order, then go sticky for this outer group;
  // the first error wins.
  const int replay_result = replay(g, reason);
  g.passthrough = true;
  g.passthrough_reason = reason;
  return replay_result != nccl::Success ? replay_result : b_.forward(c, reason);
}

int GroupMachine::group_start(GroupState& g) {
  int replay_result = nccl::Success;
  if (g.depth > 0) {  // nested: the outer group stays on NCCL
    g.init_only = false;
    replay_result = replay(g, Reason::GroupShape);
    g.passthrough = true;
    g.passthrough_reason = Reason::GroupShape;
  } else {
    g.pending.clear();
    g.inits.clear();
    g.init_only = true;
    g.passthrough = false;
    g.passthrough_reason = Reason::GroupShape;
  }
  const int r = b_.real_group_start();
  if (r == nccl::Success) ++g.depth;
  return replay_result != nccl::Success ? replay_result : r;
}

int GroupMachine::group_end(GroupState& g) {
  if (g.depth > 1) {
    --g.depth;
    return b_.real_group_end();
  }
  if (g.depth == 0) return b_.real_group_end();
  g.depth = 0;
  Outcome outcome = Outcome::Fallback;
  Reason reason = Reason::GroupShape;
  if (!g.passthrough && !g.pending.empty() &&
      g.pending.size() == size_t(g.pending[0].desc.nranks))
    outcome = b_.run(g.pending, reason);
  g.passthrough = false;
  // Never replay over partially written buffers; otherwise replay inside the
  // real group GroupStart opened.
  int result = nccl::Success;
  if (outcome == Outcome::Error) result = nccl::UnhandledCudaError;
  else if (outcome == Outcome::Fallback) result = replay(g, reason);
  g.pending.clear();
  const int end = b_.real_group_end();
  return result != nccl::Success ? result : end;
}

int GroupMachine::force_passthrough(GroupState& g, bool initialization) {
  if (g.depth == 0) return nccl::Success;
  if (!initialization) g.init_only = false;
  g.passthrough = true;
  g.passthrough_reason = Reason::GroupShape;
  return replay(g, Reason::GroupShape);
}

int GroupMachine::simulate_end(GroupState& g, void* info) {
  const int prefix = force_passthrough(g);
  if (g.depth > 0) --g.depth;
  if (g.depth == 0) g.passthrough = false;
  const int result = b_.real_simulate_end(info);
  g.inits.clear();
  return prefix != nccl::Success ? prefix : result;
}

}  // namespace nb
