// The group machine as the transition system of tla/GroupFallbackN.tla.
//
// The model has two actions over (seen, forwarded, pending, passthrough):
//   Receive(op)  a call arrives inside the outer group. It is appended to
//                `pending` when the group is still buffering and the call
//                extends a clique set; otherwise the model's Flush happens:
//                forwarded' = forwarded ++ pending ++ <<op>>, pending' = <<>>,
//                passthrough' = TRUE.
//   End          the outer group closes. A complete clique set with no
//                passthrough runs on the clique runner; anything else is
//                forwarded in arrival order.
// Each action is split here into a decision (decide_receive, decide_end:
// what the model does, given the backend's answers about the call) and its
// effects on libnccl (apply_flush, the runner), so the code reads as the
// spec's transition relation. Around it sit the parts the model abstracts
// away: nested groups (depth), the real library's GroupStart/GroupEnd, which
// run exactly once per interposed call, and ungrouped one-rank cliques.
#include "core/group.h"

namespace nb {

namespace {

// Of a sequence of libnccl results, the first failure is the one reported.
class FirstFailure {
 public:
  void see(int r) {
    if (code_ == nccl::Success) code_ = r;
  }
  int code() const { return code_; }
  bool failed() const { return code_ != nccl::Success; }

 private:
  int code_ = nccl::Success;
};

}  // namespace

// Receive(op) for a collective while buffering: the reason the call cannot
// join the pending clique set, or Reason::None when it can.
Reason GroupMachine::decide_receive(const GroupState& g, Call& c) {
  const Call* head = g.pending.empty() ? nullptr : &g.pending.front();
  if (head && head->desc.kind != c.desc.kind) return Reason::GroupShape;  // one kind per set
  const size_t room = head ? size_t(head->desc.nranks) : size_t(kMaxRanks);
  if (g.pending.size() >= room) return Reason::GroupShape;  // the set is already full
  if (!b_.query(c)) return Reason::MetadataQuery;
  const bool extends = size_t(c.desc.nranks) > g.pending.size() &&
                       (!head || c.desc.nranks == head->desc.nranks);
  if (!extends) return Reason::GroupShape;
  return gate_call(c.desc, b_.policy(c.desc.nranks));
}

// The effects of the model's Flush: pending calls, then `arriving` (when
// given), go to libnccl in order; the group turns passthrough. When
// forwarding the pending prefix fails, that error is returned and the
// arriving call is not issued.
int GroupMachine::apply_flush(GroupState& g, Reason why, const Call* arriving) {
  FirstFailure f;
  for (const Call& p : g.pending) f.see(b_.forward(p, why));
  g.pending.clear();
  g.passthrough = true;
  g.passthrough_reason = why;
  if (arriving && !f.failed()) f.see(b_.forward(*arriving, why));
  return f.code();
}

// Forward what is pending without changing the passthrough state (End's
// fallback branch).
int GroupMachine::forward_pending(GroupState& g, Reason why) {
  FirstFailure f;
  for (const Call& p : g.pending) f.see(b_.forward(p, why));
  g.pending.clear();
  return f.code();
}

// End: does the pending set run on the clique runner?
bool GroupMachine::decide_end(const GroupState& g) const {
  return !g.passthrough && !g.pending.empty() &&
         g.pending.size() == size_t(g.pending.front().desc.nranks);
}

// Outside any group there is nothing to buffer: a one-rank clique that
// passes the call gate runs at once, everything else goes to libnccl.
int GroupMachine::ungrouped(Call& c) {
  if (!b_.query(c) || c.desc.nranks != 1 || gate_call(c.desc, b_.policy(1)) != Reason::None)
    return b_.forward(c, Reason::NotGrouped);
  std::vector<Call> single{c};
  Reason why = Reason::NotGrouped;
  switch (b_.run(single, why)) {
    case Outcome::Handled: return nccl::Success;
    case Outcome::Error: return nccl::UnhandledCudaError;
    default: return b_.forward(c, why);
  }
}

int GroupMachine::enqueue(GroupState& g, Call c) {
  if (g.depth == 0) return ungrouped(c);
  g.init_only = false;
  if (g.passthrough) return b_.forward(c, g.passthrough_reason);
  const Reason why = decide_receive(g, c);
  if (why == Reason::None) {
    // Buffered; NCCL itself defers grouped work until the group ends.
    g.pending.push_back(c);
    return nccl::Success;
  }
  return apply_flush(g, why, &c);
}

// An operation the interposer never handles (or a lifecycle call) is the
// model's unsupported op: Receive(unsupported) always flushes.
int GroupMachine::force_passthrough(GroupState& g, bool initialization) {
  if (g.depth == 0) return nccl::Success;
  if (!initialization) g.init_only = false;
  return apply_flush(g, Reason::GroupShape, nullptr);
}

int GroupMachine::group_start(GroupState& g) {
  FirstFailure f;
  if (g.depth == 0) {
    g = GroupState{};  // a fresh outer group: the model's Init
  } else {
    // A nested group is outside the model's single-level grouping: the outer
    // group stays on libnccl from here.
    g.init_only = false;
    f.see(apply_flush(g, Reason::GroupShape, nullptr));
  }
  const int started = b_.real_group_start();
  if (started == nccl::Success) ++g.depth;
  f.see(started);
  return f.code();
}

int GroupMachine::group_end(GroupState& g) {
  if (g.depth != 1) {  // an inner group closes (or none is open)
    if (g.depth > 1) --g.depth;
    return b_.real_group_end();
  }
  g.depth = 0;
  FirstFailure f;
  Reason why = Reason::GroupShape;
  const Outcome o = decide_end(g) ? b_.run(g.pending, why) : Outcome::Fallback;
  g.passthrough = false;
  if (o == Outcome::Error) {
    // Data may already have moved: never replay over half-written buffers.
    f.see(nccl::UnhandledCudaError);
  } else if (o == Outcome::Fallback) {
    // Replayed inside the real group that GroupStart opened.
    f.see(forward_pending(g, why));
  }
  g.pending.clear();
  f.see(b_.real_group_end());
  return f.code();
}

int GroupMachine::simulate_end(GroupState& g, void* info) {
  FirstFailure f;
  f.see(force_passthrough(g));
  if (g.depth > 0) --g.depth;
  if (g.depth == 0) g.passthrough = false;
  f.see(b_.real_simulate_end(info));
  g.inits.clear();
  return f.code();
}

}  // namespace nb
