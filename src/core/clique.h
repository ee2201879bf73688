// Communicator cliques: the N communicators one process created together
// (one ncclCommInitAll over N distinct devices, or N grouped
// ncclCommInitRank* calls sharing one ncclUniqueId). Only the members of one
// clique may run a collective together: equal counts and devices alone
// cannot tell independent communicators apart. Any lifecycle call on a
// member (destroy, finalize, abort, split, shrink, register, ...) forgets the
// whole clique before it is forwarded.
//
// Also holds the PreMulSum registry: the scalar each communicator attached
// to each ncclRedOpCreatePreMulSum handle, so the kernels can apply it.
//
// Parity: g_known_peers / forget_pair / same_pair / note_initialization /
// register_initializations of the reference (shim/nccl_collectives_shim.cu:
// 1429-1505), which track pairs of two communicators on devices {0,1} only.
#pragma once

#include <cstdint>
#include <map>
#include <mutex>
#include <vector>

#include "core/group.h"
#include "core/types.h"

namespace nb {

struct CliqueInfo {
  int id = -1;
  int nranks = 0;
  void* comms[kMaxRanks] = {};
  int devices[kMaxRanks] = {};
};

struct PreMulScalar {
  DType dtype = DType::F32;
  int residence = 1;  // 1 host immediate, 0 device pointer
  double value = 1.0;
  uintptr_t device_ptr = 0;
};

class CliqueRegistry {
 public:
  // comms[i] is rank i on devices[i]. Replaces any clique a member was in.
  int add(void* const* comms, const int* devices, int nranks);
  void forget(void* comm);
  bool lookup(void* comm, CliqueInfo* out) const;
  // True when `comms` are exactly the members of one clique (any order).
  bool same_clique(const std::vector<void*>& comms, CliqueInfo* out) const;
  size_t size() const;

  void add_premul(void* comm, int op, const PreMulScalar& s);
  void drop_premul(void* comm, int op);
  bool find_premul(void* comm, int op, PreMulScalar* out) const;

 private:
  void forget_locked(void* comm);
  mutable std::mutex mu_;
  int next_id_ = 0;
  std::map<int, CliqueInfo> cliques_;
  std::map<void*, int> member_;
  std::map<std::pair<void*, int>, PreMulScalar> premul_;
};

// Pure validation of grouped ncclCommInitRank* calls: all share one id and
// one nranks, ranks are distinct and cover 0..N-1, outputs are distinct.
bool inits_form_clique(const std::vector<PendingInit>& inits);

}  // namespace nb
