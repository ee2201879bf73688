#include "core/clique.h"

#include <cstring>

namespace nb {

int CliqueRegistry::add(void* const* comms, const int* devices, int nranks) {
  std::lock_guard<std::mutex> lk(mu_);
  if (nranks < 1 || nranks > kMaxRanks) return -1;
  for (int i = 0; i < nranks; ++i) {
    if (!comms[i]) return -1;
    for (int j = 0; j < i; ++j)
      if (comms[j] == comms[i] || devices[j] == devices[i]) return -1;
  }
  for (int i = 0; i < nranks; ++i) forget_locked(comms[i]);
  CliqueInfo c;
  c.id = next_id_++;
  c.nranks = nranks;
  for (int i = 0; i < nranks; ++i) {
    c.comms[i] = comms[i];
    c.devices[i] = devices[i];
    member_[comms[i]] = c.id;
  }
  cliques_[c.id] = c;
  return c.id;
}

void CliqueRegistry::forget_locked(void* comm) {
  const auto it = member_.find(comm);
  if (it == member_.end()) return;
  const auto c = cliques_.find(it->second);
  if (c != cliques_.end()) {
    for (int i = 0; i < c->second.nranks; ++i) member_.erase(c->second.comms[i]);
    cliques_.erase(c);
  } else {
    member_.erase(it);
  }
}

void CliqueRegistry::forget(void* comm) {
  std::lock_guard<std::mutex> lk(mu_);
  forget_locked(comm);
  for (auto it = premul_.begin(); it != premul_.end();)
    it = it->first.first == comm ? premul_.erase(it) : std::next(it);
}

bool CliqueRegistry::lookup(void* comm, CliqueInfo* out) const {
  std::lock_guard<std::mutex> lk(mu_);
  const auto it = member_.find(comm);
  if (it == member_.end()) return false;
  const auto c = cliques_.find(it->second);
  if (c == cliques_.end()) return false;
  if (out) *out = c->second;
  return true;
}

bool CliqueRegistry::same_clique(const std::vector<void*>& comms, CliqueInfo* out) const {
  std::lock_guard<std::mutex> lk(mu_);
  if (comms.empty()) return false;
  const auto it = member_.find(comms[0]);
  if (it == member_.end()) return false;
  const auto c = cliques_.find(it->second);
  if (c == cliques_.end() || c->second.nranks != int(comms.size())) return false;
  unsigned seen = 0;
  for (void* comm : comms) {
    int idx = -1;
    for (int i = 0; i < c->second.nranks; ++i)
      if (c->second.comms[i] == comm) idx = i;
    if (idx < 0 || (seen >> idx) & 1u) return false;
    seen |= 1u << idx;
  }
  if (out) *out = c->second;
  return true;
}

size_t CliqueRegistry::size() const {
  std::lock_guard<std::mutex> lk(mu_);
  return cliques_.size();
}

void CliqueRegistry::add_premul(void* comm, int op, const PreMulScalar& s) {
  std::lock_guard<std::mutex> lk(mu_);
  premul_[{comm, op}] = s;
}

void CliqueRegistry::drop_premul(void* comm, int op) {
  std::lock_guard<std::mutex> lk(mu_);
  premul_.erase({comm, op});
}

bool CliqueRegistry::find_premul(void* comm, int op, PreMulScalar* out) const {
  std::lock_guard<std::mutex> lk(mu_);
  const auto it = premul_.find({comm, op});
  if (it == premul_.end()) return false;
  if (out) *out = it->second;
  return true;
}

bool inits_form_clique(const std::vector<PendingInit>& inits) {
  if (inits.empty() || inits.size() > size_t(kMaxRanks)) return false;
  const int n = inits[0].nranks;
  if (n != int(inits.size())) return false;
  unsigned ranks = 0;
  for (size_t i = 0; i < inits.size(); ++i) {
    const PendingInit& p = inits[i];
    if (p.nranks != n || p.rank < 0 || p.rank >= n || (ranks >> p.rank) & 1u || !p.output)
      return false;
    ranks |= 1u << p.rank;
    if (std::memcmp(p.id, inits[0].id, sizeof(p.id)) != 0) return false;
    for (size_t j = 0; j < i; ++j)
      if (inits[j].output == p.output) return false;
  }
  return true;
}

}  // namespace nb
