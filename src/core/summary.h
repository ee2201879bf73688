// Exit summary (NCCL_SHIM_SUMMARY=1): per-algorithm custom calls and logical
// bytes, per-path bytes (SM-driven NVLink, copy-engine NVLink, pinned host),
// calls per fallback reason, cliques seen, host-buffer NUMA placement,
// calibration results and device-timeout counts. Counters are relaxed
// atomics; lines are prefixed "[nccl-shim-summary]".
//
// Parity: SubmissionSummary / staging_summary / count_fallback /
// count_custom of the reference (shim/nccl_collectives_shim.cu:1222-1265),
// which report routes, fallback reasons and the source hash.
#pragma once

#include <atomic>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "core/types.h"

namespace nb {

class Summary {
 public:
  void set_enabled(bool e) { enabled_ = e; }
  bool enabled() const { return enabled_; }
  void count_fallback(Reason r);
  void count_custom(Algo a, size_t logical_bytes, int nranks, size_t sm, size_t ce, size_t host);
  void count_timeout();
  void note_clique(int nranks, const int* devices);
  void note_placement(int dev, int lane, int target, int placed, const char* method);
  void note(const std::string& line);
  // All summary lines (without the prefix), in a fixed order.
  std::vector<std::string> render(const char* build_id) const;
  uint64_t fallbacks(Reason r) const { return fallbacks_[size_t(r)].load(std::memory_order_relaxed); }
  uint64_t custom_calls(Algo a) const { return calls_[size_t(a)].load(std::memory_order_relaxed); }

 private:
  bool enabled_ = false;
  std::atomic<uint64_t> calls_[size_t(Algo::Count)]{};
  std::atomic<uint64_t> bytes_[size_t(Algo::Count)]{};
  std::atomic<uint64_t> ranks_hist_[kMaxRanks + 1]{};
  std::atomic<uint64_t> sm_bytes_{0}, ce_bytes_{0}, host_bytes_{0}, timeouts_{0};
  std::atomic<uint64_t> fallbacks_[size_t(Reason::Count)]{};
  mutable std::mutex mu_;
  std::vector<std::string> notes_;
};

}  // namespace nb
