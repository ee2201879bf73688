#include "core/summary.h"

#include <cstdio>

namespace nb {

void Summary::count_fallback(Reason r) {
  fallbacks_[size_t(r)].fetch_add(1, std::memory_order_relaxed);
}

void Summary::count_custom(Algo a, size_t logical, int nranks, size_t sm, size_t ce, size_t host) {
  calls_[size_t(a)].fetch_add(1, std::memory_order_relaxed);
  bytes_[size_t(a)].fetch_add(logical, std::memory_order_relaxed);
  if (nranks >= 0 && nranks <= kMaxRanks) ranks_hist_[nranks].fetch_add(1, std::memory_order_relaxed);
  sm_bytes_.fetch_add(sm, std::memory_order_relaxed);
  ce_bytes_.fetch_add(ce, std::memory_order_relaxed);
  host_bytes_.fetch_add(host, std::memory_order_relaxed);
}

void Summary::count_timeout() { timeouts_.fetch_add(1, std::memory_order_relaxed); }

void Summary::note_clique(int nranks, const int* devices) {
  if (!enabled_) return;
  std::string s = "clique nranks=" + std::to_string(nranks) + " devices=";
  for (int i = 0; i < nranks; ++i) s += (i ? "," : "") + std::to_string(devices[i]);
  note(s);
}

void Summary::note_placement(int dev, int lane, int target, int placed, const char* method) {
  if (!enabled_) return;
  char buf[160];
  std::snprintf(buf, sizeof buf, "staging_numa target=%d placed=%d method=%s device=%d lane=%d",
                target, placed, method, dev, lane);
  note(buf);
}

void Summary::note(const std::string& line) {
  if (!enabled_) return;
  std::lock_guard<std::mutex> lk(mu_);
  notes_.push_back(line);
}

std::vector<std::string> Summary::render(const char* build_id) const {
  std::vector<std::string> out;
  char buf[256];
  std::snprintf(buf, sizeof buf, "build=%s", build_id ? build_id : "unknown");
  out.push_back(buf);
  for (size_t a = 1; a < size_t(Algo::Count); ++a) {
    std::snprintf(buf, sizeof buf, "route=%s custom_calls=%llu logical_bytes=%llu",
                  algo_name(Algo(a)), (unsigned long long)calls_[a].load(std::memory_order_relaxed),
                  (unsigned long long)bytes_[a].load(std::memory_order_relaxed));
    out.push_back(buf);
  }
  for (int n = 1; n <= kMaxRanks; ++n) {
    const uint64_t c = ranks_hist_[n].load(std::memory_order_relaxed);
    if (!c) continue;
    std::snprintf(buf, sizeof buf, "nranks=%d custom_calls=%llu", n, (unsigned long long)c);
    out.push_back(buf);
  }
  std::snprintf(buf, sizeof buf, "path sm_nvlink_bytes=%llu ce_nvlink_bytes=%llu host_bytes=%llu",
                (unsigned long long)sm_bytes_.load(std::memory_order_relaxed),
                (unsigned long long)ce_bytes_.load(std::memory_order_relaxed),
                (unsigned long long)host_bytes_.load(std::memory_order_relaxed));
  out.push_back(buf);
  std::snprintf(buf, sizeof buf, "device_timeouts=%llu",
                (unsigned long long)timeouts_.load(std::memory_order_relaxed));
  out.push_back(buf);
  for (size_t r = 1; r < size_t(Reason::Count); ++r) {
    std::snprintf(buf, sizeof buf, "fallback_reason=%s calls=%llu", reason_name(Reason(r)),
                  (unsigned long long)fallbacks_[r].load(std::memory_order_relaxed));
    out.push_back(buf);
  }
  std::lock_guard<std::mutex> lk(mu_);
  for (const std::string& s : notes_) out.push_back(s);
  return out;
}

}  // namespace nb
