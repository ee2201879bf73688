#include "core/fault.h"

#include <cstdlib>

namespace nb {

bool FaultInjector::configure(const std::string& spec) {
  kind_ = Kind::None;
  always_ = false;
  fired_ = false;
  if (spec.empty()) return true;
  std::string s = spec;
  const std::string suffix = ":always";
  if (s.size() > suffix.size() && s.compare(s.size() - suffix.size(), suffix.size(), suffix) == 0) {
    always_ = true;
    s.resize(s.size() - suffix.size());
  }
  if (s == "setup") {
    kind_ = Kind::Setup;
    return true;
  }
  if (s.rfind("op:", 0) == 0 && s.size() > 3) {
    char* end = nullptr;
    const unsigned long long k = std::strtoull(s.c_str() + 3, &end, 10);
    if (*end) return false;
    kind_ = Kind::Op;
    index_ = size_t(k);
    return true;
  }
  return false;
}

bool FaultInjector::fail_setup() {
  if (kind_ != Kind::Setup || (!always_ && fired_.load())) return false;
  fired_ = true;
  return true;
}

bool FaultInjector::fail_op(size_t index) {
  if (kind_ != Kind::Op || index != index_ || (!always_ && fired_.load())) return false;
  fired_ = true;
  return true;
}

void FaultInjector::end_call() {}

}  // namespace nb
