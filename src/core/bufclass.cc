#include "core/bufclass.h"

namespace nb {

namespace {

struct Span {
  const PointerFacts& first;
  const PointerFacts& last;
  uint64_t addr, bytes;
  int device;
};

bool both(const Span& s, bool (*pred)(const PointerFacts&)) { return pred(s.first) && pred(s.last); }

// Each rule must hold, in this order; the first one that fails names the refusal.
struct Rule {
  const char* name;
  bool (*holds)(const Span&);
};

const Rule kRules[] = {
    {"non-empty", [](const Span& s) { return s.bytes > 0 && s.bytes - 1 <= ~uint64_t(0) - s.addr; }},
    {"known-to-driver", [](const Span& s) { return both(s, [](const PointerFacts& f) { return f.known; }); }},
    {"device-memory",
     [](const Span& s) { return both(s, [](const PointerFacts& f) { return f.device_memory; }); }},
    {"on-expected-device", [](const Span& s) { return s.first.device == s.device && s.last.device == s.device; }},
    {"one-allocation",
     [](const Span& s) {
       const PointerFacts& f = s.first;
       return f.range_size > 0 && s.addr >= f.range_start && s.addr - f.range_start < f.range_size &&
              s.bytes <= f.range_size - (s.addr - f.range_start) && s.last.range_start == f.range_start &&
              s.last.range_size == f.range_size;
     }},
    // VMM memory: a reserved range may join pieces mapped with different
    // access; both ends must lie in one mapping. (cudaMalloc memory is one
    // allocation whatever its physical backing.)
    {"one-mapping",
     [](const Span& s) {
       if (s.first.legacy_ipc != 0 && s.last.legacy_ipc != 0) return true;
       return s.first.mapping_start == s.last.mapping_start && s.first.mapping_size == s.last.mapping_size;
     }},
    {"not-pool-memory",
     [](const Span& s) { return both(s, [](const PointerFacts& f) { return !f.from_pool; }); }},
    {"same-devices-queried", [](const Span& s) { return s.first.ndev == s.last.ndev && s.first.ndev > 0; }},
    {"access-queries-answered",
     [](const Span& s) {
       for (int i = 0; i < s.first.ndev; ++i)
         if (s.first.access[i] == Access::QueryFailed || s.last.access[i] == Access::QueryFailed) return false;
       return true;
     }},
};

bool all_access(const PointerFacts& f, bool (*ok)(Access)) {
  for (int i = 0; i < f.ndev; ++i)
    if (!ok(f.access[i])) return false;
  return true;
}

bool mapped_kind(const PointerFacts& f) {
  return f.legacy_ipc == 0 && all_access(f, [](Access a) { return a == Access::ReadWrite; });
}

bool ordinary_kind(const PointerFacts& f) {
  return f.legacy_ipc == 1 && all_access(f, [](Access a) {
           return a == Access::NoMapping || a == Access::NoFlags || a == Access::ReadWrite;
         });
}

}  // namespace

BufferVerdict classify_buffer(const PointerFacts& first, const PointerFacts& last, uint64_t addr,
                              uint64_t bytes, int expected_device) {
  const Span s{first, last, addr, bytes, expected_device};
  for (const Rule& r : kRules)
    if (!r.holds(s)) return {BufferClass::Refused, r.name};
  if (mapped_kind(first) && mapped_kind(last)) return {BufferClass::Mapped, "mapped-read-write-everywhere"};
  if (ordinary_kind(first) && ordinary_kind(last)) return {BufferClass::Ordinary, "ordinary-peer-memory"};
  return {BufferClass::Refused, "neither-ordinary-nor-mapped"};
}

}  // namespace nb
