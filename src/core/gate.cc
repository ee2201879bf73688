#include "core/gate.h"

#include <cstdint>

namespace nb {

static bool op_supported(RedOp op, DType t) {
  switch (op) {
    case RedOp::Sum: case RedOp::Prod: case RedOp::Max: case RedOp::Min: case RedOp::Avg:
      return reducible(t);
    case RedOp::PreMulSum:
      return is_float(t);
    default:
      return false;
  }
}

Reason gate_message(const CallDesc& c, const Policy& p) {
  const size_t elem = elem_size(c.dtype);
  if (elem == 0) return Reason::UnsupportedType;
  const bool red = reduces(c.kind);
  if (red && !reducible(c.dtype)) return Reason::UnsupportedType;
  if (red && !op_supported(c.op, c.dtype)) return Reason::UnsupportedOp;
  const size_t n = c.nranks > 0 ? size_t(c.nranks) : 1;
  if (c.count > (SIZE_MAX / 4) / elem / n) return Reason::SizeOverflow;
  const size_t logical = logical_bytes(c);
  if (logical > p.max_message_bytes) return Reason::AboveLimit;
  if (!p.enabled) return Reason::Disabled;
  if (!p.kind_enabled[size_t(c.kind)]) return Reason::PolicyFallback;
  if (logical < p.min_bytes[size_t(c.kind)] || c.count == 0) return Reason::BelowThreshold;
  // Slot offsets feed 16-byte reduction vectors.
  if (c.kind == Kind::ReduceScatter && call_bytes(c) % 16 != 0) return Reason::BadSlot;
  return Reason::None;
}

Reason gate_call(const CallDesc& c, const Policy& p) {
  const Reason message = gate_message(c, p);
  if (message != Reason::None) return message;
  const bool bcast_nonroot = c.kind == Kind::Broadcast && c.rank != c.root;
  if (!c.recv || (!c.send && !bcast_nonroot)) return Reason::NullBuffer;
  if (c.nranks < 1 || c.nranks > kMaxRanks || c.rank < 0 || c.rank >= c.nranks || c.device < 0)
    return Reason::BadRank;
  if (c.kind == Kind::Broadcast && (c.root < 0 || c.root >= c.nranks)) return Reason::BadRank;
  // Represented ranges before any in-place arithmetic; a Broadcast
  // non-root's send pointer is never read.
  if (c.recv > UINTPTR_MAX - recv_extent(c) ||
      (!bcast_nonroot && c.send > UINTPTR_MAX - send_extent(c)))
    return Reason::AddressOverflow;
  // The reduction kernels issue 16-byte vector loads and stores.
  if (reduces(c.kind) && (c.send % 16 != 0 || c.recv % 16 != 0)) return Reason::Misaligned;
  if (bcast_nonroot) return Reason::None;
  if (!call_in_place(c) && ranges_overlap(c.send, send_extent(c), c.recv, recv_extent(c)))
    return Reason::PartialOverlap;
  return Reason::None;
}

bool algo_valid(Algo a, Kind k, int nranks, DType t, RedOp op, bool nvls_available) {
  switch (a) {
    case Algo::ArTwoShot: return k == Kind::AllReduce;
    case Algo::ArHybrid:
    case Algo::RsHybrid:
      // The hybrid routes (an NVLS gang on part of the SMs beside a P2P
      // kernel) returned wrong data at 4 GiB on 2, 4 and 8 GPUs and were
      // slower than NVLS alone where correct: refused, so forcing them takes
      // the static choice.
      return false;
    case Algo::ArNvls:
      // A multicast object needs at least two devices.
      return k == Kind::AllReduce && nvls_available && nranks >= 2 &&
             (t == DType::F32 || t == DType::F16 || t == DType::BF16) &&
             (op == RedOp::Sum || op == RedOp::Avg || op == RedOp::PreMulSum);
    case Algo::ArOneShot:
    case Algo::ArTwoShotLL:
      return k == Kind::AllReduce && nranks >= 2 && (t == DType::F32 || t == DType::F16 || t == DType::BF16);
    case Algo::RsLL:
      return k == Kind::ReduceScatter && nranks >= 2 && (t == DType::F32 || t == DType::F16 || t == DType::BF16);
    case Algo::AgLL: return k == Kind::AllGather && nranks >= 2;
    case Algo::BcLL: return k == Kind::Broadcast && nranks >= 2;
    case Algo::RsPull: return k == Kind::ReduceScatter;
    case Algo::AgPull: return k == Kind::AllGather;
    case Algo::BcPull: return k == Kind::Broadcast;
    case Algo::BcScatter: return k == Kind::Broadcast && nranks >= 3;
    case Algo::ArStaged: return k == Kind::AllReduce;
    case Algo::RsStaged: return k == Kind::ReduceScatter;
    case Algo::BcChain: return k == Kind::Broadcast;
    case Algo::BcNvls: return k == Kind::Broadcast && nvls_available && nranks >= 2;
    case Algo::AgNvls: return k == Kind::AllGather && nvls_available && nranks >= 2;
    case Algo::AgPush: return k == Kind::AllGather;
    case Algo::BcRing: return k == Kind::Broadcast && nranks >= 2;
    case Algo::RsPush:
    case Algo::ArPush:
      return k == (a == Algo::RsPush ? Kind::ReduceScatter : Kind::AllReduce) && nranks >= 2 &&
             (t == DType::F32 || t == DType::F16 || t == DType::BF16);
    case Algo::RsNvls:
      return k == Kind::ReduceScatter && nvls_available && nranks >= 2 &&
             (t == DType::F32 || t == DType::F16 || t == DType::BF16) &&
             (op == RedOp::Sum || op == RedOp::Avg || op == RedOp::PreMulSum);
    default: return false;
  }
}

Algo choose_algo(const CallDesc& c, int nranks, bool nvls_available, const Policy& p,
                 Algo preferred) {
  const Algo forced = p.force_algo[size_t(c.kind)];
  if (forced != Algo::Fallback && algo_valid(forced, c.kind, nranks, c.dtype, c.op, nvls_available))
    return forced;
  if (preferred != Algo::Fallback &&
      algo_valid(preferred, c.kind, nranks, c.dtype, c.op, nvls_available))
    return preferred;
  switch (c.kind) {
    case Kind::AllReduce: {
      const bool nvls = p.nvls != NvlsMode::Off &&
                        (p.nvls == NvlsMode::On || nranks >= p.nvls_min_ranks) &&
                        algo_valid(Algo::ArNvls, c.kind, nranks, c.dtype, c.op, nvls_available);
      return nvls ? Algo::ArNvls : Algo::ArTwoShot;
    }
    case Kind::ReduceScatter: return Algo::RsPull;
    case Kind::AllGather: return Algo::AgPull;
    case Kind::Broadcast: return nranks >= 3 ? Algo::BcScatter : Algo::BcPull;
    default: return Algo::Fallback;
  }
}

CliqueDecision gate_clique(const std::vector<CallDesc>& calls, const CliqueState& s,
                           const Policy& p) {
  const auto fallback = [](Reason r) { return CliqueDecision{Algo::Fallback, r}; };
  if (s.poisoned) return fallback(Reason::Poisoned);
  if (!s.nccl_supported) return fallback(Reason::UnsupportedNccl);
  if (calls.empty()) return fallback(Reason::GroupShape);
  const CallDesc& a = calls[0];
  const int n = a.nranks;
  if (n < 1 || n > kMaxRanks || int(calls.size()) != n || !s.known_clique)
    return fallback(Reason::NotClique);
  // Ranks and devices must each be distinct and cover 0..N-1 / N devices.
  unsigned rank_mask = 0;
  for (const CallDesc& c : calls) {
    if (c.rank < 0 || c.rank >= n || (rank_mask >> c.rank) & 1u) return fallback(Reason::NotClique);
    rank_mask |= 1u << c.rank;
    for (const CallDesc& d : calls)
      if (&d != &c && d.device == c.device) return fallback(Reason::NotClique);
  }
  for (const CallDesc& c : calls) {
    if (c.kind != a.kind || c.count != a.count || c.dtype != a.dtype || c.op != a.op ||
        c.nranks != n)
      return fallback(Reason::Mismatch);
    if (a.kind == Kind::Broadcast && (c.root != a.root || a.root < 0 || a.root >= n))
      return fallback(Reason::Mismatch);
  }
  for (const CallDesc& c : calls) {
    const Reason r = gate_call(c, p);
    if (r != Reason::None) return fallback(r);
  }
  if (s.capturing) return fallback(Reason::Capturing);
  if (p.first_pass && !s.first_pass_done) return fallback(Reason::FirstPass);
  Algo algo = choose_algo(a, n, s.nvls_available, p, s.preferred[size_t(a.kind)]);
  // The multimem kernels move whole 16-byte vectors only: every buffer and
  // every slot must be 16-byte aligned. They scale the switch's sum once, so
  // a PreMulSum takes them only when every rank passed the same host scalar.
  // The low-latency AllGather/Broadcast copies also move whole vectors.
  const bool nvls = algo == Algo::ArNvls || algo == Algo::BcNvls || algo == Algo::AgNvls ||
                    algo == Algo::RsNvls || algo == Algo::ArHybrid || algo == Algo::RsHybrid;
  const bool vec_copy = algo == Algo::AgLL || algo == Algo::BcLL;
  bool aligned = call_bytes(a) % 16 == 0;
  for (const CallDesc& c : calls)
    aligned = aligned && c.recv % 16 == 0 && (c.send % 16 == 0 || (c.kind == Kind::Broadcast && c.rank != c.root));
  bool uniform = true;
  if (a.op == RedOp::PreMulSum)
    for (const CallDesc& c : calls)
      uniform = uniform && c.scalar_residence == 1 && a.scalar_residence == 1 && c.scalar == a.scalar;
  if ((nvls && (!aligned || !uniform)) || (vec_copy && !aligned)) {
    const Policy q = [&] {
      Policy x = p;
      x.nvls = NvlsMode::Off;
      x.force_algo[size_t(a.kind)] = Algo::Fallback;
      return x;
    }();
    algo = choose_algo(a, n, false, q);
  }
  if (algo == Algo::Fallback) return fallback(Reason::PolicyFallback);
  return {algo, Reason::None};
}

CliqueDesc describe_clique(const std::vector<CallDesc>& calls) {
  CliqueDesc d;
  if (calls.empty()) return d;
  const CallDesc& a = calls[0];
  d.kind = a.kind;
  d.dtype = a.dtype;
  d.op = a.op;
  d.nranks = int(calls.size());
  d.bytes = call_bytes(a);
  d.count = a.count;
  d.root = a.kind == Kind::Broadcast ? a.root : -1;
  d.scalar = a.op == RedOp::PreMulSum ? a.scalar : 1.0;
  for (const CallDesc& c : calls)
    if (c.rank >= 0 && c.rank < kMaxRanks) d.in_place[c.rank] = call_in_place(c);
  return d;
}

}  // namespace nb
