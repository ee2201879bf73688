#include "core/plan_sim.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <random>
#include <tuple>

namespace nb {

SimLayout layout_for(const CliqueDesc& d) {
  SimLayout l;
  l.nranks = d.nranks;
  const size_t n = d.bytes;
  const size_t N = size_t(d.nranks);
  for (int r = 0; r < d.nranks; ++r) {
    size_t send_ext = n, recv_ext = n;
    if (d.kind == Kind::AllGather) recv_ext = N * n;
    if (d.kind == Kind::ReduceScatter) send_ext = N * n;
    l.send_valid[r] = !(d.kind == Kind::Broadcast && r != d.root);
    if (d.in_place[r]) {
      // NCCL in-place layouts: AG send = recv + r*n; RS recv = send + r*n.
      if (d.kind == Kind::AllGather) {
        l.recv_off[r] = 0;
        l.send_off[r] = size_t(r) * n;
        l.arena_bytes[r] = recv_ext;
      } else if (d.kind == Kind::ReduceScatter) {
        l.send_off[r] = 0;
        l.recv_off[r] = size_t(r) * n;
        l.arena_bytes[r] = send_ext;
      } else {
        l.send_off[r] = l.recv_off[r] = 0;
        l.arena_bytes[r] = n;
      }
    } else {
      l.send_off[r] = 0;
      l.recv_off[r] = (send_ext + 255) & ~size_t(255);
      l.arena_bytes[r] = l.recv_off[r] + recv_ext;
    }
  }
  return l;
}

namespace {

struct Access {
  int arena;
  size_t lo, hi;
  bool write;
};

struct StreamKey {
  uint8_t kind, dev, lane;
  bool operator<(const StreamKey& o) const {
    return std::tie(kind, dev, lane) < std::tie(o.kind, o.dev, o.lane);
  }
};
struct EventKey {
  uint8_t kind, dev, lane;
  uint16_t index;
  bool operator<(const EventKey& o) const {
    return std::tie(kind, dev, lane, index) < std::tie(o.kind, o.dev, o.lane, o.index);
  }
};

StreamKey skey(StreamId s) { return {uint8_t(s.kind), s.dev, s.lane}; }
EventKey ekey(EventId e) { return {uint8_t(e.kind), e.dev, e.lane, e.index}; }

bool is_data(OpKind k) {
  return k == OpKind::CeCopy || k == OpKind::SmCopy || k == OpKind::SmReduce ||
         k == OpKind::HostReduce || k == OpKind::NvlsReduce;
}

// Nodes: the plan's ops [0, m), the NVLS gang node m, then per rank r a
// virtual "producer" m+1+r (the caller's work before the call on its stream:
// it wrote rank r's buffers) and "consumer" m+1+N+r (the caller's work after
// the call: it reads and overwrites them). Races against these make missing
// InputReady and Join waits visible.
struct Graph {
  int nodes = 0;
  int gang = -1;
  int producer0 = 0, consumer0 = 0;
  std::vector<std::vector<int>> preds;
  std::vector<int> caller_end;  // per rank: last node on its caller stream
  std::string error;
};

Graph build_graph(const Plan& plan) {
  Graph g;
  const int m = int(plan.ops.size());
  const int n = plan.desc.nranks;
  bool has_gang = false;
  for (const PlanOp& op : plan.ops) has_gang |= op.kind == OpKind::NvlsReduce;
  g.gang = has_gang ? m : -1;
  g.producer0 = m + 1;
  g.consumer0 = m + 1 + n;
  g.nodes = m + 1 + 2 * n;
  g.preds.assign(size_t(g.nodes), {});
  std::map<StreamKey, int> last;
  std::map<EventKey, int> last_record;
  for (int r = 0; r < n; ++r) last[StreamKey{uint8_t(Strm::Caller), uint8_t(r), 0}] = g.producer0 + r;
  for (int i = 0; i < m; ++i) {
    const PlanOp& op = plan.ops[size_t(i)];
    const auto it = last.find(skey(op.stream));
    const int prev = it == last.end() ? -1 : it->second;
    if (op.kind == OpKind::NvlsReduce) {
      if (prev >= 0) g.preds[size_t(g.gang)].push_back(prev);
      g.preds[size_t(i)].push_back(g.gang);
    } else if (prev >= 0) {
      g.preds[size_t(i)].push_back(prev);
    }
    if (op.kind == OpKind::Wait) {
      const auto r = last_record.find(ekey(op.event));
      if (r != last_record.end()) g.preds[size_t(i)].push_back(r->second);
    }
    if (op.kind == OpKind::Record) last_record[ekey(op.event)] = i;
    last[skey(op.stream)] = i;
  }
  g.caller_end.assign(size_t(n), -1);
  for (int r = 0; r < n; ++r) {
    const auto it = last.find(StreamKey{uint8_t(Strm::Caller), uint8_t(r), 0});
    if (it != last.end()) g.caller_end[size_t(r)] = it->second;
    g.preds[size_t(g.consumer0 + r)].push_back(g.caller_end[size_t(r)]);
  }
  return g;
}

// Kahn's algorithm; a random pick among ready nodes when rng is given.
bool topo_order(const Graph& g, std::vector<int>& order, std::mt19937_64* rng) {
  std::vector<std::vector<int>> succ(size_t(g.nodes));
  std::vector<int> indeg(size_t(g.nodes), 0);
  for (int v = 0; v < g.nodes; ++v)
    for (int u : g.preds[size_t(v)]) {
      succ[size_t(u)].push_back(v);
      ++indeg[size_t(v)];
    }
  std::vector<int> ready;
  for (int v = 0; v < g.nodes; ++v)
    if (!indeg[size_t(v)]) ready.push_back(v);
  order.clear();
  while (!ready.empty()) {
    size_t pick = 0;
    if (rng) pick = size_t((*rng)() % ready.size());
    const int v = ready[pick];
    ready[pick] = ready.back();
    ready.pop_back();
    order.push_back(v);
    for (int w : succ[size_t(v)])
      if (--indeg[size_t(w)] == 0) ready.push_back(w);
  }
  return int(order.size()) == g.nodes;
}

int arena_of(const Loc& l, int nranks) {
  switch (l.buf) {
    case Buf::Send: case Buf::Recv: return l.dev;
    case Buf::Bounce: return nranks + int(l.dev) * kMaxLanes + l.lane;
    case Buf::HostOut: return nranks + kMaxRanks * kMaxLanes + l.lane;
    case Buf::Temp: return nranks + kMaxRanks * kMaxLanes + kMaxLanes + l.dev;
    default: return -1;
  }
}
constexpr int kTempArena0 = kMaxRanks * kMaxLanes + kMaxLanes;  // relative to nranks
size_t offset_of(const Loc& l, const SimLayout& lay) {
  switch (l.buf) {
    case Buf::Send: return lay.send_off[l.dev] + l.off;
    case Buf::Recv: return lay.recv_off[l.dev] + l.off;
    default: return l.off;
  }
}

void accesses_of(const PlanOp& op, const SimLayout& lay, const CliqueDesc& d,
                 std::vector<Access>& out) {
  const int n = lay.nranks;
  auto add = [&](const Loc& l, size_t bytes, bool write) {
    const size_t o = offset_of(l, lay);
    out.push_back({arena_of(l, n), o, o + bytes, write});
  };
  switch (op.kind) {
    case OpKind::CeCopy:
      add(op.src[0], op.bytes, false);
      add(op.dst[0], op.bytes, true);
      break;
    case OpKind::SmCopy:
      for (int i = 0; i < op.nsrc; ++i) {
        add(op.src[i], op.len[i], false);
        add(op.dst[i], op.len[i], true);
      }
      break;
    case OpKind::SmReduce: case OpKind::HostReduce:
      for (int i = 0; i < op.nsrc; ++i) add(op.src[i], op.bytes, false);
      for (int i = 0; i < op.ndst; ++i) add(op.dst[i], op.bytes, true);
      break;
    case OpKind::NvlsReduce:
      // The gang reads every rank's input and writes every rank's output:
      // AllReduce over the op's range, ReduceScatter over the op's range of
      // every slot, the other kinds over the whole message.
      for (int q = 0; q < n; ++q) {
        if (d.kind == Kind::AllReduce) {
          add(send_at(q, op.src[0].off), op.bytes, false);
          add(recv_at(q, op.dst[0].off), op.bytes, true);
        } else if (d.kind == Kind::ReduceScatter) {
          for (int r = 0; r < n; ++r) add(send_at(q, size_t(r) * d.bytes + op.src[0].off), op.bytes, false);
          add(recv_at(q, op.dst[0].off), op.bytes, true);
        } else if (d.kind == Kind::AllGather) {
          add(send_at(q, 0), d.bytes, false);
          add(recv_at(q, 0), d.bytes * size_t(n), true);
        } else {
          add(send_at(q, 0), d.bytes, false);
          add(recv_at(q, 0), d.bytes, true);
        }
      }
      break;
    default:
      break;
  }
}

}  // namespace

std::string check_plan(const Plan& plan, const SimLayout& lay) {
  char msg[512];
  const Graph g = build_graph(plan);
  std::vector<int> order;
  if (!topo_order(g, order, nullptr)) return "plan has a dependency cycle (would deadlock)";
  // Data nodes: every data op except gang members, plus the gang node.
  std::vector<int> data_nodes;
  std::vector<std::vector<Access>> acc;
  std::vector<int> data_index(size_t(g.nodes), -1);
  for (int i = 0; i < int(plan.ops.size()); ++i) {
    const PlanOp& op = plan.ops[size_t(i)];
    if (!is_data(op.kind) || op.kind == OpKind::NvlsReduce) continue;
    data_index[size_t(i)] = int(data_nodes.size());
    data_nodes.push_back(i);
    acc.emplace_back();
    accesses_of(op, lay, plan.desc, acc.back());
  }
  if (g.gang >= 0) {
    data_index[size_t(g.gang)] = int(data_nodes.size());
    data_nodes.push_back(g.gang);
    acc.emplace_back();
    // Every member's range (the low-latency two-shot gives each rank its
    // own slice; the other gangs repeat one range).
    for (const PlanOp& op : plan.ops)
      if (op.kind == OpKind::NvlsReduce) accesses_of(op, lay, plan.desc, acc.back());
  }
  // The reduction kernels issue 16-byte vector accesses: every reduce operand
  // must start on a 16-byte boundary of its (16-byte aligned) buffer.
  for (size_t i = 0; i < plan.ops.size(); ++i) {
    const PlanOp& op = plan.ops[i];
    if (op.kind != OpKind::SmReduce) continue;
    for (int k = 0; k < op.nsrc + op.ndst; ++k) {
      const Loc& l = k < op.nsrc ? op.src[k] : op.dst[k - op.nsrc];
      if (l.off % 16 != 0) {
        std::snprintf(msg, sizeof msg, "op %zu: reduce operand at offset %zu is not 16-byte aligned",
                      i, l.off);
        return msg;
      }
    }
  }
  // The caller's own work before and after the call writes the whole arena
  // of its rank (send and receive buffers, in-place aliases included).
  for (int r = 0; r < lay.nranks; ++r)
    for (int v : {g.producer0 + r, g.consumer0 + r}) {
      data_index[size_t(v)] = int(data_nodes.size());
      data_nodes.push_back(v);
      acc.push_back({Access{r, 0, lay.arena_bytes[r], true}});
    }
  // Bounds: every access inside its arena (device arenas only; host arenas
  // are sized by the plan's needs).
  for (size_t di = 0; di < acc.size(); ++di)
    for (const Access& a : acc[di]) {
      if (a.arena < 0) return "data op with an unbound location";
      if (a.arena < lay.nranks && a.hi > lay.arena_bytes[a.arena]) {
        std::snprintf(msg, sizeof msg, "op %d accesses rank %d bytes [%zu,%zu) beyond %zu",
                      data_nodes[di], a.arena, a.lo, a.hi, lay.arena_bytes[a.arena]);
        return msg;
      }
      if (a.arena >= lay.nranks && a.arena < lay.nranks + kMaxRanks * kMaxLanes &&
          a.hi > plan.needs.bounce_bytes)
        return "bounce access beyond the planned bounce size";
      if (a.arena >= lay.nranks + kTempArena0 && a.hi > plan.needs.temp_bytes)
        return "scratch access beyond the planned scratch size";
    }
  // Ancestor bitsets over data nodes, in topological order.
  const size_t D = data_nodes.size(), W = (D + 63) / 64;
  std::vector<std::vector<uint64_t>> anc(size_t(g.nodes), std::vector<uint64_t>(W, 0));
  for (int v : order) {
    for (int u : g.preds[size_t(v)]) {
      for (size_t w = 0; w < W; ++w) anc[size_t(v)][w] |= anc[size_t(u)][w];
      const int du = data_index[size_t(u)];
      if (du >= 0) anc[size_t(v)][size_t(du) / 64] |= 1ull << (size_t(du) % 64);
    }
  }
  auto before = [&](size_t a, size_t b) {  // data a happens before data b
    const int nb_ = data_nodes[b];
    return (anc[size_t(nb_)][a / 64] >> (a % 64)) & 1;
  };
  for (size_t a = 0; a < D; ++a)
    for (size_t b = a + 1; b < D; ++b) {
      bool conflict = false;
      for (const Access& x : acc[a]) {
        for (const Access& y : acc[b])
          if (x.arena == y.arena && (x.write || y.write) && x.lo < y.hi && y.lo < x.hi) {
            conflict = true;
            break;
          }
        if (conflict) break;
      }
      if (conflict && !before(a, b) && !before(b, a)) {
        auto name = [&](int v) {
          if (v >= g.consumer0) return "the caller's later work on rank " + std::to_string(v - g.consumer0);
          if (v >= g.producer0) return "the caller's earlier work on rank " + std::to_string(v - g.producer0);
          return "op " + std::to_string(v);
        };
        std::snprintf(msg, sizeof msg, "race: %s and %s touch the same bytes unordered",
                      name(data_nodes[a]).c_str(), name(data_nodes[b]).c_str());
        return msg;
      }
    }
  for (int r = 0; r < plan.desc.nranks; ++r) {
    const int end = g.caller_end[size_t(r)];
    for (size_t a = 0; a < D; ++a) {
      if (data_nodes[a] == end || data_nodes[a] >= g.consumer0) continue;
      if (end < 0 || !((anc[size_t(end)][a / 64] >> (a % 64)) & 1)) {
        std::snprintf(msg, sizeof msg, "op %d is not joined into rank %d's caller stream",
                      data_nodes[a], r);
        return msg;
      }
    }
  }
  return "";
}

std::string simulate_plan(const Plan& plan, const SimLayout& lay, const FoldParams& fp,
                          std::vector<std::vector<uint8_t>>& arenas, uint64_t seed) {
  const Graph g = build_graph(plan);
  std::mt19937_64 rng(seed);
  std::vector<int> order;
  if (!topo_order(g, order, &rng)) return "plan has a dependency cycle";
  const int n = lay.nranks;
  std::vector<std::vector<uint8_t>> host(size_t(kTempArena0 + kMaxRanks));
  for (size_t i = 0; i < host.size(); ++i)
    host[i].assign(i < size_t(kTempArena0) ? plan.needs.bounce_bytes : plan.needs.temp_bytes, 0xCD);
  auto ptr = [&](const Loc& l) -> uint8_t* {
    const int a = arena_of(l, n);
    if (a < n) return arenas[size_t(a)].data() + offset_of(l, lay);
    return host[size_t(a - n)].data() + l.off;
  };
  const size_t es = elem_size(plan.desc.dtype);
  std::vector<uint8_t> tmp;
  for (int v : order) {
    if (v == g.gang) {
      // The whole gang collective for every rank at once (an AllReduce gang
      // over the union of its ops' ranges: one shared range, or one slice
      // per rank for the low-latency two-shot).
      size_t bytes = plan.desc.bytes, goff = 0;
      const size_t slot = plan.desc.bytes;  // ReduceScatter: the stride between slots
      if (plan.desc.kind == Kind::AllReduce || plan.desc.kind == Kind::ReduceScatter) {
        size_t lo = ~size_t(0), hi = 0;
        for (const PlanOp& op : plan.ops)
          if (op.kind == OpKind::NvlsReduce) {
            lo = std::min(lo, op.src[0].off);
            hi = std::max(hi, op.src[0].off + op.bytes);
          }
        if (hi > lo) {
          goff = lo;
          bytes = hi - lo;
        }
      }
      auto send = [&](int q) { return arenas[size_t(q)].data() + lay.send_off[q] + goff; };
      auto recv = [&](int q) { return arenas[size_t(q)].data() + lay.recv_off[q] + goff; };
      switch (plan.desc.kind) {
        case Kind::AllReduce: {
          tmp.assign(bytes, 0);
          const void* srcs[kMaxRanks];
          for (int q = 0; q < n; ++q) srcs[q] = send(q);
          host_fold(fp, srcs, n, tmp.data(), bytes);
          for (int q = 0; q < n; ++q) std::memcpy(recv(q), tmp.data(), bytes);
          break;
        }
        case Kind::Broadcast:
          tmp.assign(send(plan.desc.root), send(plan.desc.root) + bytes);
          for (int q = 0; q < n; ++q) std::memcpy(recv(q), tmp.data(), bytes);
          break;
        case Kind::AllGather:
          tmp.clear();
          for (int q = 0; q < n; ++q) tmp.insert(tmp.end(), send(q), send(q) + bytes);
          for (int q = 0; q < n; ++q) std::memcpy(recv(q), tmp.data(), tmp.size());
          break;
        case Kind::ReduceScatter: {
          std::vector<uint8_t> all(bytes * size_t(n));
          for (int r = 0; r < n; ++r) {
            const void* srcs[kMaxRanks];
            for (int q = 0; q < n; ++q) srcs[q] = send(q) + size_t(r) * slot;
            host_fold(fp, srcs, n, all.data() + size_t(r) * bytes, bytes);
          }
          for (int r = 0; r < n; ++r) std::memcpy(recv(r), all.data() + size_t(r) * bytes, bytes);
          break;
        }
        default:
          break;
      }
      continue;
    }
    if (v >= int(plan.ops.size())) continue;
    const PlanOp& op = plan.ops[size_t(v)];
    switch (op.kind) {
      case OpKind::CeCopy:
        std::memmove(ptr(op.dst[0]), ptr(op.src[0]), op.bytes);
        break;
      case OpKind::SmCopy:
        for (int i = 0; i < op.nsrc; ++i) std::memmove(ptr(op.dst[i]), ptr(op.src[i]), op.len[i]);
        break;
      case OpKind::SmReduce: case OpKind::HostReduce: {
        if (es == 0 || op.bytes % es) return "reduce of a partial element";
        tmp.assign(op.bytes, 0);
        const void* srcs[kMaxRanks];
        for (int i = 0; i < op.nsrc; ++i) srcs[i] = ptr(op.src[i]);
        FoldParams p = fp;
        host_fold(p, srcs, op.nsrc, tmp.data(), op.bytes);
        for (int j = 0; j < op.ndst; ++j) std::memcpy(ptr(op.dst[j]), tmp.data(), op.bytes);
        break;
      }
      default:
        break;
    }
  }
  return "";
}

}  // namespace nb
