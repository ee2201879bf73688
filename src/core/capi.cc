// C entry points over the pure core, for the CPU test-suite (ctypes) and for
// tools. Nothing here touches CUDA or NCCL; a fake GroupBackend stands in
// for libnccl and the clique runner.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <random>
#include <string>
#include <vector>

#include "core/bufclass.h"
#include "core/calib_model.h"
#include "core/clique.h"
#include "core/nvls_sched.h"
#include "core/exec_loop.h"
#include "core/fault.h"
#include "core/gate.h"
#include "core/group.h"
#include "core/hostreduce.h"
#include "core/plan.h"
#include "core/plan_sim.h"
#include "core/policy.h"
#include "core/summary.h"

using namespace nb;

namespace {

// "K=V;K=V" -> lookup function over that map.
struct EnvMap {
  std::map<std::string, std::string> kv;
  explicit EnvMap(const char* spec) {
    if (!spec) return;
    std::string s(spec);
    size_t pos = 0;
    while (pos < s.size()) {
      size_t semi = s.find(';', pos);
      if (semi == std::string::npos) semi = s.size();
      const std::string item = s.substr(pos, semi - pos);
      const size_t eq = item.find('=');
      if (eq != std::string::npos) kv[item.substr(0, eq)] = item.substr(eq + 1);
      pos = semi + 1;
    }
  }
  Policy policy() const {
    return policy_from_env([this](const char* k) -> const char* {
      const auto it = kv.find(k);
      return it == kv.end() ? nullptr : it->second.c_str();
    });
  }
};

void copy_out(const std::string& s, char* buf, size_t cap) {
  if (!buf || !cap) return;
  const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
  std::memcpy(buf, s.data(), n);
  buf[n] = 0;
}

}  // namespace

extern "C" {

struct nb_call_t {
  int kind, dtype, op;
  uint64_t count, send, recv;
  int device, rank, nranks, root;
};

static CallDesc to_desc(const nb_call_t& c) {
  CallDesc d;
  d.kind = Kind(c.kind);
  d.dtype = DType(c.dtype);
  d.op = RedOp(c.op);
  d.count = size_t(c.count);
  d.send = uintptr_t(c.send);
  d.recv = uintptr_t(c.recv);
  d.device = c.device;
  d.rank = c.rank;
  d.nranks = c.nranks;
  d.root = c.root;
  return d;
}

const char* nb_reason_name(int r) { return reason_name(Reason(r)); }
const char* nb_algo_name(int a) { return algo_name(Algo(a)); }
int nb_reason_count() { return int(Reason::Count); }
int nb_algo_count() { return int(Algo::Count); }
int nb_dtype_from_nccl(int t) { return int(dtype_from_nccl(t)); }
uint64_t nb_elem_size(int t) { return elem_size(DType(t)); }

int nb_gate_message(const nb_call_t* c, const char* env) {
  return int(gate_message(to_desc(*c), EnvMap(env).policy()));
}
int nb_gate_call(const nb_call_t* c, const char* env) {
  return int(gate_call(to_desc(*c), EnvMap(env).policy()));
}

// flags: 1 known clique, 2 capturing, 4 first pass done, 8 poisoned,
// 16 nccl unsupported, 32 nvls available.
int nb_gate_clique(const nb_call_t* calls, int n, int flags, const char* env, int* algo) {
  std::vector<CallDesc> v;
  for (int i = 0; i < n; ++i) v.push_back(to_desc(calls[i]));
  CliqueState s;
  s.known_clique = flags & 1;
  s.capturing = flags & 2;
  s.first_pass_done = flags & 4;
  s.poisoned = flags & 8;
  s.nccl_supported = !(flags & 16);
  s.nvls_available = flags & 32;
  const CliqueDecision d = gate_clique(v, s, EnvMap(env).policy());
  if (algo) *algo = int(d.algo);
  return int(d.reason);
}

// The clique gate with per-rank PreMulSum scalars (value, residence:
// 1 host immediate, 0 device pointer).
int nb_gate_clique_scalars(const nb_call_t* calls, int n, int flags, const char* env, int* algo,
                           const double* scalars, const int* residence) {
  std::vector<CallDesc> v;
  for (int i = 0; i < n; ++i) {
    CallDesc d = to_desc(calls[i]);
    d.scalar = scalars[i];
    d.scalar_residence = residence[i];
    v.push_back(d);
  }
  CliqueState s;
  s.known_clique = flags & 1;
  s.capturing = flags & 2;
  s.first_pass_done = flags & 4;
  s.poisoned = flags & 8;
  s.nccl_supported = !(flags & 16);
  s.nvls_available = flags & 32;
  const CliqueDecision d = gate_clique(v, s, EnvMap(env).policy());
  if (algo) *algo = int(d.algo);
  return int(d.reason);
}

struct nb_plan_stats_t {
  uint64_t ops, records, waits, data_ops, sm_bytes, ce_bytes, host_bytes;
  int lanes;
  uint64_t bounce_bytes;
  int phase_events;
  uint64_t mismatches;
};

// Builds the plan, checks its happens-before structure, runs it on host
// memory in a random topological order with seeded data, and compares every
// output byte with the direct oracle (host fold over whole buffers).
// data_mode 0: exactly-summable integers; 1: uniform[-1,1] floats.
// Returns 0 on success, 1 on a plan-check error, 2 on output mismatches,
// 3 on a bad argument; `err` gets a description.
int nb_plan_simulate(int algo, int kind, int dtype, int op, int nranks, uint64_t count, int root,
                     int inplace_mask, int host_ppm, int ce_ppm, const char* env, uint64_t seed,
                     int data_mode, const double* scalars, nb_plan_stats_t* stats, char* err,
                     size_t errcap) {
  const Policy p = EnvMap(env).policy();
  CliqueDesc d;
  d.kind = Kind(kind);
  d.dtype = DType(dtype);
  d.op = RedOp(op);
  d.nranks = nranks;
  d.count = size_t(count);
  d.bytes = size_t(count) * elem_size(d.dtype);
  d.root = root;
  if (nranks < 1 || nranks > kMaxRanks || !elem_size(d.dtype)) {
    copy_out("bad arguments", err, errcap);
    return 3;
  }
  for (int r = 0; r < nranks; ++r) d.in_place[r] = (inplace_mask >> r) & 1;
  Shares s;
  s.host_ppm = host_ppm;
  s.ce_ppm = ce_ppm;
  Plan plan;
  build_plan(Algo(algo), d, p, s, plan);
  if (stats) {
    *stats = nb_plan_stats_t{};
    stats->ops = plan.ops.size();
    for (const PlanOp& o : plan.ops) {
      stats->records += o.kind == OpKind::Record;
      stats->waits += o.kind == OpKind::Wait;
      stats->data_ops += is_data_op(o.kind);
    }
    stats->sm_bytes = plan.sm_bytes;
    stats->ce_bytes = plan.ce_bytes;
    stats->host_bytes = plan.host_bytes;
    stats->lanes = plan.needs.lanes;
    stats->bounce_bytes = plan.needs.bounce_bytes;
    stats->phase_events = plan.needs.phase_events;
  }
  const SimLayout lay = layout_for(d);
  const std::string check = check_plan(plan, lay);
  if (!check.empty()) {
    copy_out(check, err, errcap);
    return 1;
  }
  // Seeded inputs.
  std::mt19937_64 rng(seed);
  std::vector<std::vector<uint8_t>> arenas{size_t(nranks)};
  for (int r = 0; r < nranks; ++r) arenas[size_t(r)].assign(lay.arena_bytes[r], 0xEE);
  const size_t es = elem_size(d.dtype);
  const size_t send_elems = (d.kind == Kind::ReduceScatter ? size_t(nranks) : 1) * d.count;
  auto gen = [&](uint8_t* dst) {
    for (size_t e = 0; e < send_elems; ++e) {
      const double u = double(rng() >> 11) * (1.0 / 9007199254740992.0);  // [0,1)
      const long long k = (long long)(rng() % 255) - 127;                   // exact
      const double v = data_mode == 1 ? 2.0 * u - 1.0 : double(k);
      switch (d.dtype) {
        case DType::F32: { const float f = float(v); std::memcpy(dst + e * 4, &f, 4); break; }
        case DType::F64: std::memcpy(dst + e * 8, &v, 8); break;
        case DType::F16: { const uint16_t h = float_to_half(float(v)); std::memcpy(dst + e * 2, &h, 2); break; }
        case DType::BF16: { const uint16_t h = float_to_bf16(float(v)); std::memcpy(dst + e * 2, &h, 2); break; }
        default: {
          const uint64_t x = rng();
          std::memcpy(dst + e * es, &x, es);
          break;
        }
      }
    }
  };
  for (int r = 0; r < nranks; ++r)
    if (lay.send_valid[r]) gen(arenas[size_t(r)].data() + lay.send_off[r]);
  // Oracle on copies of the inputs.
  std::vector<std::vector<uint8_t>> inputs{size_t(nranks)};
  for (int r = 0; r < nranks; ++r)
    if (lay.send_valid[r])
      inputs[size_t(r)].assign(arenas[size_t(r)].begin() + long(lay.send_off[r]),
                               arenas[size_t(r)].begin() + long(lay.send_off[r] + send_elems * es));
  FoldParams fp;
  fp.dtype = d.dtype;
  fp.op = d.op;
  fp.nranks = nranks;
  for (int r = 0; r < nranks; ++r) fp.scalars[r] = scalars ? scalars[r] : 1.0;
  std::vector<std::vector<uint8_t>> expect{size_t(nranks)};
  const size_t n = d.bytes;
  for (int r = 0; r < nranks; ++r) {
    switch (d.kind) {
      case Kind::AllReduce: {
        expect[size_t(r)].assign(n, 0);
        const void* srcs[kMaxRanks];
        for (int q = 0; q < nranks; ++q) srcs[q] = inputs[size_t(q)].data();
        host_fold(fp, srcs, nranks, expect[size_t(r)].data(), n);
        break;
      }
      case Kind::ReduceScatter: {
        expect[size_t(r)].assign(n, 0);
        const void* srcs[kMaxRanks];
        for (int q = 0; q < nranks; ++q) srcs[q] = inputs[size_t(q)].data() + size_t(r) * n;
        host_fold(fp, srcs, nranks, expect[size_t(r)].data(), n);
        break;
      }
      case Kind::AllGather:
        for (int q = 0; q < nranks; ++q)
          expect[size_t(r)].insert(expect[size_t(r)].end(), inputs[size_t(q)].begin(), inputs[size_t(q)].end());
        break;
      case Kind::Broadcast:
        expect[size_t(r)] = inputs[size_t(root)];
        break;
      default: break;
    }
  }
  const std::string sim = simulate_plan(plan, lay, fp, arenas, seed ^ 0x5eedull);
  if (!sim.empty()) {
    copy_out(sim, err, errcap);
    return 1;
  }
  uint64_t bad = 0;
  std::string first;
  for (int r = 0; r < nranks; ++r) {
    const uint8_t* out = arenas[size_t(r)].data() + lay.recv_off[r];
    const std::vector<uint8_t>& e = expect[size_t(r)];
    for (size_t i = 0; i < e.size(); ++i)
      if (out[i] != e[i]) {
        if (!bad) first = "rank " + std::to_string(r) + " byte " + std::to_string(i);
        ++bad;
      }
  }
  if (stats) stats->mismatches = bad;
  if (bad) {
    copy_out("mismatch at " + first, err, errcap);
    return 2;
  }
  copy_out("", err, errcap);
  return 0;
}

// Checker self-test: build a plan, delete its `drop`-th Wait op, and report
// whether the happens-before checker rejects the mutated plan (1), accepts
// it (0), or the plan has fewer waits (-1). A checker that accepts plans
// with missing waits would let real ordering bugs through.
int nb_plan_mutation(int algo, int kind, int nranks, uint64_t count, int host_ppm, int ce_ppm,
                     const char* env, int drop, char* err, size_t errcap) {
  const Policy p = EnvMap(env).policy();
  CliqueDesc d;
  d.kind = Kind(kind);
  d.dtype = DType::F32;
  d.op = RedOp::Sum;
  d.nranks = nranks;
  d.count = size_t(count);
  d.bytes = d.count * 4;
  d.root = 0;
  Shares s;
  s.host_ppm = host_ppm;
  s.ce_ppm = ce_ppm;
  Plan plan;
  build_plan(Algo(algo), d, p, s, plan);
  int seen = 0;
  for (size_t i = 0; i < plan.ops.size(); ++i) {
    if (plan.ops[i].kind != OpKind::Wait) continue;
    if (seen++ == drop) {
      plan.ops.erase(plan.ops.begin() + long(i));
      const std::string r = check_plan(plan, layout_for(d));
      copy_out(r, err, errcap);
      return r.empty() ? 0 : 1;
    }
  }
  return -1;
}

// Host fold exposed directly (tests compare it with numpy / serial sums).
void nb_host_fold(int dtype, int op, int nranks, const void* const* srcs, int nsrc, void* dst,
                  uint64_t bytes, const double* scalars, int threads) {
  FoldParams p;
  p.dtype = DType(dtype);
  p.op = RedOp(op);
  p.nranks = nranks;
  for (int i = 0; i < nsrc && i < kMaxRanks; ++i) p.scalars[i] = scalars ? scalars[i] : 1.0;
  host_fold_parallel(p, srcs, nsrc, dst, size_t(bytes), threads);
}

uint16_t nb_float_to_half(float f) { return float_to_half(f); }
float nb_half_to_float(uint16_t h) { return half_to_float(h); }
uint16_t nb_float_to_bf16(float f) { return float_to_bf16(f); }
float nb_bf16_to_float(uint16_t h) { return bf16_to_float(h); }

// Policy field readback for tests: returns the value as a double.
// Pack an NVLS kernel shape and read it back: out = {movers, unroll,
// round MiB, ramp, ahead}. Returns the packed value.
int nb_nvls_shape(int movers, int unroll, int round_mib, int ramp, int ahead, int* out) {
  const int v = pack_nvls_shape(movers, unroll, round_mib, ramp, ahead);
  Shares s;
  unpack_nvls_shape(v, &s);
  out[0] = s.nvls_movers;
  out[1] = s.nvls_unroll;
  out[2] = s.nvls_round_mib;
  out[3] = s.nvls_ramp;
  out[4] = s.nvls_ahead;
  return v;
}

// The NVLS AllReduce round schedule: the number of rounds, and round s's
// [base, base + len) when s is below it.
int nb_nvls_ar_round(uint64_t bytes, uint64_t round, int ramp, unsigned s, uint64_t* base, uint64_t* len) {
  if (round == 0) return -1;
  const unsigned n = ar_rounds(bytes, round, ramp);
  if (s < n) {
    unsigned long long b = 0, l = 0;
    ar_round(s, bytes, round, ramp, &b, &l);
    *base = b;
    *len = l;
  }
  return int(n);
}

double nb_policy_value(const char* env, const char* field) {
  const Policy p = EnvMap(env).policy();
  const std::string f(field);
  if (f == "enabled") return p.enabled;
  if (f == "local_copy_tma") return p.local_copy_tma ? 1 : 0;
  if (f == "ar_min") return double(p.min_bytes[0]);
  if (f == "ag_min") return double(p.min_bytes[1]);
  if (f == "rs_min") return double(p.min_bytes[2]);
  if (f == "bc_min") return double(p.min_bytes[3]);
  if (f == "max_bytes") return double(p.max_message_bytes);
  if (f == "first_pass") return p.first_pass;
  if (f == "nvls") return double(int(p.nvls));
  if (f == "host_share_ppm") return p.host_share_ppm;
  if (f == "ce_share_ppm") return p.ce_share_ppm;
  if (f == "lanes") return p.lanes;
  if (f == "host_piece") return double(p.host_piece);
  if (f == "summary") return p.summary;
  if (f == "timeout_ns") return double(p.device_timeout_ns);
  if (f == "force_ar") return double(int(p.force_algo[0]));
  if (f == "force_bc") return double(int(p.force_algo[3]));
  if (f == "force_ag") return double(int(p.force_algo[1]));
  if (f == "force_rs") return double(int(p.force_algo[2]));
  if (f == "ring_chunk") return double(p.ring_chunk);
  if (f == "nvls_round") return double(p.nvls_round_bytes);
  if (f == "min_host_bytes") return double(p.min_host_bytes);
  if (f == "hybrid_nvls_ppm") return p.hybrid_nvls_ppm;
  if (f == "hybrid_blocks") return p.hybrid_blocks;
  if (f == "nvls_tma") return p.nvls_tma;
  if (f == "nvls_ramp") return p.nvls_ramp;
  if (f == "nvls_strong") return p.nvls_strong;
  if (f == "nvls_buffers") return p.nvls_buffers;
  if (f == "nvls_ahead") return p.nvls_ahead;
  if (f == "nvls_trace") return p.nvls_trace;
  if (f == "nvtx") return p.nvtx;
  if (f == "nvls_movers") return p.nvls_movers;
  if (f == "tune_bytes") return double(p.tune_bytes);
  return -1;
}

void nb_shares_from(double sm, double ce, double mix, double ce_frac, double d2h, double h2d,
                    double fold, int algo, int n, int* host_ppm, int* ce_ppm) {
  CalibResult c;
  c.valid = true;
  c.nvlink_sm_gbs = sm;
  c.nvlink_ce_gbs = ce;
  c.nvlink_mix_gbs = mix;
  c.mix_ce_fraction = ce_frac;
  c.pcie_d2h_gbs = d2h;
  c.pcie_h2d_gbs = h2d;
  c.fold_gbs = fold;
  const Shares s = shares_from(c, Algo(algo), n);
  *host_ppm = s.host_ppm;
  *ce_ppm = s.ce_ppm;
}

// The size-aware route choice after a JSON round trip: AllReduce tuned to
// `pref` at the large size and `small_pref` below `below_mib`; returns the
// route for a message of `logical` bytes and the small choice's CE share.
int nb_calib_small(int pref, int small_pref, int below_mib, uint64_t logical, int* small_ce) {
  CalibResult c;
  c.valid = true;
  c.nvlink_sm_gbs = 700;
  c.preferred[0] = pref;
  c.ce_ppm[0] = 1111;
  c.small_pref[0] = small_pref;
  c.small_ce_ppm[0] = 2222;
  c.small_below_mib = below_mib;
  CalibResult d;
  if (!calib_from_json(calib_to_json(c, "k"), "k", &d)) return -1;
  *small_ce = shares_from(d, Algo(small_pref), 2, small_message(d, size_t(logical))).ce_ppm;
  return int(tuned_route(d, 0, size_t(logical)));
}

int nb_calib_roundtrip(double sm, const char* key, double* back) {
  CalibResult c;
  c.valid = true;
  c.nvlink_sm_gbs = sm;
  c.fold_gbs = 2 * sm;
  CalibResult d;
  if (!calib_from_json(calib_to_json(c, key), key, &d)) return 0;
  *back = d.nvlink_sm_gbs;
  return calib_from_json(calib_to_json(c, key), std::string(key) + "x", &d) ? 2 : 1;
}

// ---- Group machine with a fake libnccl -------------------------------------
//
// Script tokens (space separated):
//   S            ncclGroupStart        E   ncclGroupEnd
//   A<k>         AllReduce on comm k   G<k> AllGather on comm k
//   B<k>         AllReduce on comm k that fails the call gate (misaligned)
//   U            an unsupported operation (e.g. ncclSend)
//   I            ncclGroupSimulateEnd
// Comms 0..n-1 form one clique of n ranks on devices 0..n-1. The fake
// runner handles a complete set unless `run_result` says otherwise
// (0 handled, 1 fallback, 2 error). Output: one line per event:
//   F <call-id>    forwarded to "libnccl" (call ids count every collective)
//   C <ids...>     ran custom
//   RS / RE        real GroupStart / GroupEnd
//   R <code>       return code of the API call
class FakeBackend final : public GroupBackend {
 public:
  FakeBackend(int n, int run_result) : n_(n), run_result_(run_result) {
    policy_.first_pass = false;
    policy_.min_bytes[0] = policy_.min_bytes[1] = 0;
  }
  int real_group_start() override { out += "RS\n"; return 0; }
  int real_group_end() override { out += "RE\n"; return 0; }
  int real_simulate_end(void*) override { out += "RE\n"; return 0; }
  int forward(const Call& c, Reason) override {
    out += "F " + std::to_string(uintptr_t(c.stream)) + "\n";
    return 0;
  }
  bool query(Call& c) override {
    const int k = int(reinterpret_cast<uintptr_t>(c.comm)) - 1;
    c.desc.device = k;
    c.desc.rank = k;
    c.desc.nranks = n_;
    return true;
  }
  const Policy& policy(int) override { return policy_; }
  Outcome run(std::vector<Call>& calls, Reason& reason) override {
    // Like the real clique gate: one call per rank, all of one kind.
    unsigned ranks = 0;
    for (const Call& c : calls) {
      if ((ranks >> c.desc.rank) & 1u || c.desc.kind != calls[0].desc.kind) {
        reason = Reason::NotClique;
        return Outcome::Fallback;
      }
      ranks |= 1u << c.desc.rank;
    }
    reason = Reason::None;
    if (run_result_ == 1) return Outcome::Fallback;
    if (run_result_ == 2) return Outcome::Error;
    out += "C";
    for (const Call& c : calls) out += " " + std::to_string(uintptr_t(c.stream));
    out += "\n";
    return Outcome::Handled;
  }
  std::string out;

 private:
  int n_;
  int run_result_;
  Policy policy_;
};

int nb_group_script(const char* script, int nranks, int run_result, char* out, size_t cap) {
  FakeBackend fake(nranks, run_result);
  GroupMachine m(fake);
  GroupState g;
  std::string s(script);
  size_t pos = 0;
  uintptr_t next_id = 1;
  while (pos < s.size()) {
    while (pos < s.size() && s[pos] == ' ') ++pos;
    size_t end = s.find(' ', pos);
    if (end == std::string::npos) end = s.size();
    const std::string tok = s.substr(pos, end - pos);
    pos = end;
    if (tok.empty()) continue;
    int rc = 0;
    if (tok == "S") {
      rc = m.group_start(g);
    } else if (tok == "E") {
      rc = m.group_end(g);
    } else if (tok == "I") {
      rc = m.simulate_end(g, nullptr);
    } else if (tok == "U") {
      rc = m.force_passthrough(g);
    } else if (tok[0] == 'A' || tok[0] == 'G' || tok[0] == 'B') {
      const int k = std::atoi(tok.c_str() + 1);
      Call c;
      c.desc.kind = tok[0] == 'G' ? Kind::AllGather : Kind::AllReduce;
      c.desc.dtype = DType::F32;
      c.desc.count = 1 << 20;
      const uintptr_t base = 0x100000000ull * uintptr_t(k + 1);
      c.desc.send = base + (tok[0] == 'B' ? 4 : 0);
      c.desc.recv = base + 0x10000000ull;
      c.comm = reinterpret_cast<void*>(uintptr_t(k + 1));
      c.stream = reinterpret_cast<void*>(next_id++);  // the call id
      rc = m.enqueue(g, c);
    } else {
      return -1;
    }
    fake.out += "R " + std::to_string(rc) + "\n";
  }
  copy_out(fake.out, out, cap);
  return int(fake.out.size());
}

// ---- Clique registry ------------------------------------------------------
static CliqueRegistry g_test_registry;
int nb_clique_add(const uint64_t* comms, const int* devices, int n) {
  void* c[kMaxRanks];
  for (int i = 0; i < n && i < kMaxRanks; ++i) c[i] = reinterpret_cast<void*>(uintptr_t(comms[i]));
  return g_test_registry.add(c, devices, n);
}
void nb_clique_forget(uint64_t comm) { g_test_registry.forget(reinterpret_cast<void*>(uintptr_t(comm))); }
int nb_clique_same(const uint64_t* comms, int n) {
  std::vector<void*> v;
  for (int i = 0; i < n; ++i) v.push_back(reinterpret_cast<void*>(uintptr_t(comms[i])));
  return g_test_registry.same_clique(v, nullptr) ? 1 : 0;
}
int nb_clique_count() { return int(g_test_registry.size()); }

int nb_inits_form_clique(const int* ranks, const int* nranks, const int* id_bytes, int n) {
  std::vector<PendingInit> v;
  static void* outs[kMaxRanks * 2];
  for (int i = 0; i < n; ++i) {
    PendingInit p;
    p.rank = ranks[i];
    p.nranks = nranks[i];
    p.output = &outs[i];
    std::memset(p.id, id_bytes[i], sizeof(p.id));
    v.push_back(p);
  }
  return inits_form_clique(v) ? 1 : 0;
}

// ---- Error policy with the fault injector ---------------------------------
// Runs the AllReduce plan for n ranks through the submission loop with a
// submitter that always succeeds; returns 0 Ok, 1 NotStarted, 2 Failed and
// the failing op index in *at; *first_data gets the first data op's index.
int nb_fault_policy(const char* spec, int nranks, uint64_t bytes, uint64_t* at, uint64_t* first_data) {
  FaultInjector f;
  if (!f.configure(spec)) return -1;
  CliqueDesc d;
  d.kind = Kind::AllReduce;
  d.dtype = DType::F32;
  d.nranks = nranks;
  d.bytes = size_t(bytes);
  d.count = d.bytes / 4;
  Plan plan;
  build_plan(Algo::ArTwoShot, d, default_policy(), Shares{}, plan);
  *first_data = ~0ull;
  for (size_t i = 0; i < plan.ops.size(); ++i)
    if (is_data_op(plan.ops[i].kind)) {
      *first_data = i;
      break;
    }
  if (f.fail_setup()) return 3;
  int code = 0;
  size_t failed = 0;
  const ExecStatus s = run_plan_ops(plan, [](const PlanOp&, size_t) { return 0; }, &f, 999, &code, &failed);
  *at = failed;
  return s == ExecStatus::Ok ? 0 : s == ExecStatus::NotStarted ? 1 : 2;
}

// ---- Summary golden -------------------------------------------------------
int nb_summary_sample(char* out, size_t cap) {
  Summary s;
  s.set_enabled(true);
  s.count_custom(Algo::ArTwoShot, 8ull << 30, 2, 100, 10, 1);
  s.count_fallback(Reason::FirstPass);
  s.count_fallback(Reason::BelowThreshold);
  s.count_fallback(Reason::BelowThreshold);
  int devs[2] = {0, 1};
  s.note_clique(2, devs);
  s.note_placement(0, 1, 0, 0, "mbind");
  std::string all;
  for (const std::string& l : s.render("test")) all += l + "\n";
  copy_out(all, out, cap);
  return int(all.size());
}



// ---- Buffer classification (pointer facts -> class) ------------------------

struct nb_facts_t {
  int known, device_memory, device, from_pool, legacy_ipc, ndev;
  uint64_t range_start, range_size, mapping_start, mapping_size;
  int access[kMaxRanks];  // Access enum values
};

static PointerFacts to_facts(const nb_facts_t& c) {
  PointerFacts f;
  f.known = c.known != 0;
  f.device_memory = c.device_memory != 0;
  f.device = c.device;
  f.from_pool = c.from_pool != 0;
  f.legacy_ipc = c.legacy_ipc;
  f.ndev = c.ndev;
  f.range_start = c.range_start;
  f.range_size = c.range_size;
  f.mapping_start = c.mapping_start;
  f.mapping_size = c.mapping_size;
  for (int i = 0; i < kMaxRanks; ++i) f.access[i] = Access(c.access[i]);
  return f;
}

// 0 refused, 1 ordinary, 2 mapped; the deciding rule's name into `rule`.
int nb_classify_buffer(const nb_facts_t* first, const nb_facts_t* last, uint64_t addr, uint64_t bytes,
                       int device, char* rule, size_t cap) {
  const BufferVerdict v = classify_buffer(to_facts(*first), to_facts(*last), addr, bytes, device);
  copy_out(v.rule, rule, cap);
  return int(v.cls);
}

}  // extern "C"
