// Randomized self-test of the CUDA-free core, built with AddressSanitizer
// and UndefinedBehaviorSanitizer (`make sanitize`, run by the CPU test-suite).
// It drives every layer through many seeded cases so that an out-of-bounds
// access, use after free, signed overflow or misaligned load in the pure
// code aborts the run:
//   - plans: every valid (route, kind) for 1..8 ranks, random counts, dtypes,
//     ops, CE/host shares, in-place masks and roots; built, checked for races
//     and bounds, and simulated on host memory against the direct oracle;
//   - group machine: random ncclGroupStart/End/collective/unsupported/
//     SimulateEnd scripts against the fake backend;
//   - host fold: random dtypes, ops, source counts, sizes and thread counts;
//   - gates: random call descriptors through the message, call and clique
//     gates; the fault policy, summary and calibration JSON.
// Exit status 0 when every plan simulation matched its oracle.
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "core/gate.h"
#include "core/hostreduce.h"
#include "core/types.h"

extern "C" {
struct nb_call_t {
  int kind, dtype, op;
  uint64_t count, send, recv;
  int device, rank, nranks, root;
};
struct nb_plan_stats_t {
  uint64_t ops, records, waits, data_ops, sm_bytes, ce_bytes, host_bytes;
  int lanes;
  uint64_t bounce_bytes;
  int phase_events;
  uint64_t mismatches;
};
int nb_plan_simulate(int algo, int kind, int dtype, int op, int nranks, uint64_t count, int root,
                     int inplace_mask, int host_ppm, int ce_ppm, const char* env, uint64_t seed,
                     int data_mode, const double* scalars, nb_plan_stats_t* stats, char* err,
                     size_t errcap);
int nb_group_script(const char* script, int nranks, int run_result, char* out, size_t cap);
int nb_gate_message(const nb_call_t* c, const char* env);
int nb_gate_call(const nb_call_t* c, const char* env);
int nb_gate_clique(const nb_call_t* calls, int n, int flags, const char* env, int* algo);
int nb_fault_policy(const char* spec, int nranks, uint64_t bytes, uint64_t* at, uint64_t* first_data);
int nb_summary_sample(char* out, size_t cap);
int nb_calib_roundtrip(double sm, const char* key, double* back);
int nb_calib_small(int pref, int small_pref, int below_mib, uint64_t logical, int* small_ce);
}

namespace {

using namespace nb;

int plans(std::mt19937_64& rng, int cases) {
  const Kind kinds[] = {Kind::AllReduce, Kind::AllGather, Kind::ReduceScatter, Kind::Broadcast};
  const DType dtypes[] = {DType::F32, DType::BF16, DType::F16, DType::I32, DType::F64, DType::I8,
                          DType::U8, DType::I64};
  const RedOp ops[] = {RedOp::Sum, RedOp::Prod, RedOp::Max, RedOp::Min, RedOp::Avg,
                       RedOp::PreMulSum};
  const int ppms[] = {0, 0, 500, 2500, 5000, 10000};
  int failures = 0, ran = 0;
  for (int i = 0; i < cases; ++i) {
    const Kind k = kinds[rng() % 4];
    const int n = 1 + int(rng() % 8);
    const DType t = dtypes[rng() % 8];
    const RedOp op = reduces(k) ? ops[rng() % 6] : RedOp::Sum;
    std::vector<Algo> valid;
    for (int x = 1; x < int(Algo::Count); ++x)
      if (algo_valid(Algo(x), k, n, t, op, true)) valid.push_back(Algo(x));
    if (valid.empty()) continue;
    const Algo a = valid[rng() % valid.size()];
    // Counts: tiny, odd, vector tails and a few larger ones. The message gate
    // admits a ReduceScatter only when its slot is a multiple of 16 bytes.
    uint64_t count = 1 + rng() % 4099;
    if (rng() % 4 == 0) count = (1 + rng() % 16) * 1024 + rng() % 9;
    if (k == Kind::ReduceScatter) {
      const uint64_t unit = 16 / elem_size(t) ? 16 / elem_size(t) : 1;
      count = (count + unit - 1) / unit * unit;
    }
    const int host = ppms[rng() % 6] / 2, ce = ppms[rng() % 6];
    const int mask = rng() % 3 == 0 ? int((1u << n) - 1) : int(rng() % (1u << n));
    const int root = int(rng() % unsigned(n));
    double sc[8];
    for (double& s : sc) s = 0.25 * double(1 + rng() % 8);
    // Small host pieces so that short messages still use several lanes.
    const char* env = rng() % 2 ? "NCCL_B200_HOST_PIECE=4096;NCCL_B200_MIN_HOST_BYTES=0" : "";
    nb_plan_stats_t st;
    char err[512] = {0};
    const int data_mode = is_float(t) && rng() % 2 ? 1 : 0;
    const int rc = nb_plan_simulate(int(a), int(k), int(t), int(op), n, count, root, mask, host, ce,
                                    env, rng(), data_mode, sc, &st, err, sizeof err);
    ++ran;
    if (rc != 0) {
      ++failures;
      if (failures < 10)
        std::printf("plan FAIL rc=%d algo=%s kind=%s n=%d dtype=%d op=%d count=%llu mask=%d root=%d "
                    "host=%d ce=%d: %s\n",
                    rc, algo_name(a), kind_name(k), n, int(t), int(op), (unsigned long long)count,
                    mask, root, host, ce, err);
    }
  }
  std::printf("plans: %d simulated, %d failed\n", ran, failures);
  return failures;
}

void groups(std::mt19937_64& rng, int cases) {
  const char* fixed[] = {"S", "E", "U", "I"};
  char out[1 << 16];
  for (int i = 0; i < cases; ++i) {
    const int n = 1 + int(rng() % 8);
    std::string s;
    const int len = 1 + int(rng() % 40);
    for (int j = 0; j < len; ++j) {
      const unsigned r = unsigned(rng() % 10);
      if (r < 4) s += fixed[r];
      else s += std::string(1, "AAGB"[rng() % 4]) + std::to_string(rng() % unsigned(n));
      s += ' ';
    }
    nb_group_script(s.c_str(), n, int(rng() % 3), out, sizeof out);
  }
  std::printf("group scripts: %d\n", cases);
}

void folds(std::mt19937_64& rng, int cases) {
  const DType dtypes[] = {DType::F32, DType::BF16, DType::F16, DType::I32, DType::F64, DType::I8,
                          DType::U8, DType::I64, DType::U32, DType::U64};
  const RedOp ops[] = {RedOp::Sum, RedOp::Prod, RedOp::Max, RedOp::Min, RedOp::Avg,
                       RedOp::PreMulSum};
  for (int i = 0; i < cases; ++i) {
    FoldParams p;
    p.dtype = dtypes[rng() % 10];
    p.op = ops[rng() % 6];
    if (p.op == RedOp::PreMulSum && !is_float(p.dtype)) p.op = RedOp::Sum;
    const int nsrc = 1 + int(rng() % 8);
    p.nranks = nsrc;
    for (int r = 0; r < nsrc; ++r) p.scalars[r] = 0.5 * double(1 + rng() % 4);
    const size_t es = elem_size(p.dtype);
    const size_t elems = rng() % 5000;
    std::vector<std::vector<uint8_t>> src(size_t(nsrc), std::vector<uint8_t>(elems * es + 1));
    for (auto& v : src)
      for (auto& b : v) b = uint8_t(rng());
    std::vector<const void*> ptrs;
    for (auto& v : src) ptrs.push_back(v.data());
    std::vector<uint8_t> dst(elems * es + 1);
    host_fold_parallel(p, ptrs.data(), nsrc, dst.data(), elems * es, 1 + int(rng() % 4));
  }
  std::printf("host folds: %d\n", cases);
}

void gates(std::mt19937_64& rng, int cases) {
  for (int i = 0; i < cases; ++i) {
    const int n = 1 + int(rng() % 8);
    std::vector<nb_call_t> calls(static_cast<size_t>(n));
    const int kind = int(rng() % 4), dtype = int(rng() % 13), op = int(rng() % 7);
    const uint64_t count = rng() % 2 ? rng() % (1ull << 32) : rng();
    for (int r = 0; r < n; ++r) {
      nb_call_t& c = calls[size_t(r)];
      c.kind = rng() % 16 ? kind : int(rng() % 4);
      c.dtype = dtype;
      c.op = op;
      c.count = count;
      c.send = rng() % 8 ? (uint64_t(r + 1) << 36) + (rng() % 64) : rng();
      c.recv = rng() % 8 ? (uint64_t(r + 1) << 36) + (1ull << 35) : rng();
      c.device = r;
      c.rank = rng() % 16 ? r : int(rng() % 9) - 1;
      c.nranks = n;
      c.root = int(rng() % unsigned(n + 1)) - 1;
      nb_gate_message(&c, "");
      nb_gate_call(&c, "NCCL_B200_AR_MIN=0;NCCL_B200_AG_MIN=0");
    }
    int algo = -1;
    nb_gate_clique(calls.data(), n, int(rng() % 64), rng() % 2 ? "" : "NCCL_B200_ALGO=ar=nvls,bc=chain",
                   &algo);
  }
  std::printf("gate calls: %d\n", cases);
}

}  // namespace

int main(int argc, char** argv) {
  const int scale = argc > 1 ? std::atoi(argv[1]) : 1;
  std::setvbuf(stdout, nullptr, _IOLBF, 0);
  std::mt19937_64 rng(20260101);
  auto t0 = std::chrono::steady_clock::now();
  auto lap = [&](const char* what) {
    const auto t1 = std::chrono::steady_clock::now();
    std::printf("  %s: %.2f s\n", what, std::chrono::duration<double>(t1 - t0).count());
    t0 = t1;
  };
  const int failures = plans(rng, 400 * scale);
  lap("plans");
  groups(rng, 2000 * scale);
  lap("groups");
  folds(rng, 60 * scale);
  lap("folds");
  gates(rng, 2000 * scale);
  lap("gates");
  uint64_t at = 0, first = 0;
  const char* specs[] = {"", "setup", "op:0", "op:3", "op:7:always", "bad", "op:", "op:99999999999"};
  for (const char* s : specs) nb_fault_policy(s, 4, 1ull << 30, &at, &first);
  char buf[1 << 14];
  nb_summary_sample(buf, sizeof buf);
  nb_summary_sample(buf, 16);  // truncating copy
  double back = 0;
  nb_calib_roundtrip(123.5, "GPU-x|driver|nccl", &back);
  int ce = 0;
  for (uint64_t logical : {uint64_t(1) << 20, uint64_t(600) << 20, uint64_t(8) << 30})
    nb_calib_small(7, 1, 512, logical, &ce);
  std::printf("%s\n", failures ? "FAILED" : "OK");
  return failures ? 1 : 0;
}
