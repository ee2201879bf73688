#include "core/policy.h"

#include <cstdlib>
#include <cstring>

namespace nb {

Policy default_policy() { return Policy{}; }

bool parse_size(const char* s, size_t* out) {
  if (!s || !*s) return false;
  char* end = nullptr;
  const unsigned long long v = std::strtoull(s, &end, 10);
  if (end == s) return false;
  unsigned long long mul = 1;
  if (*end == 'K' || *end == 'k') mul = 1ull << 10, ++end;
  else if (*end == 'M' || *end == 'm') mul = 1ull << 20, ++end;
  else if (*end == 'G' || *end == 'g') mul = 1ull << 30, ++end;
  if (*end == 'i' || *end == 'B') ++end;
  if (*end == 'B') ++end;
  if (*end) return false;
  if (mul > 1 && v > (~0ull) / mul) return false;
  *out = size_t(v * mul);
  return true;
}

static bool parse_int(const char* s, long long* out) {
  if (!s || !*s) return false;
  char* end = nullptr;
  const long long v = std::strtoll(s, &end, 10);
  if (*end) return false;
  *out = v;
  return true;
}

static bool parse_bool(const char* s, bool* out) {
  if (!s) return false;
  if (!std::strcmp(s, "1") || !std::strcmp(s, "true") || !std::strcmp(s, "on")) return *out = true, true;
  if (!std::strcmp(s, "0") || !std::strcmp(s, "false") || !std::strcmp(s, "off")) return *out = false, true;
  return false;
}

// "allreduce=nvls", "ar=twoshot", "allgather=pull", ...
bool parse_algo(const char* s, Kind* kind, Algo* algo) {
  if (!s) return false;
  const char* eq = std::strchr(s, '=');
  if (!eq) return false;
  const std::string k(s, size_t(eq - s)), a(eq + 1);
  if (k == "allreduce" || k == "ar") *kind = Kind::AllReduce;
  else if (k == "allgather" || k == "ag") *kind = Kind::AllGather;
  else if (k == "reducescatter" || k == "rs") *kind = Kind::ReduceScatter;
  else if (k == "broadcast" || k == "bc") *kind = Kind::Broadcast;
  else return false;
  if (a == "nccl" || a == "fallback") *algo = Algo::Fallback;
  else if (a == "twoshot" && *kind == Kind::AllReduce) *algo = Algo::ArTwoShot;
  else if (a == "oneshot" && *kind == Kind::AllReduce) *algo = Algo::ArOneShot;
  else if (a == "twoshot_ll" && *kind == Kind::AllReduce) *algo = Algo::ArTwoShotLL;
  else if (a == "ll" && *kind == Kind::ReduceScatter) *algo = Algo::RsLL;
  else if (a == "ll" && *kind == Kind::AllGather) *algo = Algo::AgLL;
  else if (a == "ll" && *kind == Kind::Broadcast) *algo = Algo::BcLL;
  else if (a == "nvls" && *kind == Kind::AllReduce) *algo = Algo::ArNvls;
  else if (a == "pull" && *kind == Kind::ReduceScatter) *algo = Algo::RsPull;
  else if (a == "pull" && *kind == Kind::AllGather) *algo = Algo::AgPull;
  else if (a == "pull" && *kind == Kind::Broadcast) *algo = Algo::BcPull;
  else if (a == "scatter" && *kind == Kind::Broadcast) *algo = Algo::BcScatter;
  else if (a == "staged" && *kind == Kind::AllReduce) *algo = Algo::ArStaged;
  else if (a == "staged" && *kind == Kind::ReduceScatter) *algo = Algo::RsStaged;
  else if (a == "chain" && *kind == Kind::Broadcast) *algo = Algo::BcChain;
  else if (a == "nvls" && *kind == Kind::Broadcast) *algo = Algo::BcNvls;
  else if (a == "nvls" && *kind == Kind::AllGather) *algo = Algo::AgNvls;
  else if (a == "nvls" && *kind == Kind::ReduceScatter) *algo = Algo::RsNvls;
  else if (a == "push" && *kind == Kind::AllGather) *algo = Algo::AgPush;
  else if (a == "ring" && *kind == Kind::Broadcast) *algo = Algo::BcRing;
  else if (a == "push" && *kind == Kind::ReduceScatter) *algo = Algo::RsPush;
  else if (a == "push" && *kind == Kind::AllReduce) *algo = Algo::ArPush;
  else if (a == "hybrid" && *kind == Kind::AllReduce) *algo = Algo::ArHybrid;
  else if (a == "hybrid" && *kind == Kind::ReduceScatter) *algo = Algo::RsHybrid;
  else return false;
  return true;
}

Policy policy_from_env(const EnvLookup& env) {
  Policy p;
  bool b = false;
  long long i = 0;
  size_t z = 0;
  if (parse_bool(env("NCCL_B200_DISABLE"), &b)) p.enabled = !b;
  const char* kind_keys[] = {"NCCL_B200_ALLREDUCE", "NCCL_B200_ALLGATHER",
                             "NCCL_B200_REDUCESCATTER", "NCCL_B200_BROADCAST"};
  const char* min_keys[] = {"NCCL_B200_AR_MIN", "NCCL_B200_AG_MIN", "NCCL_B200_RS_MIN",
                            "NCCL_B200_BC_MIN"};
  for (size_t k = 0; k < size_t(Kind::Count); ++k) {
    if (parse_bool(env(kind_keys[k]), &b)) p.kind_enabled[k] = b;
    if (parse_size(env(min_keys[k]), &z)) {
      p.min_bytes[k] = z;
      p.min_bytes_set[k] = true;
    }
  }
  if (parse_size(env("NCCL_B200_MAX_BYTES"), &z)) p.max_message_bytes = z;
  if (parse_bool(env("NCCL_B200_FIRST_PASS"), &b)) p.first_pass = b;
  if (const char* s = env("NCCL_B200_NVLS")) {
    if (!std::strcmp(s, "0") || !std::strcmp(s, "off")) p.nvls = NvlsMode::Off;
    else if (!std::strcmp(s, "1") || !std::strcmp(s, "on")) p.nvls = NvlsMode::On;
    else p.nvls = NvlsMode::Auto;
  }
  if (parse_int(env("NCCL_B200_NVLS_MIN_RANKS"), &i) && i >= 1) p.nvls_min_ranks = int(i);
  if (parse_size(env("NCCL_B200_NVLS_ROUND"), &z) && z >= kMiB) p.nvls_round_bytes = z;
  if (parse_int(env("NCCL_B200_NVLS_BUFFERS"), &i) && i >= 3 && i <= 65536) p.nvls_buffers = int(i);
  if (parse_int(env("NCCL_B200_NVLS_MOVERS"), &i) && i >= 128 && i <= 736 && i % 32 == 0)
    p.nvls_movers = int(i);
  if (parse_int(env("NCCL_B200_NVLS_UNROLL"), &i) && (i == 4 || i == 8)) p.nvls_unroll = int(i);
  if (parse_bool(env("NCCL_B200_NVLS_TRACE"), &b)) p.nvls_trace = b;
  if (parse_bool(env("NCCL_B200_NVLS_TMA"), &b)) p.nvls_tma = b;
  if (parse_bool(env("NCCL_B200_NVLS_RAMP"), &b)) p.nvls_ramp = b;
  if (parse_bool(env("NCCL_B200_NVLS_STRONG"), &b)) p.nvls_strong = b;
  if (parse_bool(env("NCCL_B200_NVLS_AHEAD"), &b)) p.nvls_ahead = b;
  if (const char* v = env("NCCL_B200_LOCAL_COPY")) {
    if (std::strcmp(v, "tma") == 0) p.local_copy_tma = true;
    else if (std::strcmp(v, "sm") == 0) p.local_copy_tma = false;
  }
  if (parse_size(env("NCCL_B200_RING_CHUNK"), &z) && z >= 4096 && z <= (64u << 20) && z % 32 == 0)
    p.ring_chunk = z;
  if (parse_int(env("NCCL_B200_HYBRID_NVLS_PPM"), &i) && i >= 1000 && i <= 9000) p.hybrid_nvls_ppm = int(i);
  if (parse_int(env("NCCL_B200_HYBRID_BLOCKS"), &i) && i >= 8 && i <= 1024) p.hybrid_blocks = int(i);
  if (parse_bool(env("NCCL_B200_NVTX"), &b)) p.nvtx = b;
  if (parse_int(env("NCCL_B200_NVLS_THREADS"), &i) && (i == 512 || i == 640 || i == 768))
    p.nvls_threads = int(i);
  if (const char* s = env("NCCL_B200_ALGO")) {
    // Comma-separated list of kind=algo.
    std::string all(s);
    size_t pos = 0;
    while (pos <= all.size()) {
      const size_t comma = all.find(',', pos);
      const std::string item = all.substr(pos, comma == std::string::npos ? std::string::npos : comma - pos);
      Kind k;
      Algo a;
      if (parse_algo(item.c_str(), &k, &a)) p.force_algo[size_t(k)] = a;
      if (comma == std::string::npos) break;
      pos = comma + 1;
    }
  }
  if (parse_int(env("NCCL_B200_HOST_SHARE_PPM"), &i) && i >= -1 && i <= 5000) p.host_share_ppm = int(i);
  if (parse_int(env("NCCL_B200_CE_SHARE_PPM"), &i) && i >= -1 && i <= 10000) p.ce_share_ppm = int(i);
  if (parse_int(env("NCCL_B200_LANES"), &i) && i >= 1 && i <= kMaxLanes) p.lanes = int(i);
  if (parse_size(env("NCCL_B200_HOST_PIECE"), &z) && z >= 4096 && z % 16 == 0) p.host_piece = z;
  if (parse_size(env("NCCL_B200_MIN_HOST_BYTES"), &z)) p.min_host_bytes = z;
  if (parse_int(env("NCCL_B200_HOST_THREADS"), &i) && i >= 1 && i <= 64) p.host_threads = int(i);
  if (parse_size(env("NCCL_B200_SM_CHUNK"), &z) && z >= kMiB && z % 16 == 0) p.sm_chunk = z;
  if (parse_int(env("NCCL_B200_BLOCKS_PER_SM"), &i) && i >= 1 && i <= 8) p.blocks_per_sm = int(i);
  if (parse_int(env("NCCL_B200_THREADS"), &i) && (i == 128 || i == 256 || i == 512 || i == 1024))
    p.threads = int(i);
  if (parse_int(env("NCCL_B200_BC_PIECES"), &i) && i >= 1 && i <= 64) p.bc_pieces = int(i);
  if (parse_size(env("NCCL_B200_STAGE_PIECE"), &z) && z >= 64 * 1024 && z % 16 == 0) p.stage_piece = z;
  if (parse_int(env("NCCL_B200_STAGE_DEPTH"), &i) && i >= 1 && i <= 8) p.stage_depth = int(i);
  if (parse_bool(env("NCCL_B200_CALIBRATE"), &b)) p.calibrate = b;
  if (parse_bool(env("NCCL_B200_TUNE"), &b)) p.tune = b;
  if (parse_size(env("NCCL_B200_TUNE_BYTES"), &z) && z >= kMiB) p.tune_bytes = z;
  if (const char* s = env("NCCL_B200_CALIB_CACHE")) p.calib_cache = s;
  if (parse_int(env("NCCL_B200_TIMEOUT_MS"), &i) && i >= 1) p.device_timeout_ns = uint64_t(i) * 1000000ull;
  if (parse_int(env("NCCL_B200_TEST_NVLS_SKEW"), &i) && i >= 0) p.test_nvls_skew = unsigned(i);
  const char* summary = env("NCCL_SHIM_SUMMARY");
  if (summary && !std::strcmp(summary, "1")) p.summary = true;
  if (parse_bool(env("NCCL_B200_SUMMARY"), &b)) p.summary = b;
  if (const char* s = env("NCCL_B200_FAULT")) p.fault = s;
  return p;
}

}  // namespace nb
