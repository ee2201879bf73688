// Routing policy: compile-time defaults plus a small set of runtime overrides
// under one prefix (NCCL_B200_*). Bandwidth shares come from calibration
// (measured at init) unless an override pins them.
//
// Parity: the reference freezes every threshold, chunk size and host-share
// divisor in a constexpr `Tuning` (shim/nccl_collectives_shim.cu:47-105) and
// reads only NCCL_SHIM_SUMMARY and NCCL_COMM_BLOCKING at run time.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>

#include "core/types.h"

namespace nb {

enum class NvlsMode : uint8_t { Off, Auto, On };

struct Policy {
  bool enabled = true;              // NCCL_B200_DISABLE=1 forwards everything
  bool kind_enabled[size_t(Kind::Count)] = {true, true, true, true};
  // Logical-size thresholds (nccl-tests "size": N slots for AG/RS).
  size_t min_bytes[size_t(Kind::Count)] = {32 * kMiB, 32 * kMiB, 32 * kMiB, 32 * kMiB};
  // Set when the environment gave the threshold; otherwise the threshold of
  // a clique size may be lowered to the measured crossover with NCCL.
  bool min_bytes_set[size_t(Kind::Count)] = {false, false, false, false};
  size_t max_message_bytes = size_t(8) << 30;  // enforced logical message cap
  bool first_pass = true;           // first eligible clique call runs on NCCL
  NvlsMode nvls = NvlsMode::Auto;
  int nvls_min_ranks = 4;           // NVLS AllReduce only pays off from 4 ranks
  size_t nvls_round_bytes = 256 * kMiB;  // multicast scratch per GPU (one round)
  int nvls_threads = 768;           // threads per block of the NVLS kernels
  int nvls_movers = 512;            // of those: switch-side workers (the rest copy)
  int nvls_unroll = 4;              // multimem requests in flight per switch-side thread
  bool nvls_trace = false;          // per-block phase timing in the NVLS kernels
  bool nvls_tma = true;             // NVLS copier: TMA bulk pipeline (else SM copy warps)
  bool nvls_ramp = false;           // NVLS AllReduce: ramped first/last rounds from 4 rounds on
  // NVLS round buffers per GPU (at least 3); 0: enough for the largest
  // message (max_bytes / nvls_round_bytes + 2, + 10 with the ramp), so no
  // call reuses one.
  int nvls_buffers = 0;
  bool nvls_strong = true;
  bool nvls_ahead = false;          // NVLS AllReduce: every copy-in before the copy-outs (needs a buffer per round)          // NVLS copier: SM copies with system-scope accesses to the scratch
  bool local_copy_tma = false;      // a large copy within one GPU: TMA bulk copy (else SM stream copy)
  size_t ring_chunk = 256 * 1024;   // Broadcast chain: bytes per block per step
  int hybrid_nvls_ppm = 6000;       // hybrid AllReduce: NVLS share of the message (per 10000)
  int hybrid_blocks = 74;           // hybrid AllReduce: NVLS blocks per GPU (the rest of the SMs
                                    // run the two-shot kernel)
  bool nvtx = false;                // NVTX range per custom submission
  Algo force_algo[size_t(Kind::Count)] = {Algo::Fallback, Algo::Fallback, Algo::Fallback,
                                          Algo::Fallback};  // Fallback = choose
  // Shares in parts per 10000 of the bytes each GPU receives. Negative =
  // take the calibrated value.
  int host_share_ppm = -1;          // pinned-host PCIe lane
  int ce_share_ppm = -1;            // copy-engine peer copies (pure-copy shares)
  int lanes = 4;                    // reusable pinned-host lanes per GPU
  size_t host_piece = 16 * kMiB;    // host-lane staging piece (16-byte multiple)
  size_t min_host_bytes = 16 * kMiB;  // below this per GPU, no host share
  int host_threads = 8;             // CPU threads of the host reduction
  size_t sm_chunk = 512 * kMiB;     // pipelining piece of the SM share
  int blocks_per_sm = 2;
  int threads = 512;
  int bc_pieces = 4;                // scatter/all-gather broadcast pipeline depth
  size_t stage_piece = 128 * kMiB;  // staged routes: bytes per peer per pipelined piece
  int stage_depth = 2;              // staged routes: scratch pieces in flight
  bool calibrate = true;            // measure path bandwidths at init
  bool tune = true;                 // time candidate routes at init, keep the fastest
  size_t tune_bytes = 4 * kGiB;     // message size the route tuning runs at
  std::string calib_cache;          // JSON cache path ("" = none)
  uint64_t device_timeout_ns = 2000000000ull;  // bound of every in-kernel wait
  // Test hook: raise the NVLS barrier targets so that no arrival can meet
  // them; every wait then runs out (bounded) and reports its status.
  unsigned test_nvls_skew = 0;
  bool summary = false;             // NCCL_SHIM_SUMMARY=1 or NCCL_B200_SUMMARY=1
  int min_nccl_version = 21900;     // supported libnccl range (ncclConfig_t layout)
  int max_nccl_version = 22999;
  std::string fault;                // host-side fault injector spec ("" = off)
};

using EnvLookup = std::function<const char*(const char*)>;

// Defaults overridden from the environment. `lookup` is getenv in the
// library and a map in the unit tests.
Policy policy_from_env(const EnvLookup& lookup);
Policy default_policy();

// Parse helpers (exposed for tests): sizes accept K/M/G suffixes.
bool parse_size(const char* s, size_t* out);
bool parse_algo(const char* s, Kind* kind, Algo* algo);

}  // namespace nb
