// Process-wide interposer runtime: the real libnccl entry points, the policy,
// the clique registry, the executor, the exit summary and the error policy.
#pragma once

#include <nccl.h>

#include <mutex>
#include <string>

#include "core/calib_model.h"
#include "core/clique.h"
#include "core/fault.h"
#include "core/group.h"
#include "core/policy.h"
#include "core/summary.h"
#include "exec/executor.h"

namespace nb {

struct RealNccl {
  decltype(&::ncclGetVersion) GetVersion = nullptr;
  decltype(&::ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&::ncclAllReduce) AllReduce = nullptr;
  decltype(&::ncclAllGather) AllGather = nullptr;
  decltype(&::ncclReduceScatter) ReduceScatter = nullptr;
  decltype(&::ncclBroadcast) Broadcast = nullptr;
  decltype(&::ncclGroupStart) GroupStart = nullptr;
  decltype(&::ncclGroupEnd) GroupEnd = nullptr;
  decltype(&::ncclGroupSimulateEnd) GroupSimulateEnd = nullptr;
  decltype(&::ncclCommCuDevice) CommCuDevice = nullptr;
  decltype(&::ncclCommUserRank) CommUserRank = nullptr;
  decltype(&::ncclCommCount) CommCount = nullptr;
  decltype(&::ncclCommInitAll) CommInitAll = nullptr;
  decltype(&::ncclCommInitRank) CommInitRank = nullptr;
  decltype(&::ncclCommInitRankConfig) CommInitRankConfig = nullptr;
  decltype(&::ncclCommDestroy) CommDestroy = nullptr;
};

struct Runtime {
  RealNccl real;
  Policy policy;
  Summary summary;
  CliqueRegistry cliques;
  Executor exec;
  FaultInjector fault;
  std::mutex exec_mu;
  bool poisoned = false;
  bool first_pass_done = false;
  bool nccl_supported = false;
  int nccl_version = 0;
  // Path rates and tuned routes per clique size (measured at the first
  // prewarm of a clique of that size, or loaded from the cache).
  CalibResult calib[kMaxRanks + 1];
  bool calib_tried[kMaxRanks + 1] = {};
  bool crossover_tried[kMaxRanks + 1] = {};
  // The policy in force per clique size: `policy` with the thresholds the
  // environment left unset replaced by the measured crossover with NCCL.
  Policy eff[kMaxRanks + 1];
  const Policy& policy_for(int n) const { return n >= 1 && n <= kMaxRanks ? eff[n] : policy; }
  void refresh_policy(int n);
};

// Time every candidate route on the clique's GPUs at `bytes` and record the
// fastest per collective kind (abi/tune.cc).
void tune_routes(const int* devices, int n, size_t bytes, CalibResult* out);
// One-rank cliques: time the local copy (the SM stream copy kernel alone and
// beside copy-engine shares) at `bytes` and keep the fastest copy-engine
// share for every kind (abi/tune.cc).
void tune_single(int device, size_t bytes, CalibResult* out);

Runtime& rt();
// After the communicators of a clique exist: time the tuned routes against
// libnccl on a size ladder below the thresholds and lower each kind's
// threshold to the size from which the routes win (interposer.cc).
void measure_crossover(void* const* comms_by_rank, const int* devices, int n);
// Resolve the real libnccl once (dlsym RTLD_NEXT, then the loaded
// libnccl.so.2, then NCCL_B200_REAL_NCCL or libnccl.so.2 by name); aborts
// with a message if a required symbol is missing.
void resolve_all();
// Any other libnccl symbol by name (nullptr if absent).
void* real_symbol(const char* name);

// Prewarm a clique's devices (peer access, streams, events, host lanes,
// calibration) before the application can start a graph capture.
void prewarm(const int* devices, int n);

// Shares for an algorithm on n ranks: policy overrides, else calibration.
Shares shares_for(Algo a, int n, const CallDesc& c);

const char* build_id();

}  // namespace nb
