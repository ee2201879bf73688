// LD_PRELOAD NCCL interposer for one process driving 1..8 GPUs.
//
// Exports the NCCL C ABI. Grouped AllReduce / AllGather / ReduceScatter /
// Broadcast calls over a clique (communicators created together) are planned
// and run by the sm_100a kernels; every other call, and every call the gates
// reject, goes unchanged to the real libnccl.
//
// Error policy: a CUDA failure before a call's first copy or kernel falls
// back to NCCL; a failure at or after it returns ncclUnhandledCudaError
// (never an NCCL replay over half-written buffers), drains the clique's
// devices and disables the custom paths for the process (poison).
//
// Parity: Layer 5 of the reference (shim/nccl_collectives_shim.cu:1196-1953):
// symbol resolution, version gate, call model, group buffering, pair
// registry, init interposers with prewarm, runtime checks, pair runner,
// GroupEnd with device restore, and the passthrough wrappers.
#include <nvtx3/nvToolsExt.h>
#include <dlfcn.h>

#include <algorithm>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "abi/runtime.h"
#include "core/gate.h"
#include "core/plan.h"
#include "exec/calib.h"
#include "exec/nvls.h"
#include "exec/oneshot.h"
#include "exec/pushred.h"
#include "kernels/kernels.h"
#include "exec/ring.h"

#ifndef NB_BUILD_ID
#define NB_BUILD_ID "dev"
#endif

namespace nb {

const char* build_id() { return NB_BUILD_ID; }

// The calibration cache key: the GPUs and driver, and this build, so a cache
// written by another build (other routes, other kernel shapes) is not used.
std::string build_cache_key(const int* devices, int n) {
  return calib_cache_key(devices, n) + "-b" + build_id();
}

namespace {

struct ExitSummary {
  ~ExitSummary() {
    Runtime& r = rt();
    if (!r.summary.enabled()) return;
    for (const std::string& line : r.summary.render(build_id()))
      std::fprintf(stderr, "[nccl-shim-summary] %s\n", line.c_str());
  }
};

void* g_real_handle = nullptr;

template <typename Fn>
void resolve_one(const char* sym, Fn& fn, bool required) {
  void* p = dlsym(RTLD_NEXT, sym);
  if (!p) {
    if (!g_real_handle) g_real_handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);
    if (!g_real_handle) {
      const char* path = std::getenv("NCCL_B200_REAL_NCCL");
      g_real_handle = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    }
    if (g_real_handle) p = dlsym(g_real_handle, sym);
  }
  fn = reinterpret_cast<Fn>(p);
  if (!fn && required) {
    std::fprintf(stderr, "[nccl-b200] cannot resolve %s in the real libnccl: %s\n", sym, dlerror());
    std::abort();
  }
}

thread_local GroupState g_group;
thread_local unsigned g_init_all_depth = 0;

}  // namespace

Runtime& rt() {
  static Runtime* r = [] {
    Runtime* x = new Runtime();
    x->policy = policy_from_env([](const char* k) { return std::getenv(k); });
    x->summary.set_enabled(x->policy.summary);
    if (!x->fault.configure(x->policy.fault))
      std::fprintf(stderr, "[nccl-b200] ignoring malformed NCCL_B200_FAULT=%s\n", x->policy.fault.c_str());
    x->exec.set_policy(x->policy);
    x->exec.set_summary(&x->summary);
    for (int n = 0; n <= kMaxRanks; ++n) x->eff[n] = x->policy;
    return x;
  }();
  static ExitSummary exit_summary;
  return *r;
}

void Runtime::refresh_policy(int n) {
  if (n < 1 || n > kMaxRanks) return;
  eff[n] = policy;
  for (int k = 0; k < int(Kind::Count); ++k)
    if (!policy.min_bytes_set[k] && calib[n].engage_kib[k] > 0)
      eff[n].min_bytes[k] = std::min(policy.min_bytes[k], size_t(calib[n].engage_kib[k]) << 10);
}

void* real_symbol(const char* name) {
  void* p = dlsym(RTLD_NEXT, name);
  if (!p && g_real_handle) p = dlsym(g_real_handle, name);
  return p;
}

void resolve_all() {
  static std::once_flag once;
  std::call_once(once, [] {
    RealNccl& n = rt().real;
    resolve_one("ncclGetVersion", n.GetVersion, true);
    resolve_one("ncclCommGetAsyncError", n.CommGetAsyncError, true);
    resolve_one("ncclAllReduce", n.AllReduce, true);
    resolve_one("ncclAllGather", n.AllGather, true);
    resolve_one("ncclReduceScatter", n.ReduceScatter, true);
    resolve_one("ncclBroadcast", n.Broadcast, true);
    resolve_one("ncclGroupStart", n.GroupStart, true);
    resolve_one("ncclGroupEnd", n.GroupEnd, true);
    resolve_one("ncclGroupSimulateEnd", n.GroupSimulateEnd, false);
    resolve_one("ncclCommCuDevice", n.CommCuDevice, true);
    resolve_one("ncclCommUserRank", n.CommUserRank, true);
    resolve_one("ncclCommCount", n.CommCount, true);
    resolve_one("ncclCommInitAll", n.CommInitAll, true);
    resolve_one("ncclCommInitRank", n.CommInitRank, true);
    resolve_one("ncclCommInitRankConfig", n.CommInitRankConfig, true);
    resolve_one("ncclCommDestroy", n.CommDestroy, true);
    int version = 0;
    Runtime& r = rt();
    r.nccl_version = n.GetVersion(&version) == ncclSuccess ? version : 0;
    r.nccl_supported = r.nccl_version >= r.policy.min_nccl_version &&
                       r.nccl_version <= r.policy.max_nccl_version;
  });
}

Shares shares_for(Algo a, int n, const CallDesc& c) {
  Runtime& r = rt();
  Shares s = n >= 1 && n <= kMaxRanks && r.calib[n].valid
                 ? shares_from(r.calib[n], a, n, small_message(r.calib[n], logical_bytes(c)))
                 : Shares{};
  // The tiny band's routes move every byte on the SMs.
  if (n >= 2 && n <= kMaxRanks && r.calib[n].valid && tiny_message(r.calib[n], logical_bytes(c))) s = Shares{};
  if (r.policy.host_share_ppm >= 0) s.host_ppm = r.policy.host_share_ppm;
  if (r.policy.ce_share_ppm >= 0) s.ce_ppm = r.policy.ce_share_ppm;
  if (n <= 1) {
    // One rank: the local copy's copy-engine share (policy, else tuned).
    s = Shares{};
    const int k = int(c.kind);
    s.ce_ppm = r.policy.ce_share_ppm >= 0 ? r.policy.ce_share_ppm
                                          : (r.calib[1].valid ? std::max(0, r.calib[1].ce_ppm[k]) : 0);
    return s;
  }
  if (a == Algo::ArNvls) s.host_ppm = s.ce_ppm = 0;
  // Device-resident PreMulSum scalars cannot be applied by the host fold.
  if (c.op == RedOp::PreMulSum && c.scalar_residence == 0) s.host_ppm = 0;
  if (a == Algo::RsPull || a == Algo::RsStaged || a == Algo::ArStaged) s.ce_ppm = 0;
  return s;
}

void prewarm(const int* devices, int n) {
  Runtime& r = rt();
  std::lock_guard<std::mutex> lk(r.exec_mu);
  std::string why;
  if (!r.exec.setup(devices, n, &why)) {
    cudaGetLastError();
    if (r.summary.enabled()) r.summary.note("prewarm_failed " + why);
    return;
  }
  if (n == 1 && r.policy.tune && !r.calib_tried[1]) {
    r.calib_tried[1] = true;
    CalibResult c;
    tune_single(devices[0], r.policy.tune_bytes, &c);
    r.calib[1] = c;
    if (c.valid) {
      char line[160];
      std::snprintf(line, sizeof line, "routes n=1 local copy: sm stream copy%s (ce_ppm=%d, %.1f GB/s)",
                    c.ce_ppm[0] > 0 ? " + copy engine" : " alone", c.ce_ppm[0], c.route_gbs[0]);
      r.summary.note(line);
    }
  }
  if (r.policy.calibrate && n > 1 && !r.calib_tried[n]) {
    r.calib_tried[n] = true;
    const std::string key = build_cache_key(devices, n);
    CalibResult c;
    if (calib_load(r.policy.calib_cache, key, &c)) {
      r.summary.note("calibration loaded from " + r.policy.calib_cache);
    } else {
      c = calibrate(devices, n, r.policy, &r.summary);
      if (c.valid && r.policy.tune) tune_routes(devices, n, r.policy.tune_bytes, &c);
      calib_save(r.policy.calib_cache, key, c);
    }
    r.calib[n] = c;
    r.refresh_policy(n);
    if (c.valid) {
      char line[320];
      std::snprintf(line, sizeof line, "routes n=%d allreduce=%s allgather=%s(ce=%d) reducescatter=%s "
                    "broadcast=%s(ce=%d)", n, algo_name(Algo(c.preferred[0])),
                    algo_name(Algo(c.preferred[1])), c.ce_ppm[1], algo_name(Algo(c.preferred[2])),
                    algo_name(Algo(c.preferred[3])), c.ce_ppm[3]);
      r.summary.note(line);
      if (c.small_below_mib > 0) {
        std::snprintf(line, sizeof line, "routes n=%d below %d MiB: allreduce=%s allgather=%s "
                      "reducescatter=%s broadcast=%s", n, c.small_below_mib,
                      algo_name(Algo(c.small_pref[0])), algo_name(Algo(c.small_pref[1])),
                      algo_name(Algo(c.small_pref[2])), algo_name(Algo(c.small_pref[3])));
        r.summary.note(line);
      }
      if (c.tiny_below_kib > 0) {
        std::snprintf(line, sizeof line, "routes n=%d below %d KiB: allreduce=%s allgather=%s "
                      "reducescatter=%s broadcast=%s", n, c.tiny_below_kib,
                      algo_name(Algo(c.tiny_pref[0])), algo_name(Algo(c.tiny_pref[1])),
                      algo_name(Algo(c.tiny_pref[2])), algo_name(Algo(c.tiny_pref[3])));
        r.summary.note(line);
      }
    }
  }
  Shares s = shares_for(Algo::ArTwoShot, n, CallDesc{});
  const bool nvls = r.policy.nvls != NvlsMode::Off && nvls_supported(devices, n);
  Needs needs = prewarm_needs(n, r.policy, s, nvls);
  // Scratch of the staged routes, sized for the tuned choice.
  for (int k : {int(Kind::AllReduce), int(Kind::ReduceScatter)}) {
    const CalibResult& c = r.calib[n];
    if (n < 2 || (c.preferred[k] != int(Algo::ArStaged) && c.preferred[k] != int(Algo::RsStaged)))
      continue;
    const size_t piece = c.stage_piece_mib[k] > 0 ? size_t(c.stage_piece_mib[k]) << 20 : r.policy.stage_piece;
    const int depth = c.stage_depth[k] > 0 ? c.stage_depth[k] : r.policy.stage_depth;
    needs.temp_bytes = std::max(needs.temp_bytes, size_t(depth) * size_t(n - 1) * piece);
  }
  if (!r.exec.ensure(needs, devices, n, &why)) {
    cudaGetLastError();
    if (r.summary.enabled()) r.summary.note("prewarm_failed " + why);
  }
  r.exec.drain(devices, n);
  size_t nv_bytes = 0, nv_round = 0;
  unsigned nv_bufs = 0;
  if (r.summary.enabled() && nvls_scratch(devices, n, &nv_bytes, &nv_bufs, &nv_round)) {
    char line[160];
    std::snprintf(line, sizeof line, "nvls scratch n=%d: %zu MiB per GPU, %u round buffers of %zu MiB", n,
                  nv_bytes >> 20, nv_bufs, nv_round >> 20);
    r.summary.note(line);
  }
}

namespace {

Outcome run_clique(std::vector<Call>& calls, Reason& reason, bool probe);

// The GroupBackend the group state machine drives in the library.
class RealBackend final : public GroupBackend {
 public:
  int real_group_start() override { return rt().real.GroupStart(); }
  int real_group_end() override { return rt().real.GroupEnd(); }
  int real_simulate_end(void* info) override {
    auto fn = rt().real.GroupSimulateEnd;
    return fn ? fn(static_cast<ncclSimInfo_t*>(info)) : ncclInvalidUsage;
  }
  int forward(const Call& c, Reason reason) override {
    const RealNccl& n = rt().real;
    rt().summary.count_fallback(reason);
    const auto dt = static_cast<ncclDataType_t>(c.nccl_dtype);
    const auto op = static_cast<ncclRedOp_t>(c.nccl_op);
    const auto comm = static_cast<ncclComm_t>(c.comm);
    const auto stream = static_cast<cudaStream_t>(c.stream);
    switch (c.desc.kind) {
      case Kind::AllGather: return n.AllGather(c.sendbuff, c.recvbuff, c.desc.count, dt, comm, stream);
      case Kind::ReduceScatter:
        return n.ReduceScatter(c.sendbuff, c.recvbuff, c.desc.count, dt, op, comm, stream);
      case Kind::Broadcast:
        return n.Broadcast(c.sendbuff, c.recvbuff, c.desc.count, dt, c.desc.root, comm, stream);
      default: return n.AllReduce(c.sendbuff, c.recvbuff, c.desc.count, dt, op, comm, stream);
    }
  }
  bool query(Call& c) override {
    // A registered clique member answers from the registry (its device, rank
    // and size were checked with libnccl when the clique was registered);
    // any other communicator asks libnccl.
    CliqueInfo info;
    if (rt().cliques.lookup(c.comm, &info)) {
      for (int q = 0; q < info.nranks; ++q)
        if (info.comms[q] == c.comm) {
          c.desc.device = info.devices[q];
          c.desc.rank = q;
          c.desc.nranks = info.nranks;
          return true;
        }
    }
    const RealNccl& n = rt().real;
    const auto comm = static_cast<ncclComm_t>(c.comm);
    return n.CommCuDevice(comm, &c.desc.device) == ncclSuccess &&
           n.CommUserRank(comm, &c.desc.rank) == ncclSuccess &&
           n.CommCount(comm, &c.desc.nranks) == ncclSuccess;
  }
  const Policy& policy(int nranks) override { return rt().policy_for(nranks); }
  Outcome run(std::vector<Call>& calls, Reason& reason) override { return run_clique(calls, reason, false); }
};

RealBackend g_backend;
GroupMachine g_machine(g_backend);

// What must hold at run time, per member call, before the clique's own
// routes may touch its buffers: the communicator reports no asynchronous
// error (one that does is dropped from the registry), the call's stream
// belongs to the communicator's GPU, and every buffer the call reads or
// writes passes the buffer rules for the whole clique.
enum class MemberCheck { Ok, AsyncError, ForeignStream, Buffer };

MemberCheck check_member(Runtime& r, const Call& c, const CliqueInfo& info) {
  ncclResult_t async = ncclSuccess;
  if (r.real.CommGetAsyncError(static_cast<ncclComm_t>(c.comm), &async) != ncclSuccess || async != ncclSuccess)
    return MemberCheck::AsyncError;
  const int dev = c.desc.device;
  int owner = -1;
  const bool on_device = cudaSetDevice(dev) == cudaSuccess &&
                         cudaStreamGetDevice(static_cast<cudaStream_t>(c.stream), &owner) == cudaSuccess &&
                         owner == dev;
  if (!on_device) {
    cudaGetLastError();
    return MemberCheck::ForeignStream;
  }
  // A Broadcast non-root's send buffer is never read.
  const bool reads_send = !(c.desc.kind == Kind::Broadcast && c.desc.rank != c.desc.root);
  const bool buffers_ok =
      supported_buffer(c.recvbuff, recv_extent(c.desc), dev, info.devices, info.nranks) &&
      (!reads_send || supported_buffer(c.sendbuff, send_extent(c.desc), dev, info.devices, info.nranks));
  return buffers_ok ? MemberCheck::Ok : MemberCheck::Buffer;
}

bool runtime_checks(Runtime& r, const std::vector<Call>& calls, const CliqueInfo& info) {
  for (const Call& c : calls) {
    const MemberCheck m = check_member(r, c, info);
    if (m == MemberCheck::AsyncError) r.cliques.forget(c.comm);
    if (m != MemberCheck::Ok) return false;
  }
  return true;
}

// Gate, check, plan and execute one clique set. `probe`: a measurement at
// init (measure_crossover), which counts nothing in the summary and leaves
// the first-pass rule alone.
Outcome run_clique(std::vector<Call>& calls, Reason& reason, bool probe) {
  Runtime& r = rt();
  std::lock_guard<std::mutex> lk(r.exec_mu);
  if (!r.poisoned && tma_copy_status() != 0) {
    // An earlier bulk copy gave up on a bounded wait: its output is not to be
    // trusted, and neither are the custom routes from here on.
    r.poisoned = true;
    r.summary.count_timeout();
    std::fprintf(stderr, "[nccl-b200] a bulk copy timed out; custom paths disabled for this process\n");
  }
  CliqueState st;
  st.poisoned = r.poisoned;
  st.nccl_supported = r.nccl_supported;
  st.first_pass_done = r.first_pass_done || probe;
  std::vector<void*> comms;
  std::vector<CallDesc> descs;
  for (const Call& c : calls) {
    comms.push_back(c.comm);
    descs.push_back(c.desc);
  }
  CliqueInfo info;
  st.known_clique = r.cliques.same_clique(comms, &info);
  if (st.known_clique) {
    // The registered devices must be the ones the communicators report.
    for (const Call& c : calls)
      if (c.desc.rank < 0 || c.desc.rank >= info.nranks || info.devices[c.desc.rank] != c.desc.device ||
          info.comms[c.desc.rank] != c.comm)
        st.known_clique = false;
  }
  if (st.known_clique) {
    for (const Call& c : calls)
      if (stream_capturing(static_cast<cudaStream_t>(c.stream), c.desc.device)) st.capturing = true;
    st.nvls_available = r.policy.nvls != NvlsMode::Off && nvls_supported(info.devices, info.nranks);
    if (r.calib[info.nranks].valid)
      for (int k = 0; k < int(Kind::Count); ++k)
        st.preferred[k] = tuned_route(r.calib[info.nranks], k, logical_bytes(descs[0]));
  }
  // A probe measures sizes below the thresholds: the gate applies none.
  Policy unthresholded;
  if (probe) {
    unthresholded = r.policy_for(int(descs.size()));
    for (size_t& m : unthresholded.min_bytes) m = 0;
  }
  const CliqueDecision d = gate_clique(descs, st, probe ? unthresholded : r.policy_for(int(descs.size())));
  reason = d.reason;
  if (d.reason == Reason::FirstPass && !probe) r.first_pass_done = true;
  if (d.algo == Algo::Fallback) return Outcome::Fallback;
  reason = Reason::RuntimeUnsupported;
  if (!runtime_checks(r, calls, info)) return Outcome::Fallback;

  const int n = info.nranks;
  Binding b;
  b.nranks = n;
  const Call* by_rank[kMaxRanks] = {};
  for (const Call& c : calls) by_rank[c.desc.rank] = &c;
  b.fold.dtype = descs[0].dtype;
  b.fold.op = descs[0].op;
  b.fold.nranks = n;
  for (int q = 0; q < n; ++q) {
    const Call& c = *by_rank[q];
    b.device[q] = c.desc.device;
    b.stream[q] = static_cast<cudaStream_t>(c.stream);
    b.send[q] = c.sendbuff;
    b.recv[q] = c.recvbuff;
    b.fold.scalars[q] = c.desc.scalar;
    b.dev_scalar[q] = c.desc.op == RedOp::PreMulSum && c.desc.scalar_residence == 0
                          ? reinterpret_cast<const void*>(c.desc.scalar_ptr)
                          : nullptr;
  }
  // A Broadcast non-root's send pointer is never read.
  const Shares shares = shares_for(d.algo, n, descs[0]);
  Plan plan;
  build_plan(d.algo, describe_clique(descs), r.policy, shares, plan);

  std::string why;
  if (r.fault.fail_setup() || !r.exec.ensure(plan.needs, info.devices, n, &why)) {
    cudaGetLastError();
    if (!why.empty()) r.summary.note(std::string("setup_failed ") + algo_name(d.algo) + ": " + why);
    reason = Reason::SetupFailed;
    return Outcome::Fallback;
  }
  cudaError_t error = cudaSuccess;
  // Optional NVTX range around the submission (NCCL_B200_NVTX=1), named by
  // route, rank count and logical bytes, for timeline tools.
  if (r.policy.nvtx) {
    char label[96];
    std::snprintf(label, sizeof label, "nccl-b200 %s n=%d bytes=%zu", algo_name(d.algo), n,
                  logical_bytes(descs[0]));
    nvtxRangePushA(label);
  }
  const ExecStatus status = r.exec.execute(plan, b, &error, &r.fault);
  if (r.policy.nvtx) nvtxRangePop();
  if (status == ExecStatus::Failed) {
    r.poisoned = true;
    if (error == cudaErrorLaunchTimeout) r.summary.count_timeout();  // a bounded wait ran out
    std::fprintf(stderr,
                 "[nccl-b200] %s: CUDA error after custom work was enqueued (%s); returning "
                 "ncclUnhandledCudaError, custom paths disabled for this process\n",
                 kind_name(descs[0].kind), cudaGetErrorString(error));
    r.exec.drain(info.devices, n);
    cudaGetLastError();
    return Outcome::Error;
  }
  if (status == ExecStatus::Ok) {
    if (!probe)
      r.summary.count_custom(plan.algo, logical_bytes(descs[0]), n, plan.sm_bytes, plan.ce_bytes,
                           plan.host_bytes);
    return Outcome::Handled;
  }
  cudaGetLastError();  // consumed here; NCCL must not see it
  reason = Reason::SubmitFailedEarly;
  return Outcome::Fallback;
}

RedOp to_op(int op, void* comm, CallDesc& d) {
  if (op >= 0 && op < nccl::NumOps) return RedOp(op);  // Sum Prod Max Min Avg
  PreMulScalar s;
  if (rt().cliques.find_premul(comm, op, &s) && s.dtype == d.dtype) {
    d.scalar_residence = s.residence;
    d.scalar = s.value;
    d.scalar_ptr = s.device_ptr;
    return RedOp::PreMulSum;
  }
  return RedOp::Unsupported;
}

Call make_call(Kind kind, const void* sendbuff, void* recvbuff, size_t count, ncclDataType_t dt,
               ncclRedOp_t op, int root, ncclComm_t comm, cudaStream_t stream) {
  Call c;
  c.sendbuff = sendbuff;
  c.recvbuff = recvbuff;
  c.nccl_dtype = int(dt);
  c.nccl_op = int(op);
  c.comm = comm;
  c.stream = stream;
  c.desc.kind = kind;
  c.desc.dtype = dtype_from_nccl(int(dt));
  c.desc.op = reduces(kind) ? to_op(int(op), comm, c.desc) : RedOp::Sum;
  c.desc.count = count;
  c.desc.send = reinterpret_cast<uintptr_t>(sendbuff);
  c.desc.recv = reinterpret_cast<uintptr_t>(recvbuff);
  c.desc.root = root;
  return c;
}

// Device time (max over GPUs, ms per call) of `reps` back-to-back calls of fn.
template <typename Fn>
double time_calls(const int* devices, int n, cudaStream_t* streams, cudaEvent_t* e0, cudaEvent_t* e1,
                  int reps, Fn fn) {
  for (int i = 0; i < n; ++i) {
    cudaSetDevice(devices[i]);
    cudaEventRecord(e0[i], streams[i]);
  }
  for (int k = 0; k < reps; ++k)
    if (!fn()) return -1;
  double worst = 0;
  for (int i = 0; i < n; ++i) {
    cudaSetDevice(devices[i]);
    cudaEventRecord(e1[i], streams[i]);
  }
  for (int i = 0; i < n; ++i) {
    float ms = 0;
    if (cudaEventSynchronize(e1[i]) != cudaSuccess || cudaEventElapsedTime(&ms, e0[i], e1[i]) != cudaSuccess)
      return -1;
    worst = std::max(worst, double(ms));
  }
  return worst / reps;
}

// The interposer runs a clique's call synchronously inside the application's
// call and replays it on libnccl when it falls back, which is only the same
// contract for blocking communicators. A communicator blocks unless the
// environment or its ncclConfig_t says otherwise; a config is trusted only
// when it is large enough to hold the field, carries the initializer's magic
// number, and comes from a libnccl version whose layout is known here.
bool blocking_configuration(const ncclConfig_t* config) {
  if (const char* env = std::getenv("NCCL_COMM_BLOCKING")) {
    if (std::strcmp(env, "1") != 0) return false;
  }
  if (config == nullptr) return true;
  const Policy& p = rt().policy;
  const size_t needed = offsetof(ncclConfig_t, blocking) + sizeof(config->blocking);
  const int version = int(config->version);
  const bool readable = config->size >= needed && config->magic == 0xcafebeef;
  const bool known_layout = version >= p.min_nccl_version && version <= p.max_nccl_version;
  const bool blocks = config->blocking == NCCL_CONFIG_UNDEF_INT || config->blocking == 1;
  return readable && known_layout && blocks;
}

bool distinct_devices(const int* devs, int n) {
  for (int i = 0; i < n; ++i) {
    if (devs[i] < 0) return false;
    for (int j = 0; j < i; ++j)
      if (devs[i] == devs[j]) return false;
  }
  return true;
}

// Register a clique from communicators, checking each one's device, rank and
// async state with libnccl.
bool register_clique(ncclComm_t* comms_by_rank, int n) {
  Runtime& r = rt();
  int devices[kMaxRanks];
  void* comms[kMaxRanks];
  for (int i = 0; i < n; ++i) {
    int rank = -1, count = -1;
    ncclResult_t async = ncclSuccess;
    if (!comms_by_rank[i] || r.real.CommCuDevice(comms_by_rank[i], &devices[i]) != ncclSuccess ||
        r.real.CommUserRank(comms_by_rank[i], &rank) != ncclSuccess || rank != i ||
        r.real.CommCount(comms_by_rank[i], &count) != ncclSuccess || count != n ||
        r.real.CommGetAsyncError(comms_by_rank[i], &async) != ncclSuccess || async != ncclSuccess)
      return false;
    comms[i] = comms_by_rank[i];
  }
  if (!distinct_devices(devices, n)) return false;
  if (r.cliques.add(comms, devices, n) < 0) return false;
  r.summary.note_clique(n, devices);
  return true;
}

void note_initialization(ncclResult_t result, ncclComm_t* output, int nranks, ncclUniqueId id,
                         int rank, bool blocking) {
  if (g_init_all_depth) return;
  Runtime& r = rt();
  if (g_group.depth == 0) {
    // An ungrouped one-rank communicator is a clique of one.
    if (result == ncclSuccess && r.nccl_supported && blocking && output && nranks == 1 && rank == 0 &&
        register_clique(output, 1)) {
      int dev = -1;
      int caller = -1;
      if (r.real.CommCuDevice(*output, &dev) == ncclSuccess && cudaGetDevice(&caller) == cudaSuccess) {
        prewarm(&dev, 1);
        cudaSetDevice(caller);
      }
    }
    return;
  }
  if (!r.nccl_supported || result != ncclSuccess || !blocking || !output || nranks < 1 ||
      nranks > kMaxRanks || rank < 0 || rank >= nranks) {
    g_group.init_only = false;
    return;
  }
  // Inside a group, libnccl fills *output only when the outermost group ends:
  // keep where it will land and register the clique then.
  PendingInit p;
  p.output = reinterpret_cast<void**>(output);
  std::memcpy(p.id, id.internal, sizeof(p.id));
  p.rank = rank;
  p.nranks = nranks;
  g_group.inits.push_back(p);
}

void register_initializations() {
  Runtime& r = rt();
  if (!r.nccl_supported || !g_group.init_only || !inits_form_clique(g_group.inits)) return;
  const int n = int(g_group.inits.size());
  ncclComm_t by_rank[kMaxRanks] = {};
  for (const PendingInit& p : g_group.inits) by_rank[p.rank] = static_cast<ncclComm_t>(*p.output);
  if (!register_clique(by_rank, n)) return;
  CliqueInfo info;
  int caller = -1;
  if (r.cliques.lookup(by_rank[0], &info) && cudaGetDevice(&caller) == cudaSuccess) {
    prewarm(info.devices, n);
    measure_crossover(reinterpret_cast<void* const*>(by_rank), info.devices, n);
    cudaSetDevice(caller);
  }
}

}  // namespace

void measure_crossover(void* const* comms_by_rank, const int* devices, int n) {
  Runtime& r = rt();
  if (n < 2 || n > kMaxRanks || !r.policy.tune || r.crossover_tried[n] || !r.calib[n].valid || r.poisoned)
    return;
  r.crossover_tried[n] = true;
  CalibResult& cal = r.calib[n];
  bool cached = false;
  for (int k = 0; k < int(Kind::Count); ++k) cached = cached || cal.engage_kib[k] > 0;
  if (cached) {  // loaded with the calibration
    r.refresh_policy(n);
    return;
  }
  static const size_t kLadder[] = {64 << 10, 256 << 10, 1 << 20, 4 << 20, 16 << 20};
  constexpr int kSteps = int(sizeof(kLadder) / sizeof(kLadder[0]));
  const size_t top = kLadder[kSteps - 1];
  std::vector<void*> send(size_t(n), nullptr), recv(size_t(n), nullptr);
  std::vector<cudaStream_t> streams(size_t(n), nullptr);
  std::vector<cudaEvent_t> e0(size_t(n), nullptr), e1(size_t(n), nullptr);
  bool ok = true;
  for (int i = 0; i < n && ok; ++i)
    ok = cudaSetDevice(devices[i]) == cudaSuccess && cudaMalloc(&send[size_t(i)], top) == cudaSuccess &&
         cudaMalloc(&recv[size_t(i)], top) == cudaSuccess && cudaMemset(send[size_t(i)], 0, top) == cudaSuccess &&
         cudaStreamCreateWithFlags(&streams[size_t(i)], cudaStreamNonBlocking) == cudaSuccess &&
         cudaEventCreate(&e0[size_t(i)]) == cudaSuccess && cudaEventCreate(&e1[size_t(i)]) == cudaSuccess;
  const RealNccl& nccl = r.real;
  for (int k = 0; ok && k < int(Kind::Count); ++k) {
    if (r.policy.min_bytes_set[k]) continue;
    const Kind kind = Kind(k);
    const bool slots = kind == Kind::AllGather || kind == Kind::ReduceScatter;
    double ours[kSteps], base[kSteps];
    int measured = 0;
    for (int j = 0; j < kSteps && kLadder[j] < r.policy.min_bytes[k]; ++j, ++measured) {
      const size_t logical = kLadder[j];
      const size_t count = (slots ? logical / size_t(n) : logical) / 4;
      auto custom = [&]() {
        std::vector<Call> calls;
        for (int q = 0; q < n; ++q) {
          Call c = make_call(kind, send[size_t(q)], recv[size_t(q)], count, ncclFloat, ncclSum, 0,
                             static_cast<ncclComm_t>(comms_by_rank[q]), streams[size_t(q)]);
          c.desc.device = devices[q];
          c.desc.rank = q;
          c.desc.nranks = n;
          calls.push_back(c);
        }
        Reason why = Reason::None;
        return run_clique(calls, why, true) == Outcome::Handled;
      };
      auto stock = [&]() {
        if (nccl.GroupStart() != ncclSuccess) return false;
        bool good = true;
        for (int q = 0; q < n; ++q) {
          const auto comm = static_cast<ncclComm_t>(comms_by_rank[q]);
          void* sb = send[size_t(q)];
          void* rb = recv[size_t(q)];
          const cudaStream_t st = streams[size_t(q)];
          ncclResult_t res;
          switch (kind) {
            case Kind::AllGather: res = nccl.AllGather(sb, rb, count, ncclFloat, comm, st); break;
            case Kind::ReduceScatter: res = nccl.ReduceScatter(sb, rb, count, ncclFloat, ncclSum, comm, st); break;
            case Kind::Broadcast: res = nccl.Broadcast(sb, rb, count, ncclFloat, 0, comm, st); break;
            default: res = nccl.AllReduce(sb, rb, count, ncclFloat, ncclSum, comm, st); break;
          }
          good = good && res == ncclSuccess;
        }
        return nccl.GroupEnd() == ncclSuccess && good;
      };
      // Warm both (NCCL connects lazily per algorithm), then time 10 calls each.
      ours[j] = time_calls(devices, n, streams.data(), e0.data(), e1.data(), 3, custom);
      base[j] = time_calls(devices, n, streams.data(), e0.data(), e1.data(), 3, stock);
      ours[j] = time_calls(devices, n, streams.data(), e0.data(), e1.data(), 10, custom);
      base[j] = time_calls(devices, n, streams.data(), e0.data(), e1.data(), 10, stock);
      if (ours[j] < 0 || base[j] < 0) {
        ok = false;
        break;
      }
    }
    if (!ok || measured == 0) break;
    // The smallest ladder size from which the routes win at every larger
    // measured size (the threshold itself always engages).
    int from = measured;
    while (from > 0 && ours[from - 1] <= base[from - 1]) --from;
    std::string line = std::string("crossover n=") + std::to_string(n) + " " + kind_name(kind) + ":";
    for (int j = 0; j < measured; ++j) {
      char cell[96];
      std::snprintf(cell, sizeof cell, " %zuKiB ours=%.1fus nccl=%.1fus", kLadder[j] >> 10, ours[j] * 1e3,
                    base[j] * 1e3);
      line += cell;
    }
    if (from < measured) {
      cal.engage_kib[k] = int(kLadder[from] >> 10);
      line += " -> engage from " + std::to_string(kLadder[from] >> 10) + " KiB";
    } else {
      line += " -> keep the threshold";
    }
    r.summary.note(line);
  }
  for (int i = 0; i < n; ++i) {
    if (cudaSetDevice(devices[i]) != cudaSuccess) continue;
    cudaDeviceSynchronize();
    if (send[size_t(i)]) cudaFree(send[size_t(i)]);
    if (recv[size_t(i)]) cudaFree(recv[size_t(i)]);
    if (streams[size_t(i)]) cudaStreamDestroy(streams[size_t(i)]);
    if (e0[size_t(i)]) cudaEventDestroy(e0[size_t(i)]);
    if (e1[size_t(i)]) cudaEventDestroy(e1[size_t(i)]);
  }
  cudaGetLastError();
  r.refresh_policy(n);
  if (!r.policy.calib_cache.empty()) calib_save(r.policy.calib_cache, build_cache_key(devices, n), cal);
}

namespace {

int force_passthrough(bool initialization = false) {
  return g_machine.force_passthrough(g_group, initialization);
}

template <typename Fn>
Fn real_fn(const char* name) {
  resolve_all();
  return reinterpret_cast<Fn>(real_symbol(name));
}

}  // namespace
}  // namespace nb

using namespace nb;

extern "C" {

ncclResult_t ncclGroupStart() {
  resolve_all();
  return ncclResult_t(g_machine.group_start(g_group));
}

ncclResult_t ncclGroupEnd() {
  resolve_all();
  int caller = -1;
  const cudaError_t get_error = cudaGetDevice(&caller);
  const bool outer = g_group.depth == 1;
  const int result = g_machine.group_end(g_group);
  const cudaError_t restore = get_error == cudaSuccess ? cudaSetDevice(caller) : get_error;
  if (outer) {
    if (result == ncclSuccess && restore == cudaSuccess) register_initializations();
    g_group.inits.clear();
  }
  if (restore != cudaSuccess) return result == ncclSuccess ? ncclUnhandledCudaError : ncclResult_t(result);
  return ncclResult_t(result);
}

ncclResult_t ncclGroupSimulateEnd(ncclSimInfo_t* info) {
  resolve_all();
  return ncclResult_t(g_machine.simulate_end(g_group, info));
}

ncclResult_t ncclCommInitAll(ncclComm_t* comms, int ndev, const int* devlist) {
  resolve_all();
  Runtime& r = rt();
  const bool outer = g_group.depth == 0;
  const int prefix = force_passthrough();
  if (prefix != ncclSuccess) return ncclResult_t(prefix);
  int devs[kMaxRanks] = {};
  bool clique = outer && r.nccl_supported && blocking_configuration(nullptr) && ndev >= 1 &&
                ndev <= kMaxRanks;
  if (clique) {
    for (int i = 0; i < ndev; ++i) devs[i] = devlist ? devlist[i] : i;
    clique = distinct_devices(devs, ndev);
  }
  bool restored = true;
  if (clique) {
    int caller = -1;
    if (cudaGetDevice(&caller) == cudaSuccess) {
      prewarm(devs, ndev);
      restored = cudaSetDevice(caller) == cudaSuccess;
    }
  }
  ++g_init_all_depth;
  const ncclResult_t res = r.real.CommInitAll(comms, ndev, devlist);
  --g_init_all_depth;
  if (res == ncclSuccess && clique && restored && comms && register_clique(comms, ndev)) {
    int caller = -1;
    if (cudaGetDevice(&caller) == cudaSuccess) {
      measure_crossover(reinterpret_cast<void* const*>(comms), devs, ndev);
      restored = cudaSetDevice(caller) == cudaSuccess;
    }
  }
  if (res == ncclSuccess && !restored) return ncclUnhandledCudaError;
  return res;
}

ncclResult_t ncclCommInitRank(ncclComm_t* comm, int nranks, ncclUniqueId commId, int rank) {
  resolve_all();
  const int prefix = force_passthrough(true);
  if (prefix != ncclSuccess) return ncclResult_t(prefix);
  const ncclResult_t res = rt().real.CommInitRank(comm, nranks, commId, rank);
  note_initialization(res, comm, nranks, commId, rank, blocking_configuration(nullptr));
  return res;
}

ncclResult_t ncclCommInitRankConfig(ncclComm_t* comm, int nranks, ncclUniqueId commId, int rank,
                                    ncclConfig_t* config) {
  resolve_all();
  const int prefix = force_passthrough(true);
  if (prefix != ncclSuccess) return ncclResult_t(prefix);
  const ncclResult_t res = rt().real.CommInitRankConfig(comm, nranks, commId, rank, config);
  note_initialization(res, comm, nranks, commId, rank, blocking_configuration(config));
  return res;
}

ncclResult_t ncclCommDestroy(ncclComm_t comm) {
  resolve_all();
  const int prefix = force_passthrough();
  rt().cliques.forget(comm);
  return prefix != ncclSuccess ? ncclResult_t(prefix) : rt().real.CommDestroy(comm);
}

ncclResult_t ncclAllReduce(const void* sendbuff, void* recvbuff, size_t count,
                           ncclDataType_t datatype, ncclRedOp_t op, ncclComm_t comm,
                           cudaStream_t stream) {
  resolve_all();
  return ncclResult_t(g_machine.enqueue(
      g_group, make_call(Kind::AllReduce, sendbuff, recvbuff, count, datatype, op, -1, comm, stream)));
}

ncclResult_t ncclAllGather(const void* sendbuff, void* recvbuff, size_t sendcount,
                           ncclDataType_t datatype, ncclComm_t comm, cudaStream_t stream) {
  resolve_all();
  return ncclResult_t(g_machine.enqueue(
      g_group, make_call(Kind::AllGather, sendbuff, recvbuff, sendcount, datatype, ncclSum, -1, comm, stream)));
}

ncclResult_t ncclReduceScatter(const void* sendbuff, void* recvbuff, size_t recvcount,
                               ncclDataType_t datatype, ncclRedOp_t op, ncclComm_t comm,
                               cudaStream_t stream) {
  resolve_all();
  return ncclResult_t(g_machine.enqueue(
      g_group, make_call(Kind::ReduceScatter, sendbuff, recvbuff, recvcount, datatype, op, -1, comm, stream)));
}

ncclResult_t ncclBroadcast(const void* sendbuff, void* recvbuff, size_t count,
                           ncclDataType_t datatype, int root, ncclComm_t comm, cudaStream_t stream) {
  resolve_all();
  return ncclResult_t(g_machine.enqueue(
      g_group, make_call(Kind::Broadcast, sendbuff, recvbuff, count, datatype, ncclSum, root, comm, stream)));
}

// Legacy in-place broadcast, interposed so a buffered clique set cannot be
// reordered around it.
ncclResult_t ncclBcast(void* buff, size_t count, ncclDataType_t datatype, int root, ncclComm_t comm,
                       cudaStream_t stream) {
  return ncclBroadcast(buff, buff, count, datatype, root, comm, stream);
}

// ---- Unsupported operations: visible to the group state machine ----------

#define NB_PASSTHROUGH(ret_expr_name, sig, args)                                        \
  ncclResult_t ret_expr_name sig {                                                      \
    using Fn = decltype(&::ret_expr_name);                                              \
    static const Fn real = real_fn<Fn>(#ret_expr_name);                                 \
    const int prefix = force_passthrough();                                             \
    if (prefix != ncclSuccess) return ncclResult_t(prefix);                             \
    return real ? real args : ncclInvalidUsage;                                         \
  }

#define NB_LIFECYCLE(ret_expr_name, sig, comm_arg, args)                                \
  ncclResult_t ret_expr_name sig {                                                      \
    using Fn = decltype(&::ret_expr_name);                                              \
    static const Fn real = real_fn<Fn>(#ret_expr_name);                                 \
    const int prefix = force_passthrough();                                             \
    rt().cliques.forget(comm_arg);                                                      \
    if (prefix != ncclSuccess) return ncclResult_t(prefix);                             \
    return real ? real args : ncclInvalidUsage;                                         \
  }

NB_PASSTHROUGH(ncclReduce, (const void* s, void* r, size_t n, ncclDataType_t t, ncclRedOp_t o, int root,
                            ncclComm_t c, cudaStream_t st), (s, r, n, t, o, root, c, st))
NB_PASSTHROUGH(ncclSend, (const void* s, size_t n, ncclDataType_t t, int peer, ncclComm_t c,
                          cudaStream_t st), (s, n, t, peer, c, st))
NB_PASSTHROUGH(ncclRecv, (void* r, size_t n, ncclDataType_t t, int peer, ncclComm_t c, cudaStream_t st),
               (r, n, t, peer, c, st))
NB_PASSTHROUGH(ncclAlltoAll, (const void* s, void* r, size_t n, ncclDataType_t t, ncclComm_t c,
                              cudaStream_t st), (s, r, n, t, c, st))
NB_PASSTHROUGH(ncclGather, (const void* s, void* r, size_t n, ncclDataType_t t, int root, ncclComm_t c,
                            cudaStream_t st), (s, r, n, t, root, c, st))
NB_PASSTHROUGH(ncclScatter, (const void* s, void* r, size_t n, ncclDataType_t t, int root, ncclComm_t c,
                             cudaStream_t st), (s, r, n, t, root, c, st))
NB_PASSTHROUGH(ncclCommInitRankScalable, (ncclComm_t* out, int nranks, int rank, int nid,
                                          ncclUniqueId* ids, ncclConfig_t* cfg),
               (out, nranks, rank, nid, ids, cfg))

NB_LIFECYCLE(ncclCommFinalize, (ncclComm_t comm), comm, (comm))
NB_LIFECYCLE(ncclCommAbort, (ncclComm_t comm), comm, (comm))
NB_LIFECYCLE(ncclCommSplit, (ncclComm_t comm, int color, int key, ncclComm_t* out, ncclConfig_t* cfg),
             comm, (comm, color, key, out, cfg))
NB_LIFECYCLE(ncclCommShrink, (ncclComm_t comm, int* excluded, int count, ncclComm_t* out,
                              ncclConfig_t* cfg, int flags), comm, (comm, excluded, count, out, cfg, flags))
NB_LIFECYCLE(ncclCommRegister, (const ncclComm_t comm, void* buff, size_t size, void** handle), comm,
             (comm, buff, size, handle))
NB_LIFECYCLE(ncclCommDeregister, (const ncclComm_t comm, void* handle), comm, (comm, handle))
NB_LIFECYCLE(ncclCommWindowRegister, (ncclComm_t comm, void* buff, size_t size, ncclWindow_t* win,
                                      int flags), comm, (comm, buff, size, win, flags))
NB_LIFECYCLE(ncclCommWindowDeregister, (ncclComm_t comm, ncclWindow_t win), comm, (comm, win))

// PreMulSum: forwarded so NCCL can still run the op on fallback, and
// recorded so the kernels can apply the same per-rank scalar.
ncclResult_t ncclRedOpCreatePreMulSum(ncclRedOp_t* op, void* scalar, ncclDataType_t datatype,
                                      ncclScalarResidence_t residence, ncclComm_t comm) {
  using Fn = decltype(&::ncclRedOpCreatePreMulSum);
  static const Fn real = real_fn<Fn>("ncclRedOpCreatePreMulSum");
  const int prefix = force_passthrough();
  if (prefix != ncclSuccess) return ncclResult_t(prefix);
  if (!real) return ncclInvalidUsage;
  const ncclResult_t res = real(op, scalar, datatype, residence, comm);
  if (res == ncclSuccess && op && scalar) {
    PreMulScalar s;
    s.dtype = dtype_from_nccl(int(datatype));
    s.residence = residence == ncclScalarHostImmediate ? 1 : 0;
    if (s.residence) {
      switch (s.dtype) {
        case DType::F32: s.value = *static_cast<const float*>(scalar); break;
        case DType::F64: s.value = *static_cast<const double*>(scalar); break;
        case DType::F16: s.value = half_to_float(*static_cast<const uint16_t*>(scalar)); break;
        case DType::BF16: s.value = bf16_to_float(*static_cast<const uint16_t*>(scalar)); break;
        default: s.dtype = DType::Unsupported; break;
      }
    } else {
      s.device_ptr = reinterpret_cast<uintptr_t>(scalar);
    }
    if (s.dtype != DType::Unsupported) rt().cliques.add_premul(comm, int(*op), s);
  }
  return res;
}

ncclResult_t ncclRedOpDestroy(ncclRedOp_t op, ncclComm_t comm) {
  using Fn = decltype(&::ncclRedOpDestroy);
  static const Fn real = real_fn<Fn>("ncclRedOpDestroy");
  const int prefix = force_passthrough();
  rt().cliques.drop_premul(comm, int(op));
  if (prefix != ncclSuccess) return ncclResult_t(prefix);
  return real ? real(op, comm) : ncclInvalidUsage;
}

// ---- Introspection for tests and the benchmark (not NCCL ABI) -------------

int nb_custom_calls(int algo) {
  return algo >= 0 && algo < int(Algo::Count) ? int(rt().summary.custom_calls(Algo(algo))) : -1;
}
int nb_fallbacks(int reason) {
  return reason >= 0 && reason < int(Reason::Count) ? int(rt().summary.fallbacks(Reason(reason))) : -1;
}
int nb_poisoned() { return rt().poisoned ? 1 : 0; }
// The blocking-configuration check of InitRankConfig for a config built from
// NCCL's initializer with the given fields overridden (size 0: keep the
// initializer's; null config when use_config is 0). 1 = a blocking
// communicator the interposer may drive.
int nb_blocking_config(int use_config, size_t size, unsigned magic, unsigned version, int blocking) {
  if (!use_config) return blocking_configuration(nullptr) ? 1 : 0;
  ncclConfig_t c = NCCL_CONFIG_INITIALIZER;
  if (size) c.size = size;
  c.magic = magic;
  c.version = version;
  c.blocking = blocking;
  return blocking_configuration(&c) ? 1 : 0;
}
uint64_t nb_kernel_launches() { return rt().exec.kernel_launches(); }
const char* nb_build_id() { return build_id(); }
int nb_nccl_version() {
  resolve_all();
  return rt().nccl_version;
}
// Copies the summary lines, newline-separated, into buf; returns the length.
size_t nb_summary_text(char* buf, size_t cap) {
  std::string all;
  for (const std::string& s : rt().summary.render(build_id())) all += s + "\n";
  if (buf && cap) {
    const size_t n = all.size() < cap - 1 ? all.size() : cap - 1;
    std::memcpy(buf, all.data(), n);
    buf[n] = 0;
  }
  return all.size();
}
int nb_nvls_supported(const int* devices, int n) { return nvls_supported(devices, n) ? 1 : 0; }
unsigned nb_nvls_status(const int* devices, int n) { return nvls_status(devices, n); }
unsigned nb_ring_status(const int* devices, int n) { return ring_status(devices, n); }
unsigned nb_pushred_status(const int* devices, int n) { return pushred_status(devices, n); }
unsigned nb_oneshot_status(const int* devices, int n) { return oneshot_status(devices, n); }
int nb_nvls_trace(const int* devices, int n, int rank, double* out6, int reset) {
  return nvls_trace_read(devices, n, rank, out6, reset != 0);
}
int nb_pushred_trace(const int* devices, int n, int rank, double* out4, int reset) {
  return pushred_trace_read(devices, n, rank, out4, reset != 0);
}
int nb_ring_trace(const int* devices, int n, int rank, double* out2, int reset) {
  return ring_trace_read(devices, n, rank, out2, reset != 0);
}

// The tuned route of a collective kind on cliques of n ranks (-1 untuned).
int nb_route(int n, int kind) {
  if (n < 1 || n > kMaxRanks || kind < 0 || kind >= int(Kind::Count) || !rt().calib[n].valid) return -1;
  return rt().calib[n].preferred[kind];
}

}  // extern "C"
