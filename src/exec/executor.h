// Executor: binds plan ids to CUDA streams, events and buffers for the
// devices of a clique and submits each op in plan order, checking every CUDA
// return code.
//
// Resources are process-wide and created idempotently: per device an
// auxiliary SM stream, a copy-engine stream, per-lane D2H/H2D streams, the
// plan's events and the NUMA-local pinned bounce buffers; per lane a host
// stream (on one device) with its events and the host-reduction output.
// Peer access is enabled between every pair of clique devices at setup, so
// the kernels address the caller's cudaMalloc buffers on every GPU directly.
//
// Status: NotStarted means no copy or kernel was attempted (only event
// records/waits reached the streams, which order but never touch data), so
// NCCL may still run the call; Failed means data work may be in flight.
//
// Parity: Resources / ensure_base / enable_peer_access / ensure_capacity /
// bind_stream / bind_loc / submit / execute_plan of the reference
// (shim/nccl_collectives_shim.cu:853-1194), for a fixed device pair.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "core/exec_loop.h"
#include "core/fault.h"
#include "core/hostreduce.h"
#include "core/plan.h"
#include "core/summary.h"

namespace nb {

struct Binding {
  int nranks = 0;
  int device[kMaxRanks] = {};
  cudaStream_t stream[kMaxRanks] = {};
  const void* send[kMaxRanks] = {};
  void* recv[kMaxRanks] = {};
  FoldParams fold;
  const void* dev_scalar[kMaxRanks] = {};  // PreMulSum device scalars per rank
};

struct DeviceResources {
  int dev = -1;
  bool ready = false;
  int sm_count = 0;
  cudaStream_t aux = nullptr, copy = nullptr, push = nullptr, hub = nullptr;
  cudaStream_t d2h[kMaxLanes] = {}, h2d[kMaxLanes] = {};
  cudaEvent_t input_ready = nullptr, join = nullptr, temp_free = nullptr, gang_done = nullptr;
  cudaEvent_t all_ready = nullptr, all_joined = nullptr;  // recorded on the hub stream
  void* temp = nullptr;  // device scratch of the staged routes
  size_t temp_bytes = 0;
  cudaEvent_t done[size_t(Strm::Count)][kMaxLanes] = {};
  cudaEvent_t d2h_done[kMaxLanes] = {}, h2d_done[kMaxLanes] = {};
  std::vector<cudaEvent_t> phase;
  void* bounce[kMaxLanes] = {};
  size_t bounce_bytes[kMaxLanes] = {};
  size_t bounce_mapped[kMaxLanes] = {};  // nonzero: mmap'd and registered
};

struct LaneResources {
  int dev = -1;
  cudaStream_t host[kMaxLanes] = {};
  cudaEvent_t host_done[kMaxLanes] = {}, lane_free[kMaxLanes] = {};
  void* out[kMaxLanes] = {};
  size_t out_bytes[kMaxLanes] = {};
};

class Executor {
 public:
  // Enable peer access between every pair and create per-device streams
  // and events. Idempotent; safe to retry after a failure.
  bool setup(const int* devices, int n, std::string* why);
  // Allocate what `needs` asks for on these devices.
  bool ensure(const Needs& needs, const int* devices, int n, std::string* why);
  ExecStatus execute(const Plan& plan, const Binding& b, cudaError_t* error, FaultInjector* fault);
  int sm_count(int dev) const;
  void set_policy(const Policy& p) { policy_ = p; }
  void set_summary(Summary* s) { summary_ = s; }
  // Wait for every device of a clique (used on the error path).
  void drain(const int* devices, int n);
  DeviceResources* device(int dev);
  // Kernels this executor launched (tests and the benchmark read it).
  uint64_t kernel_launches() const { return launches_.load(std::memory_order_relaxed); }

 private:
  std::atomic<uint64_t> launches_{0};
  bool ensure_device(int dev, std::string* why);
  bool ensure_lanes(int dev, int lanes, size_t bytes, const int* devices, int n, std::string* why);
  cudaStream_t bind_stream(StreamId s, const Binding& b);
  int stream_device(StreamId s, const Binding& b);
  cudaEvent_t bind_event(EventId e, const Binding& b);
  char* bind_loc(const Loc& l, const Binding& b);
  cudaError_t submit(const PlanOp& op, const Plan& plan, const Binding& b);

  Policy policy_;
  Summary* summary_ = nullptr;
  std::vector<DeviceResources> devs_;
  LaneResources lanes_;
  std::vector<std::pair<int, int>> peer_enabled_;
};

// NUMA-local pinned host memory (mmap + mbind + first touch + move_pages
// check + cudaHostRegister, falling back to cudaHostAlloc). Returns the
// pointer; *mapped is the mapping size when mmap'd (0 for cudaHostAlloc).
void* alloc_pinned_near(int dev, size_t bytes, size_t* mapped, int* target, int* placed,
                        const char** method);
bool free_pinned(void* p, size_t bytes, size_t mapped);
int gpu_numa_node(int dev);

// Runtime safety checks.
bool stream_capturing(cudaStream_t s, int dev);  // unknown counts as capturing
// Device memory on `dev`, one covering non-pool allocation, and reachable
// from every device of the clique (ordinary cudaMalloc with peer access, or
// VMM memory mapped READWRITE for all of them).
bool supported_buffer(const void* ptr, size_t bytes, int dev, const int* devices, int n);

}  // namespace nb
