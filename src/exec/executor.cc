#include "exec/executor.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "exec/nvls.h"
#include "exec/oneshot.h"
#include "exec/pushred.h"
#include "exec/ring.h"
#include "kernels/kernels.h"

namespace nb {

namespace {

bool make_stream(cudaStream_t& s) {
  if (s) return true;
  cudaStream_t created = nullptr;
  if (cudaStreamCreateWithFlags(&created, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  s = created;
  return true;
}

bool make_event(cudaEvent_t& e) {
  if (e) return true;
  cudaEvent_t created = nullptr;
  if (cudaEventCreateWithFlags(&created, cudaEventDisableTiming) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  e = created;
  return true;
}

// Payload of one host-lane reduction, owned by the callback.
struct HostFoldTask {
  FoldParams fold;
  const void* src[kMaxRanks];
  int nsrc;
  void* dst;
  size_t bytes;
  int threads;
};

void CUDART_CB host_fold_cb(void* arg) {
  HostFoldTask* t = static_cast<HostFoldTask*>(arg);
  host_fold_parallel(t->fold, t->src, t->nsrc, t->dst, t->bytes, t->threads);
  delete t;
}

}  // namespace

DeviceResources* Executor::device(int dev) {
  if (dev < 0) return nullptr;
  if (size_t(dev) >= devs_.size()) devs_.resize(size_t(dev) + 1);
  return &devs_[size_t(dev)];
}

int Executor::sm_count(int dev) const {
  return dev >= 0 && size_t(dev) < devs_.size() ? devs_[size_t(dev)].sm_count : 0;
}

bool Executor::ensure_device(int dev, std::string* why) {
  DeviceResources& r = *device(dev);
  if (r.ready) return true;
  r.dev = dev;
  if (cudaSetDevice(dev) != cudaSuccess) {
    cudaGetLastError();
    if (why) *why = "cudaSetDevice failed";
    return false;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    if (why) *why = "SM count query failed";
    return false;
  }
  r.sm_count = sms;
  bool ok = make_stream(r.aux) && make_stream(r.copy) && make_stream(r.push) && make_stream(r.hub) &&
            make_event(r.input_ready) && make_event(r.join) && make_event(r.temp_free) &&
            make_event(r.gang_done) && make_event(r.all_ready) && make_event(r.all_joined);
  for (int l = 0; ok && l < kMaxLanes; ++l)
    ok = make_stream(r.d2h[l]) && make_stream(r.h2d[l]) && make_event(r.d2h_done[l]) &&
         make_event(r.h2d_done[l]);
  for (size_t k = 0; ok && k < size_t(Strm::Count); ++k)
    for (int l = 0; ok && l < kMaxLanes; ++l) ok = make_event(r.done[k][l]);
  if (!ok) {
    if (why) *why = "stream/event creation failed";
    return false;
  }
  r.ready = true;
  return true;
}

bool Executor::setup(const int* devices, int n, std::string* why) {
  for (int i = 0; i < n; ++i)
    if (!ensure_device(devices[i], why)) return false;
  // The bulk copy's status word is pinned host memory: allocate it here, at
  // init, rather than at a first copy that may run beside a stream capture.
  if (!tma_copy_prepare()) {
    if (why) *why = "bulk copy status word";
    return false;
  }
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < n; ++j) {
      if (i == j) continue;
      const int a = devices[i], b = devices[j];
      bool done = false;
      for (const auto& p : peer_enabled_) done |= p.first == a && p.second == b;
      if (done) continue;
      int can = 0;
      if (cudaDeviceCanAccessPeer(&can, a, b) != cudaSuccess || !can) {
        cudaGetLastError();
        if (why) *why = "no peer access between clique devices";
        return false;
      }
      if (cudaSetDevice(a) != cudaSuccess) {
        cudaGetLastError();
        return false;
      }
      const cudaError_t e = cudaDeviceEnablePeerAccess(b, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
      } else if (e != cudaSuccess) {
        cudaGetLastError();
        if (why) *why = std::string("cudaDeviceEnablePeerAccess: ") + cudaGetErrorString(e);
        return false;
      }
      peer_enabled_.push_back({a, b});
    }
  return true;
}

bool Executor::ensure_lanes(int dev, int lanes, size_t bytes, const int* devices, int n,
                            std::string* why) {
  if (lanes_.dev < 0) lanes_.dev = dev;
  if (cudaSetDevice(lanes_.dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  for (int l = 0; l < lanes; ++l)
    if (!make_stream(lanes_.host[l]) || !make_event(lanes_.host_done[l]) ||
        !make_event(lanes_.lane_free[l])) {
      if (why) *why = "lane stream/event creation failed";
      return false;
    }
  // Growing a buffer first drains every device that may still use it.
  bool drained = false;
  auto drain_all = [&] {
    if (drained) return true;
    for (size_t d = 0; d < devs_.size(); ++d)
      if (devs_[d].ready && (cudaSetDevice(int(d)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)) {
        cudaGetLastError();
        return false;
      }
    drained = true;
    return true;
  };
  for (int l = 0; l < lanes; ++l) {
    if (lanes_.out_bytes[l] >= bytes) continue;
    if (lanes_.out[l]) {
      if (!drain_all() || cudaFreeHost(lanes_.out[l]) != cudaSuccess) return false;
      lanes_.out[l] = nullptr;
      lanes_.out_bytes[l] = 0;
    }
    void* p = nullptr;
    if (cudaSetDevice(lanes_.dev) != cudaSuccess || cudaHostAlloc(&p, bytes, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      if (why) *why = "pinned host-out allocation failed";
      return false;
    }
    lanes_.out[l] = p;
    lanes_.out_bytes[l] = bytes;
  }
  for (int i = 0; i < n; ++i) {
    DeviceResources& r = *device(devices[i]);
    for (int l = 0; l < lanes; ++l) {
      if (r.bounce_bytes[l] >= bytes) continue;
      if (r.bounce[l]) {
        if (!drain_all() || !free_pinned(r.bounce[l], r.bounce_bytes[l], r.bounce_mapped[l])) return false;
        r.bounce[l] = nullptr;
        r.bounce_bytes[l] = r.bounce_mapped[l] = 0;
      }
      int target = -1, placed = -1;
      const char* method = "none";
      size_t mapped = 0;
      void* p = alloc_pinned_near(devices[i], bytes, &mapped, &target, &placed, &method);
      if (!p) {
        if (why) *why = "pinned bounce allocation failed";
        return false;
      }
      r.bounce[l] = p;
      r.bounce_bytes[l] = bytes;
      r.bounce_mapped[l] = mapped;
      if (summary_) summary_->note_placement(devices[i], l, target, placed, method);
    }
  }
  return true;
}

bool Executor::ensure(const Needs& needs, const int* devices, int n, std::string* why) {
  if (!setup(devices, n, why)) return false;
  for (int i = 0; i < n; ++i) {
    DeviceResources& r = *device(devices[i]);
    if (cudaSetDevice(devices[i]) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    while (r.phase.size() < needs.phase_events) {
      cudaEvent_t e = nullptr;
      if (!make_event(e)) {
        if (why) *why = "event creation failed";
        return false;
      }
      r.phase.push_back(e);
    }
    if (needs.temp_bytes > r.temp_bytes) {
      // Growing the scratch first drains this device (work may still read it).
      if (r.temp && (cudaDeviceSynchronize() != cudaSuccess || cudaFree(r.temp) != cudaSuccess)) {
        cudaGetLastError();
        if (why) *why = "scratch release failed";
        return false;
      }
      r.temp = nullptr;
      r.temp_bytes = 0;
      void* p = nullptr;
      if (cudaMalloc(&p, needs.temp_bytes) != cudaSuccess) {
        cudaGetLastError();
        if (why) *why = "scratch allocation failed";
        return false;
      }
      r.temp = p;
      r.temp_bytes = needs.temp_bytes;
    }
  }
  if (needs.lanes > 0 && !ensure_lanes(devices[0], needs.lanes, needs.bounce_bytes, devices, n, why))
    return false;
  if (needs.nvls_bytes > 0) {
    // Enough round buffers for the largest message (plus partial rounds, and
    // the ramped schedule's eight short rounds when it is on), so that no
    // call reuses one, unless the environment set a number.
    const size_t extra = policy_.nvls_ramp ? 10 : 2;
    const int nbuf = policy_.nvls_buffers > 0
                         ? policy_.nvls_buffers
                         : int(std::min<size_t>(policy_.max_message_bytes / needs.nvls_bytes + extra, 1 << 16));
    if (!nvls_ensure(devices, n, needs.nvls_bytes, nbuf, why)) return false;
  }
  if (needs.ring && !ring_ensure(devices, n, why)) return false;
  if (needs.pushred && !pushred_ensure(devices, n, why)) return false;
  if (needs.oneshot && !oneshot_ensure(devices, n, why)) return false;
  return true;
}

cudaStream_t Executor::bind_stream(StreamId s, const Binding& b) {
  if (s.kind == Strm::Caller) return b.stream[s.dev];
  if (s.kind == Strm::Host) return lanes_.host[s.lane];
  DeviceResources& r = *device(b.device[s.dev]);
  switch (s.kind) {
    case Strm::Aux: return r.aux;
    case Strm::Copy: return r.copy;
    case Strm::Push: return r.push;
    case Strm::Hub: return r.hub;
    case Strm::D2H: return r.d2h[s.lane];
    case Strm::H2D: return r.h2d[s.lane];
    default: return nullptr;
  }
}

int Executor::stream_device(StreamId s, const Binding& b) {
  return s.kind == Strm::Host ? lanes_.dev : b.device[s.dev];
}

cudaEvent_t Executor::bind_event(EventId e, const Binding& b) {
  switch (e.kind) {
    case Ev::HostDone: return lanes_.host_done[e.lane];
    case Ev::LaneFree: return lanes_.lane_free[e.lane];
    default: break;
  }
  DeviceResources& r = *device(b.device[e.dev]);
  switch (e.kind) {
    case Ev::InputReady: return r.input_ready;
    case Ev::Join: return r.join;
    case Ev::TempFree: return r.temp_free;
    case Ev::GangDone: return r.gang_done;
    case Ev::AllReady: return r.all_ready;
    case Ev::AllJoined: return r.all_joined;
    case Ev::Phase: return e.index < r.phase.size() ? r.phase[e.index] : nullptr;
    case Ev::Done: return r.done[e.index][e.lane];
    case Ev::D2HDone: return r.d2h_done[e.lane];
    case Ev::H2DDone: return r.h2d_done[e.lane];
    default: return nullptr;
  }
}

char* Executor::bind_loc(const Loc& l, const Binding& b) {
  switch (l.buf) {
    case Buf::Send: return const_cast<char*>(static_cast<const char*>(b.send[l.dev])) + l.off;
    case Buf::Recv: return static_cast<char*>(b.recv[l.dev]) + l.off;
    case Buf::Bounce: return static_cast<char*>(device(b.device[l.dev])->bounce[l.lane]) + l.off;
    case Buf::HostOut: return static_cast<char*>(lanes_.out[l.lane]) + l.off;
    case Buf::Temp: return static_cast<char*>(device(b.device[l.dev])->temp) + l.off;
    default: return nullptr;
  }
}

cudaError_t Executor::submit(const PlanOp& op, const Plan& plan, const Binding& b) {
  const cudaStream_t s = bind_stream(op.stream, b);
  const int dev = stream_device(op.stream, b);
  switch (op.kind) {
    case OpKind::Record: {
      cudaEvent_t e = bind_event(op.event, b);
      return e ? cudaEventRecord(e, s) : cudaErrorInvalidResourceHandle;
    }
    case OpKind::Wait: {
      cudaEvent_t e = bind_event(op.event, b);
      return e ? cudaStreamWaitEvent(s, e, 0) : cudaErrorInvalidResourceHandle;
    }
    case OpKind::CeCopy:
      return cudaMemcpyAsync(bind_loc(op.dst[0], b), bind_loc(op.src[0], b), op.bytes,
                             cudaMemcpyDefault, s);
    case OpKind::SmCopy: {
      CopyLaunch c;
      c.nseg = op.nsrc;
      c.local = true;
      c.prefer_tma = policy_.local_copy_tma;
      const auto on_device = [&](const Loc& l) {
        return (l.buf == Buf::Send || l.buf == Buf::Recv || l.buf == Buf::Temp) &&
               b.device[l.dev] == b.device[op.stream.dev];
      };
      for (int i = 0; i < op.nsrc; ++i) {
        c.src[i] = bind_loc(op.src[i], b);
        c.dst[i] = bind_loc(op.dst[i], b);
        c.len[i] = op.len[i];
        c.local = c.local && on_device(op.src[i]) && on_device(op.dst[i]);
      }
      launches_.fetch_add(1, std::memory_order_relaxed);
      return launch_copy(c, shape_for(op.bytes, sm_count(dev), policy_.blocks_per_sm, policy_.threads), s);
    }
    case OpKind::SmReduce: {
      ReduceLaunch r;
      r.nsrc = op.nsrc;
      r.ndst = op.ndst;
      r.bytes = op.bytes;
      r.fold = b.fold;
      for (int i = 0; i < op.nsrc; ++i) {
        r.src[i] = bind_loc(op.src[i], b);
        // Sources are in rank order for every reduction plan.
        if (op.src[i].buf == Buf::Send) {
          r.fold.scalars[i] = b.fold.scalars[op.src[i].dev];
          r.dev_scalar[i] = b.dev_scalar[op.src[i].dev];
        }
      }
      for (int i = 0; i < op.ndst; ++i) r.dst[i] = bind_loc(op.dst[i], b);
      launches_.fetch_add(1, std::memory_order_relaxed);
      return launch_reduce(r, shape_for(op.bytes, sm_count(dev), policy_.blocks_per_sm, policy_.threads), s);
    }
    case OpKind::HostReduce: {
      HostFoldTask* t = new HostFoldTask();
      t->fold = b.fold;
      t->nsrc = op.nsrc;
      for (int i = 0; i < op.nsrc; ++i) t->src[i] = bind_loc(op.src[i], b);
      t->dst = bind_loc(op.dst[0], b);
      t->bytes = op.bytes;
      t->threads = policy_.host_threads;
      const cudaError_t e = cudaLaunchHostFunc(s, host_fold_cb, t);
      if (e != cudaSuccess) delete t;
      return e;
    }
    case OpKind::NvlsReduce:
      launches_.fetch_add(1, std::memory_order_relaxed);
      if (plan.algo == Algo::BcRing) return ring_launch(op, plan, b, policy_, s);
      if (plan.algo == Algo::RsPush || plan.algo == Algo::ArPush) return pushred_launch(op, plan, b, policy_, s);
      if (plan.algo == Algo::ArOneShot || plan.algo == Algo::ArTwoShotLL || plan.algo == Algo::RsLL ||
          plan.algo == Algo::AgLL || plan.algo == Algo::BcLL)
        return oneshot_launch(op, plan, b, policy_, s);
      return nvls_launch(op, plan, b, policy_, s, dev);
    default:
      return cudaErrorNotSupported;
  }
}

ExecStatus Executor::execute(const Plan& plan, const Binding& b, cudaError_t* error,
                             FaultInjector* fault) {
  int current = -1;
  int code = 0;
  const ExecStatus st = run_plan_ops(
      plan,
      [&](const PlanOp& op, size_t) -> int {
        const int dev = stream_device(op.stream, b);
        if (dev != current) {
          const cudaError_t e = cudaSetDevice(dev);
          if (e != cudaSuccess) return int(e);
          current = dev;
        }
        return int(submit(op, plan, b));
      },
      fault, int(cudaErrorUnknown), &code, nullptr);
  if (st != ExecStatus::Ok) *error = cudaError_t(code);
  return st;
}

void Executor::drain(const int* devices, int n) {
  for (int i = 0; i < n; ++i)
    if (cudaSetDevice(devices[i]) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
      cudaGetLastError();
}

}  // namespace nb
