// C entry points for single-GPU kernel tests and tools. They run the real
// kernels and the real executor with N *virtual* ranks whose buffers all
// live on the current device: every rank binds to the same device and one
// caller stream, so the plan's ops run one after another (no kernel ever
// waits on another). This checks the multi-source reduce / multi-segment
// copy numerics and the planners' byte ranges on a one-GPU box. Host-lane
// shares are not supported here (virtual ranks would share bounce buffers).
#include <cuda_runtime.h>

#include <cstring>

#include "abi/runtime.h"
#include "core/plan.h"
#include "kernels/kernels.h"

using namespace nb;

extern "C" {

int nb_emu_reduce(const void* const* srcs, int nsrc, void* const* dsts, int ndst, uint64_t bytes,
                  int dtype, int op, int nranks, const double* scalars, void* stream) {
  ReduceLaunch r;
  r.nsrc = nsrc;
  r.ndst = ndst;
  r.bytes = size_t(bytes);
  r.fold.dtype = DType(dtype);
  r.fold.op = RedOp(op);
  r.fold.nranks = nranks;
  for (int i = 0; i < nsrc && i < kMaxRanks; ++i) {
    r.src[i] = srcs[i];
    r.fold.scalars[i] = scalars ? scalars[i] : 1.0;
  }
  for (int i = 0; i < ndst && i < kMaxRanks; ++i) r.dst[i] = dsts[i];
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const Policy& p = rt().policy;
  return int(launch_reduce(r, shape_for(r.bytes, sms, p.blocks_per_sm, p.threads),
                           static_cast<cudaStream_t>(stream)));
}

int nb_emu_copy(const void* const* srcs, void* const* dsts, const uint64_t* lens, int nseg, void* stream) {
  CopyLaunch c;
  c.nseg = nseg;
  c.local = true;  // virtual ranks: every buffer is on the current GPU
  c.prefer_tma = rt().policy.local_copy_tma;
  size_t total = 0;
  for (int i = 0; i < nseg && i < kMaxRanks; ++i) {
    c.src[i] = srcs[i];
    c.dst[i] = dsts[i];
    c.len[i] = size_t(lens[i]);
    total += c.len[i];
  }
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const Policy& p = rt().policy;
  return int(launch_copy(c, shape_for(total, sms, p.blocks_per_sm, p.threads),
                         static_cast<cudaStream_t>(stream)));
}

// Runs the full plan of `algo` for `nranks` virtual ranks on the current
// device. Returns 0 on success, -1 on bad arguments, else the CUDA error.
int nb_emu_plan(int algo, int kind, int dtype, int op, int nranks, uint64_t count, int root,
                int ce_ppm, const void* const* sends, void* const* recvs, const double* scalars,
                void* stream) {
  if (nranks < 1 || nranks > kMaxRanks) return -1;
  CliqueDesc d;
  d.kind = Kind(kind);
  d.dtype = DType(dtype);
  d.op = RedOp(op);
  d.nranks = nranks;
  d.count = size_t(count);
  d.bytes = d.count * elem_size(d.dtype);
  d.root = root;
  for (int r = 0; r < nranks; ++r) {
    const char* s = static_cast<const char*>(sends[r]);
    const char* v = static_cast<const char*>(recvs[r]);
    switch (d.kind) {
      case Kind::AllGather: d.in_place[r] = s == v + size_t(r) * d.bytes; break;
      case Kind::ReduceScatter: d.in_place[r] = v == s + size_t(r) * d.bytes; break;
      default: d.in_place[r] = s == v; break;
    }
  }
  Shares sh;
  sh.ce_ppm = ce_ppm;
  Runtime& rtm = rt();
  Plan plan;
  build_plan(Algo(algo), d, rtm.policy, sh, plan);
  // Gang ops (NVLS, the Broadcast chain) wait on their counterparts inside
  // the kernel; virtual ranks on one GPU would run them as separate launches
  // that wait on one another, which is never done.
  for (const PlanOp& op : plan.ops)
    if (op.kind == OpKind::NvlsReduce) return int(cudaErrorNotSupported);
  int dev = 0;
  cudaGetDevice(&dev);
  Binding b;
  b.nranks = nranks;
  b.fold.dtype = d.dtype;
  b.fold.op = d.op;
  b.fold.nranks = nranks;
  for (int r = 0; r < nranks; ++r) {
    b.device[r] = dev;
    b.stream[r] = static_cast<cudaStream_t>(stream);
    b.send[r] = sends[r];
    b.recv[r] = recvs[r];
    b.fold.scalars[r] = scalars ? scalars[r] : 1.0;
  }
  std::lock_guard<std::mutex> lk(rtm.exec_mu);
  std::string why;
  int devs[1] = {dev};
  if (!rtm.exec.ensure(plan.needs, devs, 1, &why)) return int(cudaErrorMemoryAllocation);
  cudaError_t err = cudaSuccess;
  const ExecStatus st = rtm.exec.execute(plan, b, &err, nullptr);
  cudaSetDevice(dev);
  return st == ExecStatus::Ok ? 0 : int(err ? err : cudaErrorUnknown);
}

}  // extern "C"
