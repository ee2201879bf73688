// Low-latency collectives over peer memory, synchronized inside the kernel
// instead of by cross-device events: one-shot and two-shot AllReduce,
// ReduceScatter (slot r of every input folded into rank r's output),
// AllGather (rank r's input stored into slot r of every output) and
// Broadcast (every rank copies the root's input); the last two are
// one-source copies that move 32-bit words unchanged.
//
// One kernel per rank, launched on the caller's own stream with nothing
// around it. Block b of every rank's kernel:
//   1. arrives: stores the call's epoch into word (b, r) of every peer's
//      arrive table (P2P stores after a system-scope release fence) -- this
//      rank's stream has reached the call, so its whole input is ready;
//   2. waits until every peer's block b arrived here (relaxed polls of this
//      GPU's own table, then one acquire fence);
//   3. folds its share of its range (grid-stride 16/32-byte vectors) from
//      its sources in rank order -- its own from HBM, the peers' over
//      NVLink -- with fp32 accumulation. One-shot: the range is the whole
//      message and the result goes to this rank's output only. Two-shot:
//      the range is slice r and the result goes to slice r of every rank's
//      output (P2P stores), so each GPU moves 2(N-1)/N of the message
//      instead of N-1 times it. The other kinds: see the launch;
//   4. departs: stores the epoch into the peers' depart tables, and waits
//      until every peer's block b departed, i.e. finished reading this
//      rank's input and (two-shot) writing this rank's output; only then may
//      this rank's stream go on (the caller may reuse both buffers).
// A call thus costs N kernel launches and no event traffic: the two
// cross-device event fans of an event-ordered plan (every stream waiting on
// every peer before and after) are what bound small messages otherwise.
//
// Calls on the same streams need no further ordering: a rank's next kernel
// starts after its previous one, which ended only after every peer had
// departed from it; arrive and depart use separate tables, so a peer still
// waiting in its depart phase sees no stray arrival. When a call comes on
// streams other than the previous call's (another stream of the same
// clique, or a clique over the same GPUs), each rank's stream first waits
// for the previous call's kernels on every GPU (one event per GPU,
// recorded after every launch).
//
// Every wait is bounded by %globaltimer: on expiry the kernel writes the
// status word (mapped host memory) and returns; the host then reports
// ncclUnhandledCudaError and disables the route.
//
// Counterpart: the reference's direct peer-read route ArPeerRead
// (shim/nccl_collectives_shim.cu:547-565), which is planned but never
// selected, reads the peer's half with a kernel between event waits.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "exec/oneshot.h"
#include "kernels/fold.cuh"

namespace nb {

namespace {

using namespace kfold;

struct OsArgs {
  const void* src[kMaxRanks];         // every rank's input at the range (peer pointers)
  void* dst[kMaxRanks];               // outputs at the range: this rank's (one-shot) or every rank's
  int ndst;
  const void* dev_scalar[kMaxRanks];  // PreMulSum scalars in device memory, per rank
  double scale[kMaxRanks];            // host PreMulSum scalars, per rank
  unsigned* arrive_mine;              // this GPU's tables: [block][rank]
  unsigned* depart_mine;
  unsigned* arrive_peer[kMaxRanks];   // every rank's tables (peer pointers)
  unsigned* depart_peer[kMaxRanks];
  unsigned long long nvec;            // whole vectors
  unsigned long long tail_elems;      // trailing elements
  unsigned long long timeout_ns;
  unsigned* status;                   // mapped host word: nonzero = a wait expired
  unsigned epoch;
  unsigned skew;                      // added to wait targets (bounded-wait test only)
  int op, nranks, rank;
};

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread 0 publishes this block's step to every rank, then waits (bounded)
// for every rank's block with the same index; the block then proceeds. False
// when a wait expired. One release fence orders everything before the
// barrier (this rank's input, written before the kernel; at departure, the
// block's loads of the peers' inputs, joined by the CTA barrier) before the
// relaxed flag stores; the waits poll with relaxed loads and take one
// acquire fence once every flag is seen, so the reads after the barrier see
// what the peers published.
__device__ bool block_barrier(const OsArgs& a, unsigned* const* peer_tables, const unsigned* mine,
                              volatile int* abort_flag) {
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int q = 0; q < a.nranks; ++q)
      st_relaxed(peer_tables[q] + blockIdx.x * unsigned(kMaxRanks) + unsigned(a.rank), a.epoch);
    const unsigned target = a.epoch + a.skew;
    const unsigned long long t0 = gtimer();
    for (int q = 0; q < a.nranks && !*abort_flag; ++q) {
      const unsigned* w = mine + blockIdx.x * unsigned(kMaxRanks) + unsigned(q);
      while (int(ld_relaxed(w) - target) < 0) {
        if (gtimer() - t0 > a.timeout_ns) {
          *reinterpret_cast<volatile unsigned*>(a.status) = 1u;
          __threadfence_system();
          *abort_flag = 1;
          break;
        }
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
  }
  __syncthreads();
  return *abort_flag == 0;
}

template <int VB>
struct Vec {
  uint4 h[VB / 16];
};

template <int VB>
__device__ __forceinline__ Vec<VB> ld_vec(const void* p) {
  Vec<VB> v;
  if constexpr (VB == 32) {
    asm volatile("ld.global.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v.h[0].x), "=r"(v.h[0].y), "=r"(v.h[0].z), "=r"(v.h[0].w), "=r"(v.h[1].x),
                   "=r"(v.h[1].y), "=r"(v.h[1].z), "=r"(v.h[1].w)
                 : "l"(p)
                 : "memory");
  } else {
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.h[0].x), "=r"(v.h[0].y), "=r"(v.h[0].z), "=r"(v.h[0].w)
                 : "l"(p)
                 : "memory");
  }
  return v;
}

template <int VB>
__device__ __forceinline__ void st_vec(void* p, const Vec<VB>& v) {
  if constexpr (VB == 32) {
    asm volatile("st.global.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.h[0].x),
                 "r"(v.h[0].y), "r"(v.h[0].z), "r"(v.h[0].w), "r"(v.h[1].x), "r"(v.h[1].y),
                 "r"(v.h[1].z), "r"(v.h[1].w)
                 : "memory");
  } else {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.h[0].x), "r"(v.h[0].y),
                 "r"(v.h[0].z), "r"(v.h[0].w)
                 : "memory");
  }
}

template <typename T>
__device__ __forceinline__ typename Acc<T>::type scalar_of(const OsArgs& a, int q) {
  using A = typename Acc<T>::type;
  if (a.dev_scalar[q]) return to_acc<T>(*static_cast<const T*>(a.dev_scalar[q]));
  return A(a.scale[q]);
}

template <typename T, int NSRC, int VB>
__global__ void __launch_bounds__(512) oneshot_kernel(const __grid_constant__ OsArgs a) {
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;
  __syncthreads();
  if (!block_barrier(a, a.arrive_peer, a.arrive_mine, &abort_flag)) return;
  using A = typename Acc<T>::type;
  using V = Vec<VB>;
  constexpr int U = (8 * 16 / VB / NSRC) > 0 ? (8 * 16 / VB / NSRC) : 1;  // ~8 16-byte loads in flight
  A s[NSRC];
#pragma unroll
  for (int k = 0; k < NSRC; ++k) s[k] = scalar_of<T>(a, k);
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long base = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; base < a.nvec;
       base += stride * U) {
    V v[U][NSRC];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const unsigned long long i = base + u * stride;
      if (i < a.nvec) {
#pragma unroll
        for (int k = 0; k < NSRC; ++k) v[u][k] = ld_vec<VB>(static_cast<const char*>(a.src[k]) + i * VB);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const unsigned long long i = base + u * stride;
      if (i < a.nvec) {
        V out;
#pragma unroll
        for (int j = 0; j < VB / 16; ++j) {
          uint4 part[NSRC];
#pragma unroll
          for (int k = 0; k < NSRC; ++k) part[k] = v[u][k].h[j];
          out.h[j] = fold_vec<T, NSRC>(part, a.op, a.nranks, s);
        }
        for (int q = 0; q < a.ndst; ++q) st_vec<VB>(static_cast<char*>(a.dst[q]) + i * VB, out);
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < a.tail_elems) {
    const unsigned long long e = a.nvec * (VB / sizeof(T)) + threadIdx.x;
    A acc = first<T>(static_cast<const T*>(a.src[0])[e], a.op, s[0]);
#pragma unroll
    for (int k = 1; k < NSRC; ++k) acc = combine<T>(acc, static_cast<const T*>(a.src[k])[e], a.op, s[k]);
    const T out = finish<T>(acc, a.op, a.nranks);
    for (int q = 0; q < a.ndst; ++q) static_cast<T*>(a.dst[q])[e] = out;
  }
  __syncthreads();
  block_barrier(a, a.depart_peer, a.depart_mine, &abort_flag);
}

using OsFn = void (*)(OsArgs);

template <typename T, int VB>
OsFn by_ranks(int n) {
  switch (n) {
    case 2: return oneshot_kernel<T, 2, VB>;
    case 3: return oneshot_kernel<T, 3, VB>;
    case 4: return oneshot_kernel<T, 4, VB>;
    case 5: return oneshot_kernel<T, 5, VB>;
    case 6: return oneshot_kernel<T, 6, VB>;
    case 7: return oneshot_kernel<T, 7, VB>;
    case 8: return oneshot_kernel<T, 8, VB>;
    default: return nullptr;
  }
}

OsFn pick(DType t, int n, bool wide) {
  switch (t) {
    case DType::F32: return wide ? by_ranks<float, 32>(n) : by_ranks<float, 16>(n);
    case DType::F16: return wide ? by_ranks<__half, 32>(n) : by_ranks<__half, 16>(n);
    case DType::BF16: return wide ? by_ranks<__nv_bfloat16, 32>(n) : by_ranks<__nv_bfloat16, 16>(n);
    default: return nullptr;
  }
}

// Copies (AllGather, Broadcast): one source, moved as 32-bit words by a
// one-source Sum, which performs no arithmetic (bit patterns, NaNs included,
// pass unchanged); payloads are whole 16-byte vectors (the gate's rule).
OsFn pick_copy(bool wide) { return wide ? oneshot_kernel<float, 1, 32> : oneshot_kernel<float, 1, 16>; }

constexpr int kThreads = 512;

struct OsContext {
  std::vector<int> devices;
  std::vector<unsigned*> arrive, depart;  // per device: blocks x kMaxRanks words
  std::vector<cudaEvent_t> done;          // per device: recorded after each launch there
  std::vector<cudaStream_t> last;         // per device: the stream of the previous call
  unsigned* status = nullptr;
  unsigned* status_dev = nullptr;
  unsigned epoch = 0;
  int launched = 0;
  int blocks = 0;
  bool broken = false;
};

std::mutex g_os_mu;
std::vector<OsContext*> g_os;

OsContext* find_os(const int* devices, int n) {
  for (OsContext* c : g_os) {
    if (int(c->devices.size()) != n) continue;
    bool same = true;
    for (int i = 0; i < n; ++i) same &= c->devices[size_t(i)] == devices[i];
    if (same) return c;
  }
  return nullptr;
}

}  // namespace

bool oneshot_supported(DType t, int n) { return pick(t, n, false) != nullptr; }

bool oneshot_ensure(const int* devices, int n, std::string* why) {
  std::lock_guard<std::mutex> lk(g_os_mu);
  if (OsContext* c = find_os(devices, n)) {
    if (c->broken && why) *why = "one-shot route disabled after a device timeout";
    return !c->broken;
  }
  auto fail = [&](const char* what) {
    if (why) *why = std::string("one-shot setup: ") + what;
    cudaGetLastError();
    return false;
  };
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, devices[0]) != cudaSuccess)
    return fail("SM count");
  OsContext* c = new OsContext();
  c->devices.assign(devices, devices + n);
  c->blocks = sms;
  const size_t words = size_t(sms) * kMaxRanks * sizeof(unsigned);
  for (int i = 0; i < n; ++i) {
    unsigned *ar = nullptr, *de = nullptr;
    cudaEvent_t ev = nullptr;
    if (cudaSetDevice(devices[i]) != cudaSuccess || cudaMalloc(&ar, words) != cudaSuccess ||
        cudaMalloc(&de, words) != cudaSuccess || cudaMemset(ar, 0, words) != cudaSuccess ||
        cudaMemset(de, 0, words) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
      delete c;
      return fail("arrive/depart tables");
    }
    c->arrive.push_back(ar);
    c->depart.push_back(de);
    c->done.push_back(ev);
    c->last.push_back(nullptr);
  }
  if (cudaHostAlloc(reinterpret_cast<void**>(&c->status), sizeof(unsigned),
                    cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess ||
      cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->status_dev), c->status, 0) != cudaSuccess) {
    delete c;
    return fail("status word");
  }
  *c->status = 0;
  g_os.push_back(c);
  return true;
}

cudaError_t oneshot_launch(const PlanOp& op, const Plan& plan, const Binding& b, const Policy& p,
                           cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_os_mu);
  OsContext* c = find_os(b.device, b.nranks);
  if (!c || c->broken) return cudaErrorNotSupported;
  const int n = b.nranks, r = op.stream.dev;
  if (c->launched == 0) {
    if (*static_cast<volatile unsigned*>(c->status) != 0) {
      c->broken = true;  // a previous call timed out: the tables are no longer in step
      return cudaErrorLaunchTimeout;
    }
    // A new call: its epoch, and whether any rank changed streams. If one
    // did, every rank's stream waits for the previous call's kernels on every
    // GPU -- all these waits are enqueued now, before this call re-records
    // any of those events.
    ++c->epoch;
    bool fence = false;
    for (int q = 0; q < n; ++q) fence = fence || (c->last[size_t(q)] && c->last[size_t(q)] != b.stream[q]);
    for (int w = 0; fence && w < n; ++w) {
      cudaError_t e = cudaSetDevice(b.device[w]);
      for (int q = 0; q < n && e == cudaSuccess; ++q) e = cudaStreamWaitEvent(b.stream[w], c->done[size_t(q)], 0);
      if (e != cudaSuccess) {
        cudaSetDevice(b.device[r]);
        return e;
      }
    }
    if (fence) {
      const cudaError_t e = cudaSetDevice(b.device[r]);
      if (e != cudaSuccess) return e;
    }
  }
  // Per route: this rank's sources (nsrc of them, rank order), its
  // destinations, and the bytes each moves.
  //   one-shot AllReduce: every input -> own output, the whole message;
  //   two-shot AllReduce: slice r of every input -> slice r of every output;
  //   ReduceScatter:      slot r of every input -> own output;
  //   AllGather:          own input -> slot r of every output (a copy);
  //   Broadcast:          the root's input -> own output (a copy).
  const Algo al = plan.algo;
  const bool copy = al == Algo::AgLL || al == Algo::BcLL;
  const size_t es = copy ? sizeof(float) : elem_size(plan.desc.dtype);
  const size_t msg = plan.desc.bytes;  // AllReduce/Broadcast message, AllGather/ReduceScatter slot
  const char* src[kMaxRanks] = {};
  char* dst[kMaxRanks] = {};
  int nsrc = n, ndst = 1;
  size_t bytes = msg, span = msg;
  if (al == Algo::ArTwoShotLL) {
    const size_t off = op.src[0].off;
    bytes = op.bytes;
    span = msg / size_t(n);
    for (int q = 0; q < n; ++q) {
      src[q] = static_cast<const char*>(b.send[q]) + off;
      dst[q] = static_cast<char*>(b.recv[q]) + off;
    }
    ndst = n;
  } else if (al == Algo::RsLL) {
    for (int q = 0; q < n; ++q) src[q] = static_cast<const char*>(b.send[q]) + size_t(r) * msg;
    dst[0] = static_cast<char*>(b.recv[r]);
  } else if (al == Algo::AgLL) {
    nsrc = 1;
    src[0] = static_cast<const char*>(b.send[r]);
    for (int q = 0; q < n; ++q) dst[q] = static_cast<char*>(b.recv[q]) + size_t(r) * msg;
    ndst = n;
  } else if (al == Algo::BcLL) {
    nsrc = 1;
    src[0] = static_cast<const char*>(b.send[plan.desc.root]);
    dst[0] = static_cast<char*>(b.recv[r]);
  } else {
    for (int q = 0; q < n; ++q) src[q] = static_cast<const char*>(b.send[q]);
    dst[0] = static_cast<char*>(b.recv[r]);
  }
  uintptr_t any = 0;
  for (int q = 0; q < nsrc; ++q) any |= reinterpret_cast<uintptr_t>(src[q]);
  for (int q = 0; q < ndst; ++q) any |= reinterpret_cast<uintptr_t>(dst[q]);
  if (!es || bytes % es || any % 16) return cudaErrorInvalidValue;
  const bool wide = any % 32 == 0;
  const int vb = wide ? 32 : 16;
  const OsFn fn = copy ? pick_copy(wide) : pick(plan.desc.dtype, n, wide);
  if (!fn) return cudaErrorInvalidValue;
  OsArgs a{};
  for (int q = 0; q < n; ++q) {
    a.src[q] = src[q];
    a.dev_scalar[q] = copy ? nullptr : b.dev_scalar[q];
    a.scale[q] = copy ? 1.0 : b.fold.scalars[q];
    a.arrive_peer[q] = c->arrive[size_t(q)];
    a.depart_peer[q] = c->depart[size_t(q)];
  }
  a.ndst = ndst;
  for (int q = 0; q < ndst; ++q) a.dst[q] = dst[q];
  a.arrive_mine = c->arrive[size_t(r)];
  a.depart_mine = c->depart[size_t(r)];
  a.nvec = bytes / size_t(vb);
  a.tail_elems = (bytes - a.nvec * size_t(vb)) / es;
  a.timeout_ns = p.device_timeout_ns;
  a.status = c->status_dev;
  a.epoch = c->epoch;
  a.skew = p.test_nvls_skew;
  a.op = copy ? int(RedOp::Sum) : int(b.fold.op);  // a one-source Sum moves words unchanged
  a.nranks = n;
  a.rank = r;
  // One block per 8 KiB of this rank's range, at least 8 and at most one
  // per SM: the peers' inputs come over NVLink, and each SM sustains only a
  // share of the link rate, so even a 1 MiB range is spread over 128 SMs.
  // Every rank uses the same grid (block b pairs with block b everywhere),
  // so the two-shot grid follows the common slice length, not this rank's.
  const unsigned blocks =
      unsigned(std::min<size_t>(std::max<size_t>(8, (span + 8191) / 8192), size_t(c->blocks)));
  cudaError_t e = cudaSuccess;
  {
    void* argv[] = {&a};
    // Cooperative: every block of the grid is resident at once, so a block
    // waiting for its counterparts never keeps another block of its own
    // kernel from running.
    e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(fn), dim3(blocks), dim3(kThreads), argv, 0, s);
  }
  if (e == cudaSuccess) e = cudaEventRecord(c->done[size_t(r)], s);
  c->last[size_t(r)] = s;
  if (++c->launched == n) c->launched = 0;
  return e;
}

unsigned oneshot_status(const int* devices, int n) {
  std::lock_guard<std::mutex> lk(g_os_mu);
  OsContext* c = find_os(devices, n);
  return c && c->status ? *static_cast<volatile unsigned*>(c->status) : 0u;
}

}  // namespace nb
