// Push-reduce engine: ReduceScatter and two-shot AllReduce with NVLink
// stores only.
//
// Rank q owns segment q (AllReduce: slice q of the buffer; ReduceScatter:
// slot q). Every rank runs one kernel (one block per SM, cooperative launch)
// with two warp groups that progress independently:
//   sender  : stores its own input's piece of segment q into q's scratch for
//             every owner q != r (P2P stores into q's memory), drains the
//             store stream once per round (one system fence), then publishes
//             "filled" to every owner;
//   reducer : once every sender filled this piece of its own segment, folds
//             the pieces in rank order (its own input in place r) with fp32
//             accumulation, writes the result to its output (AllReduce: to
//             every rank's output, P2P stores), then publishes "consumed" to
//             every sender.
// Pieces: block b handles C-byte piece k = j*B + b of every segment in round
// j; the scratch holds D rounds per (sender, block), so a sender waits for
// the owner's "consumed" of round j-D before reusing a slot. Progress words
// live in each GPU's memory and are written by peers with system-scope
// releases; every wait is bounded by %globaltimer (status word in mapped
// host memory, then return). Remote loads are never used: over NVLink a
// store stream runs faster than a load stream, whose requests share the
// return direction.
//
// Counterpart: the reference's staged reduce (shim.cu:518-545) pulls the
// peer's half into a scratch buffer with a copy engine and adds it with a
// separate kernel, for two GPUs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "exec/pushred.h"
#include "kernels/fold.cuh"

namespace nb {

namespace {

using namespace kfold;

constexpr int kDepth = 2;                   // rounds of scratch per (sender, block)
constexpr unsigned long long kPiece = 262144;  // C: bytes per block per round per segment

struct PrArgs {
  const char* send;
  char* recv[kMaxRanks];        // AllReduce: every rank's output; ReduceScatter: [rank] only
  char* scratch[kMaxRanks];     // every rank's scratch base (index: the owner)
  unsigned* filled[kMaxRanks];  // every rank's "filled" words [sender][block]
  unsigned* consumed[kMaxRanks];// every rank's "consumed" words [owner][block]
  const void* dev_scalar[kMaxRanks];
  double scale[kMaxRanks];
  unsigned long long seg_off[kMaxRanks];  // segment q's offset in the input
  unsigned long long seg_len[kMaxRanks];
  unsigned long long out_off;   // AllReduce: seg_off[rank]; ReduceScatter: 0
  unsigned long long timeout_ns;
  unsigned* status;
  unsigned base, skew;
  unsigned rounds;
  int nranks, rank, op, allreduce, senders;  // senders: threads of the sender group
  // Optional phase timing (NCCL_B200_NVLS_TRACE): per block, ns accumulated
  // over calls: {sender waiting, sender total, reducer waiting, reducer total}.
  unsigned long long* trace;
};

__device__ __forceinline__ unsigned long long timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void release(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Scratch slot of (sender s, block b, round j) in an owner's scratch.
__device__ __forceinline__ unsigned long long slot_off(int s, unsigned j) {
  return ((unsigned long long)(s * gridDim.x + blockIdx.x) * kDepth + (j % kDepth)) * kPiece;
}
__device__ __forceinline__ unsigned flag_idx(int who) { return unsigned(who) * gridDim.x + blockIdx.x; }

// Group leader: wait until p[i] >= v for every listed word; false when a
// wait expired (status set) or the block is aborting.
__device__ bool leader_wait(const PrArgs& a, const unsigned* const* words, int count, unsigned v,
                            volatile int* abort) {
  const unsigned target = v + a.skew;
  const unsigned long long t0 = timer_ns();
  for (int i = 0; i < count; ++i) {
    while (int(acquire(words[i]) - target) < 0) {
      if (*abort) return false;
      if (timer_ns() - t0 > a.timeout_ns) {
        *reinterpret_cast<volatile unsigned*>(a.status) = 1u;
        __threadfence_system();
        *abort = 1;
        return false;
      }
    }
  }
  return true;
}

// Copy len bytes (a multiple of 16) with nt threads: 16-byte vectors, four
// in flight per thread.
__device__ __forceinline__ void push_copy(char* dst, const char* src, unsigned long long len, unsigned t,
                                          unsigned nt) {
  const unsigned nv = unsigned(len / 16);
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  unsigned i = t;
  for (; i + 3 * nt < nv; i += 4 * nt) {
    const uint4 x0 = __ldcs(s + i), x1 = __ldcs(s + i + nt), x2 = __ldcs(s + i + 2 * nt),
                x3 = __ldcs(s + i + 3 * nt);
    d[i] = x0;
    d[i + nt] = x1;
    d[i + 2 * nt] = x2;
    d[i + 3 * nt] = x3;
  }
  for (; i < nv; i += nt) d[i] = __ldcs(s + i);
}

template <typename T, int N>
__global__ void __launch_bounds__(512, 1) pushred_kernel(const __grid_constant__ PrArgs a) {
  using A = typename Acc<T>::type;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;
  __syncthreads();
  const int r = a.rank;
  const bool sender = int(threadIdx.x) < a.senders;
  const unsigned t = sender ? threadIdx.x : threadIdx.x - a.senders;
  const unsigned nt = sender ? a.senders : blockDim.x - a.senders;
  const int gid = sender ? 1 : 2;
  volatile int* abort = &abort_flag;
  // Phase timing, kept by each group's leader.
  const unsigned long long t_start = a.trace && t == 0 ? timer_ns() : 0;
  unsigned long long waited = 0;
  auto timed_wait = [&](const unsigned* const* w, int c, unsigned v) {
    const unsigned long long w0 = a.trace ? timer_ns() : 0;
    leader_wait(a, w, c, v, abort);
    if (a.trace) waited += timer_ns() - w0;
  };
  auto trace_out = [&](int slot) {
    if (!a.trace || t != 0) return;
    unsigned long long* rec = a.trace + 4ull * blockIdx.x + slot;
    atomicAdd(rec, waited);
    atomicAdd(rec + 1, timer_ns() - t_start);
  };
  if (sender) {
    for (unsigned j = 0; j < a.rounds; ++j) {
      const unsigned long long k = (unsigned long long)j * gridDim.x + blockIdx.x;
      // Every owner consumed round j - kDepth (this round's scratch slots).
      if (j >= kDepth) {
        if (t == 0) {
          const unsigned* w[kMaxRanks];
          int c = 0;
          for (int i = 1; i < N; ++i) w[c++] = a.consumed[r] + flag_idx((r + i) % N);
          timed_wait(w, c, a.base + j - kDepth + 1);
        }
        bar(gid, nt);
        if (*abort) return;
      }
      // Push this round's piece to every owner, then drain the stores once.
      for (int i = 1; i < N; ++i) {
        const int q = (r + i) % N;
        const unsigned long long cs = k * kPiece;
        const unsigned long long len = cs < a.seg_len[q] ? min(kPiece, a.seg_len[q] - cs) : 0;
        // Whole 16-byte units; a trailing partial vector goes element-wise.
        const unsigned long long body = len & ~15ull;
        char* dst = a.scratch[q] + slot_off(r, j);
        const char* src = a.send + a.seg_off[q] + cs;
        push_copy(dst, src, body, t, nt);
        for (unsigned long long e = body + t; e < len; e += nt) dst[e] = src[e];
      }
      bar(gid, nt);
      if (t == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int i = 1; i < N; ++i) release(a.filled[(r + i) % N] + flag_idx(r), a.base + j + 1);
      }
    }
    trace_out(0);
    return;
  }
  // Reducer group.
  A s[N];
#pragma unroll
  for (int q = 0; q < N; ++q)
    s[q] = a.dev_scalar[q] ? to_acc<T>(*reinterpret_cast<const T*>(a.dev_scalar[q])) : A(a.scale[q]);
  constexpr int E = 16 / sizeof(T);
  for (unsigned j = 0; j < a.rounds; ++j) {
    const unsigned long long k = (unsigned long long)j * gridDim.x + blockIdx.x;
    if (t == 0) {
      const unsigned* w[kMaxRanks];
      int c = 0;
      for (int q = 0; q < N; ++q)
        if (q != r) w[c++] = a.filled[r] + flag_idx(q);
      timed_wait(w, c, a.base + j + 1);
    }
    bar(gid, nt);
    if (*abort) return;
    const unsigned long long cs = k * kPiece;
    const unsigned long long len = cs < a.seg_len[r] ? min(kPiece, a.seg_len[r] - cs) : 0;
    const char* src[N];
#pragma unroll
    for (int q = 0; q < N; ++q)
      src[q] = q == r ? a.send + a.seg_off[r] + cs : a.scratch[r] + slot_off(q, j);
    const unsigned nv = unsigned(len / 16);
    const int ndst = a.allreduce ? N : 1;
    // About eight 16-byte loads in flight per thread (the sources are local).
    constexpr int U = 8 / N > 0 ? 8 / N : 1;
    for (unsigned v0 = t; v0 < nv; v0 += nt * U) {
      uint4 x[U][N];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (v0 + u * nt < nv) {
#pragma unroll
          for (int q = 0; q < N; ++q) x[u][q] = reinterpret_cast<const uint4*>(src[q])[v0 + u * nt];
        }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const unsigned v = v0 + u * nt;
        if (v >= nv) break;
        const uint4 y = fold_vec<T, N>(x[u], a.op, a.nranks, s);
        for (int d = 0; d < ndst; ++d) {
          const int q = a.allreduce ? (r + d) % N : r;  // own output first, then r+1, ...
          reinterpret_cast<uint4*>(a.recv[q] + a.out_off + cs)[v] = y;
        }
      }
    }
    // Trailing elements of a segment that do not fill a vector.
    for (unsigned long long e = (unsigned long long)nv * E + t; e < len / sizeof(T); e += nt) {
      A acc = first<T>(reinterpret_cast<const T*>(src[0])[e], a.op, s[0]);
#pragma unroll
      for (int q = 1; q < N; ++q) acc = combine<T>(acc, reinterpret_cast<const T*>(src[q])[e], a.op, s[q]);
      const T out = finish<T>(acc, a.op, a.nranks);
      for (int d = 0; d < ndst; ++d) {
        const int q = a.allreduce ? (r + d) % N : r;
        reinterpret_cast<T*>(a.recv[q] + a.out_off + cs)[e] = out;
      }
    }
    bar(gid, nt);
    if (t == 0) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      for (int q = 0; q < N; ++q)
        if (q != r) release(a.consumed[q] + flag_idx(r), a.base + j + 1);
    }
  }
  trace_out(2);
}

template <typename T>
const void* pick_n(int n) {
  switch (n) {
    case 2: return reinterpret_cast<const void*>(pushred_kernel<T, 2>);
    case 3: return reinterpret_cast<const void*>(pushred_kernel<T, 3>);
    case 4: return reinterpret_cast<const void*>(pushred_kernel<T, 4>);
    case 5: return reinterpret_cast<const void*>(pushred_kernel<T, 5>);
    case 6: return reinterpret_cast<const void*>(pushred_kernel<T, 6>);
    case 7: return reinterpret_cast<const void*>(pushred_kernel<T, 7>);
    case 8: return reinterpret_cast<const void*>(pushred_kernel<T, 8>);
    default: return nullptr;
  }
}

const void* pick(DType t, int n) {
  switch (t) {
    case DType::F32: return pick_n<float>(n);
    case DType::BF16: return pick_n<__nv_bfloat16>(n);
    case DType::F16: return pick_n<__half>(n);
    default: return nullptr;
  }
}

struct PrContext {
  std::vector<int> devices;
  std::vector<char*> scratch;
  std::vector<unsigned*> filled, consumed;
  std::vector<unsigned long long*> trace;  // per device: blocks x 4 phase-time records
  unsigned* status = nullptr;
  unsigned* status_dev = nullptr;
  unsigned long long epoch = 0;
  int launched = 0;
  int blocks = 0;
  bool broken = false;
};

std::mutex g_pr_mu;
std::vector<PrContext*> g_prs;

PrContext* find_pr(const int* devices, int n) {
  for (PrContext* c : g_prs) {
    if (int(c->devices.size()) != n) continue;
    bool same = true;
    for (int i = 0; i < n; ++i) same &= c->devices[size_t(i)] == devices[i];
    if (same) return c;
  }
  return nullptr;
}

}  // namespace

bool pushred_supported(DType t, int n) { return n >= 2 && n <= kMaxRanks && pick(t, n) != nullptr; }

bool pushred_ensure(const int* devices, int n, std::string* why) {
  std::lock_guard<std::mutex> lk(g_pr_mu);
  if (PrContext* c = find_pr(devices, n)) {
    if (c->broken && why) *why = "push-reduce route disabled after a device timeout";
    return !c->broken;
  }
  auto fail = [&](const char* what) {
    if (why) *why = std::string("push-reduce setup: ") + what;
    cudaGetLastError();
    return false;
  };
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, devices[0]) != cudaSuccess)
    return fail("SM count");
  PrContext* c = new PrContext();
  c->devices.assign(devices, devices + n);
  c->blocks = sms;
  const size_t scratch = size_t(n) * size_t(sms) * kDepth * kPiece;
  const size_t words = size_t(n) * size_t(sms) * sizeof(unsigned);
  for (int i = 0; i < n; ++i) {
    char* sc = nullptr;
    unsigned *f = nullptr, *u = nullptr;
    if (cudaSetDevice(devices[i]) != cudaSuccess || cudaMalloc(&sc, scratch) != cudaSuccess ||
        cudaMalloc(&f, words) != cudaSuccess || cudaMalloc(&u, words) != cudaSuccess ||
        cudaMemset(f, 0, words) != cudaSuccess || cudaMemset(u, 0, words) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
      delete c;
      return fail("scratch and progress words");
    }
    unsigned long long* tr = nullptr;
    if (cudaMalloc(&tr, size_t(sms) * 4 * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(tr, 0, size_t(sms) * 4 * sizeof(unsigned long long)) != cudaSuccess) {
      delete c;
      return fail("trace records");
    }
    c->scratch.push_back(sc);
    c->filled.push_back(f);
    c->consumed.push_back(u);
    c->trace.push_back(tr);
  }
  if (cudaHostAlloc(reinterpret_cast<void**>(&c->status), sizeof(unsigned),
                    cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess ||
      cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->status_dev), c->status, 0) != cudaSuccess) {
    delete c;
    return fail("status word");
  }
  *c->status = 0;
  g_prs.push_back(c);
  return true;
}

cudaError_t pushred_launch(const PlanOp& op, const Plan& plan, const Binding& b, const Policy& p,
                           cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_pr_mu);
  PrContext* c = find_pr(b.device, b.nranks);
  if (!c || c->broken) return cudaErrorNotSupported;
  const int n = b.nranks, r = op.stream.dev;
  if (r == 0 && *static_cast<volatile unsigned*>(c->status) != 0) {
    c->broken = true;
    return cudaErrorLaunchTimeout;
  }
  const void* fn = pick(plan.desc.dtype, n);
  if (!fn) return cudaErrorNotSupported;
  const bool ar = plan.desc.kind == Kind::AllReduce;
  PrArgs a{};
  a.send = static_cast<const char*>(b.send[r]);
  unsigned long long longest = 0;
  for (int q = 0; q < n; ++q) {
    a.recv[q] = static_cast<char*>(ar || q == r ? b.recv[q] : nullptr);
    a.scratch[q] = c->scratch[size_t(q)];
    a.filled[q] = c->filled[size_t(q)];
    a.consumed[q] = c->consumed[size_t(q)];
    a.dev_scalar[q] = b.dev_scalar[q];
    a.scale[q] = b.fold.scalars[q];
    size_t off = 0, len = 0;
    if (ar) {
      slice_of(plan.desc.bytes, n, q, &off, &len);
    } else {
      off = size_t(q) * plan.desc.bytes;
      len = plan.desc.bytes;
    }
    a.seg_off[q] = off;
    a.seg_len[q] = len;
    longest = std::max<unsigned long long>(longest, len);
  }
  a.out_off = ar ? a.seg_off[r] : 0;
  a.timeout_ns = p.device_timeout_ns;
  a.status = c->status_dev;
  a.base = unsigned(c->epoch);
  a.skew = p.test_nvls_skew;
  const unsigned long long per_round = kPiece * (unsigned long long)c->blocks;
  a.rounds = unsigned((longest + per_round - 1) / per_round);
  a.nranks = n;
  a.rank = r;
  a.op = int(plan.desc.op);
  a.allreduce = ar ? 1 : 0;
  a.senders = 256;
  a.trace = p.nvls_trace ? c->trace[size_t(r)] : nullptr;
  void* argv[] = {&a};
  const cudaError_t e = cudaLaunchCooperativeKernel(fn, dim3(unsigned(c->blocks)), dim3(512), argv, 0, s);
  if (++c->launched == n) {
    c->launched = 0;
    c->epoch += a.rounds;
  }
  return e;
}

unsigned pushred_status(const int* devices, int n) {
  std::lock_guard<std::mutex> lk(g_pr_mu);
  PrContext* c = find_pr(devices, n);
  return c && c->status ? *static_cast<volatile unsigned*>(c->status) : 0u;
}

int pushred_trace_read(const int* devices, int n, int rank, double out[4], bool reset) {
  std::lock_guard<std::mutex> lk(g_pr_mu);
  PrContext* c = find_pr(devices, n);
  if (!c || rank < 0 || rank >= n) return -1;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(devices[rank]) != cudaSuccess) return -1;
  std::vector<unsigned long long> rec(size_t(c->blocks) * 4);
  const size_t bytes = rec.size() * sizeof(unsigned long long);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(rec.data(), c->trace[size_t(rank)], bytes, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && reset) e = cudaMemset(c->trace[size_t(rank)], 0, bytes);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return -1;
  int ran = 0;
  double sum[4] = {};
  for (int b = 0; b < c->blocks; ++b) {
    const unsigned long long* r = &rec[size_t(b) * 4];
    if (!(r[1] | r[3])) continue;
    ++ran;
    for (int k = 0; k < 4; ++k) sum[k] += double(r[k]);
  }
  for (int k = 0; k < 4; ++k) out[k] = ran ? sum[k] / double(ran) : 0.0;  // mean ns per block
  return ran;
}

}  // namespace nb
