// Pipelined Broadcast chain over peer memory with in-kernel flags.
//
// The ranks form a chain root -> root+1 -> ... -> root-1. Every rank except
// the last runs one kernel (one block per SM). The message is cut into steps
// of blocks x C bytes; block b of a rank handles the b-th C-byte piece of
// every step. Per step, a block waits until its predecessor's block b has
// stored that piece into this rank's output (a progress word in this GPU's
// memory, written by the predecessor with a system-scope release), then
// loads the piece from its own output (the root: from its input) and stores
// it into the successor's output over NVLink (P2P stores), and publishes
// the step to the successor's progress word. The root also writes its own
// output when the call is out of place, from the same loads. Data goes
// straight to the final buffers, so there is no scratch and no reuse hazard;
// blocks never wait on another block of their own GPU.
//
// Each GPU's link carries the message once in (from the predecessor) and
// once out (to the successor), with pieces of a few hundred KiB in flight
// per block, which keeps both directions busy; stores (push) run faster
// than remote loads over NVLink.
//
// Every wait is bounded by %globaltimer: on expiry the kernel writes a
// status word in mapped host memory and returns; the host turns it into
// ncclUnhandledCudaError. Progress words only grow: the host advances the
// epoch by each call's step count.
//
// Counterpart: the reference's Broadcast route (shim.cu:660-682) moves the
// non-root's share by one copy-engine copy plus host lanes for two GPUs.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "exec/ring.h"

namespace nb {

namespace {

struct RingArgs {
  const char* src;          // root: its input; others: its own output
  char* own;                // root out of place: its output (else null)
  char* next;               // the successor's output
  const unsigned* wait;     // this GPU's progress words (null at the root)
  unsigned* post;           // the successor's progress words
  unsigned long long bytes;
  unsigned long long chunk; // bytes per block per step (a multiple of 32)
  unsigned long long timeout_ns;
  unsigned* status;         // mapped host word: nonzero = a wait expired
  unsigned base;            // epoch before this call
  unsigned skew;            // added to wait targets (bounded-wait test only)
  // Optional phase timing (NCCL_B200_NVLS_TRACE): per block, ns accumulated
  // over calls: {waiting for the predecessor, total}.
  unsigned long long* trace;
};

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acq(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_rel(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct V32 {
  uint4 lo, hi;
};
__device__ __forceinline__ V32 ld32(const void* p) {
  V32 v;
  asm volatile("ld.global.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.lo.x), "=r"(v.lo.y), "=r"(v.lo.z), "=r"(v.lo.w), "=r"(v.hi.x), "=r"(v.hi.y),
                 "=r"(v.hi.z), "=r"(v.hi.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st32(void* p, const V32& v) {
  asm volatile("st.global.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.lo.x), "r"(v.lo.y),
               "r"(v.lo.z), "r"(v.lo.w), "r"(v.hi.x), "r"(v.hi.y), "r"(v.hi.z), "r"(v.hi.w)
               : "memory");
}

// Copy [off, off+len) of src to next (and own): 32-byte vectors when every
// pointer allows, else 16-byte, else bytes; U loads in flight per thread.
__device__ __forceinline__ void forward(const RingArgs& a, unsigned long long off, unsigned long long len) {
  constexpr int U = 4;
  const char* s = a.src + off;
  char* d = a.next + off;
  char* o = a.own ? a.own + off : nullptr;
  const unsigned t = threadIdx.x, nt = blockDim.x;
  const uintptr_t align = reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d) |
                          (o ? reinterpret_cast<uintptr_t>(o) : 0);
  unsigned long long done = 0;
  if ((align & 31) == 0) {
    const unsigned nv = unsigned(len / 32);
    unsigned i = t;
    for (; i + nt * (U - 1) < nv; i += nt * U) {
      V32 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = ld32(s + size_t(i + u * nt) * 32);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        st32(d + size_t(i + u * nt) * 32, v[u]);
        if (o) st32(o + size_t(i + u * nt) * 32, v[u]);
      }
    }
    for (; i < nv; i += nt) {
      const V32 v = ld32(s + size_t(i) * 32);
      st32(d + size_t(i) * 32, v);
      if (o) st32(o + size_t(i) * 32, v);
    }
    done = size_t(nv) * 32;
  } else if ((align & 15) == 0) {
    const unsigned nv = unsigned(len / 16);
    for (unsigned i = t; i < nv; i += nt) {
      const uint4 v = reinterpret_cast<const uint4*>(s)[i];
      reinterpret_cast<uint4*>(d)[i] = v;
      if (o) reinterpret_cast<uint4*>(o)[i] = v;
    }
    done = size_t(nv) * 16;
  }
  for (unsigned long long i = done + t; i < len; i += nt) {
    d[i] = s[i];
    if (o) o[i] = s[i];
  }
}

__global__ void __launch_bounds__(512, 1) bc_ring_kernel(const __grid_constant__ RingArgs a) {
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;
  __syncthreads();
  const unsigned long long step = a.chunk * gridDim.x;
  const unsigned steps = unsigned((a.bytes + step - 1) / step);
  const unsigned long long t_start = a.trace && threadIdx.x == 0 ? gtimer() : 0;
  unsigned long long waited = 0;
  for (unsigned k = 0; k < steps; ++k) {
    const unsigned long long off = k * step + a.chunk * blockIdx.x;
    const unsigned long long len = off < a.bytes ? min(a.chunk, a.bytes - off) : 0;
    if (a.wait) {
      if (threadIdx.x == 0) {
        const unsigned target = a.base + k + 1 + a.skew;
        const unsigned long long t0 = gtimer();
        while (int(ld_acq(a.wait + blockIdx.x) - target) < 0) {
          if (gtimer() - t0 > a.timeout_ns) {
            *reinterpret_cast<volatile unsigned*>(a.status) = 1u;
            __threadfence_system();
            abort_flag = 1;
            break;
          }
        }
        if (a.trace) waited += gtimer() - t0;
      }
      __syncthreads();
      if (abort_flag) return;
    }
    if (len) forward(a, off, len);
    __syncthreads();
    if (threadIdx.x == 0) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      st_rel(a.post + blockIdx.x, a.base + k + 1);
    }
  }
  if (a.trace && threadIdx.x == 0) {
    atomicAdd(a.trace + 2ull * blockIdx.x, waited);
    atomicAdd(a.trace + 2ull * blockIdx.x + 1, gtimer() - t_start);
  }
}

struct RingContext {
  std::vector<int> devices;
  std::vector<unsigned*> flags;  // per device: `blocks` progress words
  std::vector<unsigned long long*> trace;  // per device: blocks x 2 phase-time records
  unsigned* status = nullptr;
  unsigned* status_dev = nullptr;
  unsigned long long epoch = 0;
  int launched = 0;  // ranks of the current call submitted so far
  int blocks = 0;
  bool broken = false;
};

std::mutex g_ring_mu;
std::vector<RingContext*> g_rings;

RingContext* find_ring(const int* devices, int n) {
  for (RingContext* c : g_rings) {
    if (int(c->devices.size()) != n) continue;
    bool same = true;
    for (int i = 0; i < n; ++i) same &= c->devices[size_t(i)] == devices[i];
    if (same) return c;
  }
  return nullptr;
}

}  // namespace

bool ring_ensure(const int* devices, int n, std::string* why) {
  std::lock_guard<std::mutex> lk(g_ring_mu);
  if (RingContext* c = find_ring(devices, n)) {
    if (c->broken && why) *why = "ring route disabled after a device timeout";
    return !c->broken;
  }
  auto fail = [&](const char* what) {
    if (why) *why = std::string("ring setup: ") + what;
    cudaGetLastError();
    return false;
  };
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, devices[0]) != cudaSuccess)
    return fail("SM count");
  RingContext* c = new RingContext();
  c->devices.assign(devices, devices + n);
  c->blocks = sms;
  for (int i = 0; i < n; ++i) {
    unsigned* f = nullptr;
    if (cudaSetDevice(devices[i]) != cudaSuccess || cudaMalloc(&f, size_t(sms) * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(f, 0, size_t(sms) * sizeof(unsigned)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
      delete c;
      return fail("progress words");
    }
    unsigned long long* tr = nullptr;
    if (cudaMalloc(&tr, size_t(sms) * 2 * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(tr, 0, size_t(sms) * 2 * sizeof(unsigned long long)) != cudaSuccess) {
      delete c;
      return fail("trace records");
    }
    c->flags.push_back(f);
    c->trace.push_back(tr);
  }
  if (cudaHostAlloc(reinterpret_cast<void**>(&c->status), sizeof(unsigned),
                    cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess ||
      cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->status_dev), c->status, 0) != cudaSuccess) {
    delete c;
    return fail("status word");
  }
  *c->status = 0;
  g_rings.push_back(c);
  return true;
}

cudaError_t ring_launch(const PlanOp& op, const Plan& plan, const Binding& b, const Policy& p,
                        cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_ring_mu);
  RingContext* c = find_ring(b.device, b.nranks);
  if (!c || c->broken) return cudaErrorNotSupported;
  const int n = b.nranks, r = op.stream.dev, root = plan.desc.root;
  if (r == root && *static_cast<volatile unsigned*>(c->status) != 0) {
    c->broken = true;  // a previous call timed out: progress words are no longer in step
    return cudaErrorLaunchTimeout;
  }
  const unsigned long long chunk = p.ring_chunk;
  const unsigned long long stepb = chunk * (unsigned long long)c->blocks;
  const unsigned long long steps = (plan.desc.bytes + stepb - 1) / stepb;
  const int hop = (r - root + n) % n;  // position in the chain
  cudaError_t e = cudaSuccess;
  if (hop != n - 1) {  // the last rank only receives
    const int next = (r + 1) % n;
    RingArgs a{};
    a.src = hop == 0 ? static_cast<const char*>(b.send[r]) : static_cast<const char*>(b.recv[r]);
    a.own = hop == 0 && !plan.desc.in_place[r] ? static_cast<char*>(b.recv[r]) : nullptr;
    a.next = static_cast<char*>(b.recv[next]);
    a.wait = hop == 0 ? nullptr : c->flags[size_t(r)];
    a.post = c->flags[size_t(next)];
    a.bytes = plan.desc.bytes;
    a.chunk = chunk;
    a.timeout_ns = p.device_timeout_ns;
    a.status = c->status_dev;
    a.base = unsigned(c->epoch);
    a.skew = p.test_nvls_skew;
    a.trace = p.nvls_trace ? c->trace[size_t(r)] : nullptr;
    bc_ring_kernel<<<dim3(unsigned(c->blocks)), dim3(512), 0, s>>>(a);
    e = cudaGetLastError();
  }
  // Once every rank of the call is submitted, the epoch moves past it.
  if (++c->launched == n) {
    c->launched = 0;
    c->epoch += steps;
  }
  return e;
}

unsigned ring_status(const int* devices, int n) {
  std::lock_guard<std::mutex> lk(g_ring_mu);
  RingContext* c = find_ring(devices, n);
  return c && c->status ? *static_cast<volatile unsigned*>(c->status) : 0u;
}

int ring_trace_read(const int* devices, int n, int rank, double out[2], bool reset) {
  std::lock_guard<std::mutex> lk(g_ring_mu);
  RingContext* c = find_ring(devices, n);
  if (!c || rank < 0 || rank >= n) return -1;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(devices[rank]) != cudaSuccess) return -1;
  std::vector<unsigned long long> rec(size_t(c->blocks) * 2);
  const size_t bytes = rec.size() * sizeof(unsigned long long);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(rec.data(), c->trace[size_t(rank)], bytes, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && reset) e = cudaMemset(c->trace[size_t(rank)], 0, bytes);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return -1;
  int ran = 0;
  double sum[2] = {};
  for (int b = 0; b < c->blocks; ++b) {
    if (!rec[size_t(b) * 2 + 1]) continue;
    ++ran;
    sum[0] += double(rec[size_t(b) * 2]);
    sum[1] += double(rec[size_t(b) * 2 + 1]);
  }
  out[0] = ran ? sum[0] / ran : 0.0;
  out[1] = ran ? sum[1] / ran : 0.0;
  return ran;
}

}  // namespace nb
