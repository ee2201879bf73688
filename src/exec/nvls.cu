// NVLS AllReduce: multicast objects over the clique's GPUs and the multimem
// gang kernel.
//
// Setup (once per device set): one multicast object spans every clique GPU;
// each GPU binds its own physical scratch (cuMemCreate) into it and maps
// both a unicast view (its own memory) and a multicast view. The scratch
// holds three round buffers of R bytes plus one flag word per block.
//
// Kernel (one per GPU, all launched for the same call form a gang): the
// message is processed in rounds of R bytes, each cut into N slices; rank r
// owns slice r. Per round: A) copy this GPU's input round into its scratch
// (unicast); B) for slice r, multimem.ld_reduce through the multicast view
// (the switch reads every GPU's scratch and returns the sum, accumulated in
// fp32 for 16-bit types) and multimem.st of the result (the switch writes it
// into every GPU's scratch); C) copy the round out of the scratch into the
// output. Steps are software-pipelined over three buffers: step s runs
// C(s-2), B(s-1), A(s), then one cross-GPU barrier per block
// (multimem.red.release.sys increments that block's flag on every GPU; the
// block waits with ld.acquire until all N arrived). Every wait is bounded by
// %globaltimer: on expiry the kernel writes a status word in mapped host
// memory and returns; the host turns it into ncclUnhandledCudaError and
// disables the route. No TMA, and no multicast TMA, is used.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "exec/nvls.h"

namespace nb {

namespace {

// ---------------------------------------------------------------- device side

struct NvlsArgs {
  const char* send;
  char* recv;
  char* uc;        // unicast view of this GPU's scratch
  char* mc;        // multicast view (same offsets)
  unsigned* uc_flags;
  unsigned* mc_flags;
  unsigned long long bytes;
  unsigned long long round;  // R
  unsigned long long buf_stride;
  unsigned long long timeout_ns;
  unsigned* status;          // mapped host word: nonzero = a wait expired
  unsigned base;             // flag value before this call's first barrier
  int nranks, rank, dtype, avg;
  int movers;                // threads of a block that work through the switch
  int mode;                  // collective kind (xfer kernel)
  int root;                  // Broadcast
  unsigned long long slot;   // AllGather / ReduceScatter per-rank slot bytes
};

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void mc_arrive(unsigned* p) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(1u) : "memory");
}

__device__ __forceinline__ uint4 ld_reduce(const void* p, int dtype) {
  uint4 v;
  if (dtype == int(DType::BF16)) {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  } else if (dtype == int(DType::F16)) {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  } else {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  }
  return v;
}

__device__ __forceinline__ void mc_store(void* p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 scale(uint4 v, int dtype, float inv) {
  if (dtype == int(DType::F32)) {
    float* f = reinterpret_cast<float*>(&v);
    for (int i = 0; i < 4; ++i) f[i] = f[i] * inv;
  } else if (dtype == int(DType::BF16)) {
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&v);
    for (int i = 0; i < 8; ++i) h[i] = __float2bfloat16_rn(__bfloat162float(h[i]) * inv);
  } else {
    __half* h = reinterpret_cast<__half*>(&v);
    for (int i = 0; i < 8; ++i) h[i] = __float2half_rn(__half2float(h[i]) * inv);
  }
  return v;
}

// This block's part [lo, hi) of slice q of a round of `rlen` bytes; all
// boundaries are 16-byte aligned (the message is a multiple of 16 bytes).
__device__ __forceinline__ void portion(unsigned long long rlen, int n, int q, unsigned long long* lo,
                                        unsigned long long* hi) {
  // Slices and block parts start on 32-byte boundaries (the copiers' vector).
  const unsigned long long base = (rlen / (unsigned long long)n) & ~31ull;
  const unsigned long long soff = base * (unsigned long long)q;
  const unsigned long long slen = q == n - 1 ? rlen - soff : base;
  const unsigned long long per = ((slen + gridDim.x - 1) / gridDim.x + 31) & ~31ull;
  const unsigned long long a = min(slen, per * blockIdx.x), b = min(slen, a + per);
  *lo = soff + a;
  *hi = soff + b;
}

struct V32 {
  uint4 lo, hi;
};
__device__ __forceinline__ V32 ld32(const void* p) {
  V32 v;
  asm volatile("ld.global.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.lo.x), "=r"(v.lo.y), "=r"(v.lo.z), "=r"(v.lo.w), "=r"(v.hi.x), "=r"(v.hi.y),
                 "=r"(v.hi.z), "=r"(v.hi.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st32(void* p, const V32& v) {
  asm volatile("st.global.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.lo.x), "r"(v.lo.y),
               "r"(v.lo.z), "r"(v.lo.w), "r"(v.hi.x), "r"(v.hi.y), "r"(v.hi.z), "r"(v.hi.w)
               : "memory");
}

// Copy `bytes` (a multiple of 16) with the `nthreads` threads of a warp group
// (thread index t): 32-byte vectors when both ends allow, else 16-byte.
__device__ __forceinline__ void copy16(char* dst, const char* src, unsigned long long bytes, int t,
                                       int nthreads) {
  constexpr int U = 4;
  unsigned long long done = 0;
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 31) == 0) {
    const unsigned long long nv = bytes / 32;
    for (unsigned long long i = t; i < nv; i += (unsigned long long)nthreads * U) {
      V32 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i + u * nthreads < nv) v[u] = ld32(src + (i + u * nthreads) * 32);
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i + u * nthreads < nv) st32(dst + (i + u * nthreads) * 32, v[u]);
    }
    done = nv * 32;
  }
  const unsigned long long nv = (bytes - done) / 16;
  src += done;
  dst += done;
  for (unsigned long long i = t; i < nv; i += (unsigned long long)nthreads * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i + u * nthreads < nv) v[u] = __ldcs(reinterpret_cast<const uint4*>(src) + i + u * nthreads);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i + u * nthreads < nv) __stcs(reinterpret_cast<uint4*>(dst) + i + u * nthreads, v[u]);
  }
}

// Warp specialization: the first half of the block's warps reduce through
// the switch (NVLink-bound) while the second half copies rounds in and out
// of the scratch (HBM-bound), so the two resources work at the same time.
// U: multimem requests in flight per switch-side thread.
template <int U, int DT>
__global__ void __launch_bounds__(768, 1) nvls_allreduce_kernel(const __grid_constant__ NvlsArgs a) {
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;
  __syncthreads();
  const int n = a.nranks;
  const unsigned long long rounds = (a.bytes + a.round - 1) / a.round;
  const float inv = 1.0f / float(n);
  // The first a.movers threads work through the switch; the rest copy.
  const bool reducer = int(threadIdx.x) < a.movers;
  const int t = reducer ? threadIdx.x : threadIdx.x - a.movers;
  const int half = reducer ? a.movers : int(blockDim.x) - a.movers;  // this group's size
  for (unsigned long long s = 0; s < rounds + 2; ++s) {
    if (!reducer) {
      // C(s-2): copy the reduced round out of the scratch.
      if (s >= 2) {
        const unsigned long long i = s - 2, rbase = i * a.round;
        const unsigned long long rlen = min(a.round, a.bytes - rbase);
        const char* buf = a.uc + (i % 3) * a.buf_stride;
        for (int q = 0; q < n; ++q) {
          unsigned long long lo, hi;
          portion(rlen, n, q, &lo, &hi);
          copy16(a.recv + rbase + lo, buf + lo, hi - lo, t, half);
        }
      }
      // A(s): copy this GPU's input round into its scratch.
      if (s < rounds) {
        const unsigned long long rbase = s * a.round;
        const unsigned long long rlen = min(a.round, a.bytes - rbase);
        char* buf = a.uc + (s % 3) * a.buf_stride;
        for (int q = 0; q < n; ++q) {
          unsigned long long lo, hi;
          portion(rlen, n, q, &lo, &hi);
          copy16(buf + lo, a.send + rbase + lo, hi - lo, t, half);
        }
      }
    } else if (s >= 1 && s - 1 < rounds) {
      // B(s-1): reduce and multicast this rank's slice.
      const unsigned long long i = s - 1, rbase = i * a.round;
      const unsigned long long rlen = min(a.round, a.bytes - rbase);
      char* mbuf = a.mc + (i % 3) * a.buf_stride;
      unsigned long long lo, hi;
      portion(rlen, n, a.rank, &lo, &hi);
      const unsigned long long nv = (hi - lo) / 16;
      for (unsigned long long v = t; v < nv; v += (unsigned long long)half * U) {
        uint4 x[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (v + u * half < nv) x[u] = ld_reduce(mbuf + lo + (v + u * half) * 16, DT);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (v + u * half < nv)
            mc_store(mbuf + lo + (v + u * half) * 16, a.avg ? scale(x[u], DT, inv) : x[u]);
      }
    }
    // Barrier: this block's counterparts on every GPU finished step s.
    __syncthreads();
    if (threadIdx.x == 0) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      mc_arrive(a.mc_flags + blockIdx.x);
      const unsigned target = a.base + unsigned(n) * unsigned(s + 1);
      const unsigned long long start = globaltimer();
      while (int(ld_acquire(a.uc_flags + blockIdx.x) - target) < 0) {
        if (globaltimer() - start > a.timeout_ns) {
          *reinterpret_cast<volatile unsigned*>(a.status) = 1u;  // mapped host word
          __threadfence_system();
          abort_flag = 1;
          break;
        }
      }
    }
    __syncthreads();
    if (abort_flag) return;
  }
}

// This block's part [lo, hi) of a flat range of `len` bytes (16-byte units).
__device__ __forceinline__ void flat_portion(unsigned long long len, unsigned long long* lo,
                                             unsigned long long* hi) {
  const unsigned long long per = ((len + gridDim.x - 1) / gridDim.x + 31) & ~31ull;
  *lo = min(len, per * blockIdx.x);
  *hi = min(len, *lo + per);
}

__device__ __forceinline__ bool nvls_barrier(const NvlsArgs& a, unsigned long long s, int* abort_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    mc_arrive(a.mc_flags + blockIdx.x);
    const unsigned target = a.base + unsigned(a.nranks) * unsigned(s + 1);
    const unsigned long long start = globaltimer();
    while (int(ld_acquire(a.uc_flags + blockIdx.x) - target) < 0) {
      if (globaltimer() - start > a.timeout_ns) {
        *reinterpret_cast<volatile unsigned*>(a.status) = 1u;
        __threadfence_system();
        *abort_flag = 1;
        break;
      }
    }
  }
  __syncthreads();
  return *abort_flag == 0;
}

// Broadcast / AllGather / ReduceScatter through the switch, with the same
// three-buffer scratch, per-block bounded barriers and warp split as the
// AllReduce kernel:
//  Broadcast: the root multicasts round s of its input (multimem.st) while
//    every GPU copies round s-1 out of its scratch; root sends each byte once.
//  AllGather: every rank multicasts its part of round s into its own part of
//    the round buffer; every GPU copies round s-1 (all parts) out.
//  ReduceScatter: every GPU copies round s of its input in; every rank
//    multimem.ld_reduces its own part of round s-1 straight into its output.
template <int U, int DT>
__global__ void __launch_bounds__(768, 1) nvls_xfer_kernel(const __grid_constant__ NvlsArgs a) {
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;
  __syncthreads();
  const int n = a.nranks;
  const bool mover = int(threadIdx.x) < a.movers;  // switch-side warps
  const int t = mover ? threadIdx.x : threadIdx.x - a.movers;
  const int half = mover ? a.movers : int(blockDim.x) - a.movers;  // this group's size
  const float inv = 1.0f / float(n);
  const bool bc = a.mode == int(Kind::Broadcast);
  const unsigned long long part = bc ? a.round : ((a.round / (unsigned long long)n) & ~31ull);
  const unsigned long long total = bc ? a.bytes : a.slot;
  const unsigned long long rounds = (total + part - 1) / part;
  for (unsigned long long s = 0; s < rounds + 1; ++s) {
    if (a.mode == int(Kind::ReduceScatter)) {
      if (!mover && s < rounds) {  // A(s): copy every slot's part of round s in
        const unsigned long long plen = min(part, total - s * part);
        char* buf = a.uc + (s % 3) * a.buf_stride;
        unsigned long long lo, hi;
        flat_portion(plen, &lo, &hi);
        for (int q = 0; q < n; ++q)
          copy16(buf + q * part + lo, a.send + q * a.slot + s * part + lo, hi - lo, t, half);
      }
      if (mover && s >= 1) {  // B(s-1): reduce the own part into the output
        const unsigned long long i = s - 1, plen = min(part, total - i * part);
        const char* mbuf = a.mc + (i % 3) * a.buf_stride + a.rank * part;
        unsigned long long lo, hi;
        flat_portion(plen, &lo, &hi);
        const unsigned long long nv = (hi - lo) / 16;
        for (unsigned long long v = t; v < nv; v += (unsigned long long)half * U) {
          uint4 x[U];
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (v + u * half < nv) x[u] = ld_reduce(mbuf + lo + (v + u * half) * 16, DT);
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (v + u * half < nv)
              __stcs(reinterpret_cast<uint4*>(a.recv + i * part + lo) + v + u * half,
                     a.avg ? scale(x[u], DT, inv) : x[u]);
        }
      }
    } else {
      if (!mover && s >= 1) {  // C(s-1): copy round s-1 out
        const unsigned long long i = s - 1, plen = min(part, total - i * part);
        const char* buf = a.uc + (i % 3) * a.buf_stride;
        unsigned long long lo, hi;
        flat_portion(plen, &lo, &hi);
        if (bc) {
          copy16(a.recv + i * part + lo, buf + lo, hi - lo, t, half);
        } else {
          for (int q = 0; q < n; ++q)
            copy16(a.recv + q * a.slot + i * part + lo, buf + q * part + lo, hi - lo, t, half);
        }
      }
      if (mover && s < rounds && (!bc || a.rank == a.root)) {  // B(s): multicast
        const unsigned long long plen = min(part, total - s * part);
        char* mbuf = a.mc + (s % 3) * a.buf_stride + (bc ? 0 : a.rank * part);
        const char* src = a.send + s * part;
        unsigned long long lo, hi;
        flat_portion(plen, &lo, &hi);
        const unsigned long long nv = (hi - lo) / 16;
        for (unsigned long long v = t; v < nv; v += (unsigned long long)half * U) {
          uint4 x[U];
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (v + u * half < nv) x[u] = __ldcs(reinterpret_cast<const uint4*>(src + lo) + v + u * half);
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (v + u * half < nv) mc_store(mbuf + lo + (v + u * half) * 16, x[u]);
        }
      }
    }
    if (!nvls_barrier(a, s, &abort_flag)) return;
  }
}

// ------------------------------------------------------------------ host side

template <int U>
const void* pick_dtype(bool ar, DType t) {
  constexpr int F = int(DType::F32), B = int(DType::BF16), H = int(DType::F16);
  switch (t) {
    case DType::BF16:
      return ar ? reinterpret_cast<const void*>(nvls_allreduce_kernel<U, B>)
                : reinterpret_cast<const void*>(nvls_xfer_kernel<U, B>);
    case DType::F16:
      return ar ? reinterpret_cast<const void*>(nvls_allreduce_kernel<U, H>)
                : reinterpret_cast<const void*>(nvls_xfer_kernel<U, H>);
    default:  // fp32, and the raw 16-byte copies of AllGather/Broadcast
      return ar ? reinterpret_cast<const void*>(nvls_allreduce_kernel<U, F>)
                : reinterpret_cast<const void*>(nvls_xfer_kernel<U, F>);
  }
}

const void* pick_kernel(bool ar, bool u8, DType t) {
  return u8 ? pick_dtype<8>(ar, t) : pick_dtype<4>(ar, t);
}

template <typename Fn>
Fn drv(const char* name) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return reinterpret_cast<Fn>(fn);
}

struct Driver {
  CUresult (*DeviceGet)(CUdevice*, int) = nullptr;
  CUresult (*DeviceGetAttribute)(int*, CUdevice_attribute, CUdevice) = nullptr;
  CUresult (*MulticastCreate)(CUmemGenericAllocationHandle*, const CUmulticastObjectProp*) = nullptr;
  CUresult (*MulticastAddDevice)(CUmemGenericAllocationHandle, CUdevice) = nullptr;
  CUresult (*MulticastBindMem)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle,
                               size_t, size_t, unsigned long long) = nullptr;
  CUresult (*MulticastGetGranularity)(size_t*, const CUmulticastObjectProp*,
                                      CUmulticastGranularity_flags) = nullptr;
  CUresult (*MemCreate)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*,
                        unsigned long long) = nullptr;
  CUresult (*MemGetAllocationGranularity)(size_t*, const CUmemAllocationProp*,
                                          CUmemAllocationGranularity_flags) = nullptr;
  CUresult (*MemAddressReserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long) = nullptr;
  CUresult (*MemMap)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long) = nullptr;
  CUresult (*MemSetAccess)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t) = nullptr;
  bool ok = false;
};

const Driver& driver() {
  static Driver d = [] {
    Driver x;
    x.DeviceGet = drv<decltype(x.DeviceGet)>("cuDeviceGet");
    x.DeviceGetAttribute = drv<decltype(x.DeviceGetAttribute)>("cuDeviceGetAttribute");
    x.MulticastCreate = drv<decltype(x.MulticastCreate)>("cuMulticastCreate");
    x.MulticastAddDevice = drv<decltype(x.MulticastAddDevice)>("cuMulticastAddDevice");
    x.MulticastBindMem = drv<decltype(x.MulticastBindMem)>("cuMulticastBindMem");
    x.MulticastGetGranularity = drv<decltype(x.MulticastGetGranularity)>("cuMulticastGetGranularity");
    x.MemCreate = drv<decltype(x.MemCreate)>("cuMemCreate");
    x.MemGetAllocationGranularity = drv<decltype(x.MemGetAllocationGranularity)>("cuMemGetAllocationGranularity");
    x.MemAddressReserve = drv<decltype(x.MemAddressReserve)>("cuMemAddressReserve");
    x.MemMap = drv<decltype(x.MemMap)>("cuMemMap");
    x.MemSetAccess = drv<decltype(x.MemSetAccess)>("cuMemSetAccess");
    x.ok = x.DeviceGet && x.DeviceGetAttribute && x.MulticastCreate && x.MulticastAddDevice &&
           x.MulticastBindMem && x.MulticastGetGranularity && x.MemCreate &&
           x.MemGetAllocationGranularity && x.MemAddressReserve && x.MemMap && x.MemSetAccess;
    return x;
  }();
  return d;
}

struct Context {
  std::vector<int> devices;
  size_t round = 0;       // R
  size_t stride = 0;      // distance between round buffers
  size_t size = 0;        // bytes bound per GPU
  std::vector<char*> uc, mc;
  unsigned* status = nullptr;  // mapped pinned host word
  unsigned* status_dev = nullptr;
  unsigned long long barriers = 0;  // per-block barriers run so far on this scratch
  int blocks = 0;
  bool broken = false;
};

std::mutex g_mu;
std::vector<Context*> g_ctx;

Context* find(const int* devices, int n) {
  for (Context* c : g_ctx) {
    if (int(c->devices.size()) != n) continue;
    bool same = true;
    for (int i = 0; i < n; ++i) same &= c->devices[size_t(i)] == devices[i];
    if (same) return c;
  }
  return nullptr;
}

size_t round_up(size_t x, size_t g) { return (x + g - 1) / g * g; }

}  // namespace

bool nvls_supported(const int* devices, int n) {
  static std::mutex mu;
  static std::vector<std::pair<std::vector<int>, bool>> cache;
  std::lock_guard<std::mutex> lk(mu);
  std::vector<int> key(devices, devices + n);
  for (const auto& e : cache)
    if (e.first == key) return e.second;
  const Driver& d = driver();
  bool ok = d.ok && n >= 2;  // cuMulticastCreate rejects a one-device team
  for (int i = 0; ok && i < n; ++i) {
    CUdevice dev;
    int mc = 0;
    ok = d.DeviceGet(&dev, devices[i]) == CUDA_SUCCESS &&
         d.DeviceGetAttribute(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev) == CUDA_SUCCESS && mc;
  }
  {
    std::lock_guard<std::mutex> g(g_mu);
    if (Context* c = find(devices, n)) ok = ok && !c->broken;
  }
  cache.push_back({key, ok});
  return ok;
}

bool nvls_ensure(const int* devices, int n, size_t round_bytes, std::string* why) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (Context* c = find(devices, n)) {
    if (c->broken) {
      if (why) *why = "NVLS disabled after a device timeout";
      return false;
    }
    return true;  // the round size is fixed at creation
  }
  const Driver& d = driver();
  if (!d.ok) {
    if (why) *why = "driver multicast entry points missing";
    return false;
  }
  auto fail = [&](const char* what) {
    if (why) *why = std::string("NVLS setup: ") + what;
    cudaGetLastError();
    return false;
  };
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, devices[0]) != cudaSuccess)
    return fail("SM count");
  const int blocks = sms;  // one resident block per SM (cooperative launch)
  const size_t round = std::max<size_t>(round_bytes / 16 * 16, size_t(n) * size_t(blocks) * 16);
  const size_t stride = round_up(round, 1 << 21);
  const size_t flags_bytes = round_up(size_t(blocks) * sizeof(unsigned), 4096);
  CUmulticastObjectProp mprop{};
  mprop.numDevices = unsigned(n);
  mprop.handleTypes = 0;
  mprop.size = 3 * stride + flags_bytes;
  size_t mgran = 0;
  if (d.MulticastGetGranularity(&mgran, &mprop, CU_MULTICAST_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS)
    return fail("multicast granularity");
  CUmemAllocationProp aprop{};
  aprop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  aprop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  aprop.location.id = devices[0];
  size_t agran = 0;
  if (d.MemGetAllocationGranularity(&agran, &aprop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS)
    return fail("allocation granularity");
  const size_t gran = std::max(mgran, agran);
  const size_t size = round_up(mprop.size, gran);
  mprop.size = size;
  CUmemGenericAllocationHandle mc = 0;
  const CUresult cr = d.MulticastCreate(&mc, &mprop);
  if (cr != CUDA_SUCCESS) {
    char what[96];
    std::snprintf(what, sizeof what, "cuMulticastCreate(devices=%d, size=%zu) returned %d", n, size,
                  int(cr));
    return fail(what);
  }
  for (int i = 0; i < n; ++i) {
    CUdevice dev;
    if (d.DeviceGet(&dev, devices[i]) != CUDA_SUCCESS || d.MulticastAddDevice(mc, dev) != CUDA_SUCCESS)
      return fail("cuMulticastAddDevice");
  }
  Context* c = new Context();
  c->devices.assign(devices, devices + n);
  c->round = round;
  c->stride = stride;
  c->size = size;
  c->blocks = blocks;
  for (int i = 0; i < n; ++i) {
    if (cudaSetDevice(devices[i]) != cudaSuccess) return fail("cudaSetDevice");
    aprop.location.id = devices[i];
    CUmemGenericAllocationHandle phys = 0;
    if (d.MemCreate(&phys, size, &aprop, 0) != CUDA_SUCCESS) return fail("cuMemCreate");
    if (d.MulticastBindMem(mc, 0, phys, 0, size, 0) != CUDA_SUCCESS) return fail("cuMulticastBindMem");
    CUdeviceptr uc = 0, mv = 0;
    CUmemAccessDesc acc{};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = devices[i];
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    if (d.MemAddressReserve(&uc, size, gran, 0, 0) != CUDA_SUCCESS ||
        d.MemMap(uc, size, 0, phys, 0) != CUDA_SUCCESS || d.MemSetAccess(uc, size, &acc, 1) != CUDA_SUCCESS)
      return fail("unicast mapping");
    if (d.MemAddressReserve(&mv, size, gran, 0, 0) != CUDA_SUCCESS ||
        d.MemMap(mv, size, 0, mc, 0) != CUDA_SUCCESS || d.MemSetAccess(mv, size, &acc, 1) != CUDA_SUCCESS)
      return fail("multicast mapping");
    c->uc.push_back(reinterpret_cast<char*>(uc));
    c->mc.push_back(reinterpret_cast<char*>(mv));
    if (cudaMemset(reinterpret_cast<char*>(uc) + 3 * stride, 0, flags_bytes) != cudaSuccess)
      return fail("flag init");
  }
  for (int i = 0; i < n; ++i)
    if (cudaSetDevice(devices[i]) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
      return fail("setup drain");
  if (cudaHostAlloc(reinterpret_cast<void**>(&c->status), sizeof(unsigned), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess ||
      cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->status_dev), c->status, 0) != cudaSuccess)
    return fail("status word");
  *c->status = 0;
  g_ctx.push_back(c);
  return true;
}

cudaError_t nvls_launch(const PlanOp& op, const Plan& plan, const Binding& b, const Policy& p,
                        cudaStream_t s, int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  Context* c = find(b.device, b.nranks);
  if (!c || c->broken) return cudaErrorNotSupported;
  const int r = op.stream.dev;
  if (r == 0 && *static_cast<volatile unsigned*>(c->status) != 0) {
    c->broken = true;  // a previous gang timed out: flags are no longer in step
    return cudaErrorLaunchTimeout;
  }
  if (plan.desc.bytes % 16 != 0) return cudaErrorInvalidValue;
  NvlsArgs a{};
  a.send = static_cast<const char*>(b.send[r]);
  a.recv = static_cast<char*>(b.recv[r]);
  a.uc = c->uc[size_t(r)];
  a.mc = c->mc[size_t(r)];
  a.uc_flags = reinterpret_cast<unsigned*>(a.uc + 3 * c->stride);
  a.mc_flags = reinterpret_cast<unsigned*>(a.mc + 3 * c->stride);
  a.bytes = plan.desc.bytes;
  a.round = c->round;
  a.buf_stride = c->stride;
  a.timeout_ns = p.device_timeout_ns;
  a.status = c->status_dev;
  a.base = unsigned(c->barriers * (unsigned long long)b.nranks) + p.test_nvls_skew;
  a.nranks = b.nranks;
  a.rank = r;
  a.dtype = int(plan.desc.dtype);
  a.avg = plan.desc.op == RedOp::Avg;
  a.mode = int(plan.desc.kind);
  a.root = plan.desc.root;
  a.slot = plan.desc.bytes;  // AG send slot / RS receive slot
  (void)dev;
  const bool ar = plan.desc.kind == Kind::AllReduce;
  // Barriers this call runs (one per step); every rank runs the same count.
  unsigned long long steps = 0;
  if (ar) {
    steps = (a.bytes + a.round - 1) / a.round + 2;
  } else {
    const bool bc = plan.desc.kind == Kind::Broadcast;
    const unsigned long long part = bc ? a.round : ((a.round / (unsigned long long)b.nranks) & ~31ull);
    steps = (plan.desc.bytes + part - 1) / part + 1;
    if (!bc && part == 0) return cudaErrorInvalidValue;
  }
  const int threads = p.nvls_threads;
  a.movers = std::min(p.nvls_movers, threads - 128);
  void* argv[] = {&a};
  const void* fn = pick_kernel(ar, p.nvls_unroll >= 8, plan.desc.dtype);
  const cudaError_t e =
      cudaLaunchCooperativeKernel(fn, dim3(unsigned(c->blocks)), dim3(unsigned(threads)), argv, 0, s);
  if (r == b.nranks - 1) c->barriers += steps;
  return e;
}

unsigned nvls_status(const int* devices, int n) {
  std::lock_guard<std::mutex> lk(g_mu);
  Context* c = find(devices, n);
  return c && c->status ? *static_cast<volatile unsigned*>(c->status) : 0u;
}

}  // namespace nb
