// sm_100a collective kernels: fused multi-source reduce-and-push and
// multi-segment pull copies over NVLink peer memory.
//
// Reduce kernel: thread i folds 16-byte vector i of every source in source
// (= rank) order, accumulating in fp32 for fp16/bf16/fp32 (fp64 for doubles,
// the type's own width with wrap-around for integers), applies the op's
// finalization (average, pre-multiplied scalars) and stores the converted
// result to every destination. Sources and destinations are plain global
// pointers: local HBM or a peer GPU's HBM through NVLink/NVSwitch. Each
// thread keeps ~8 independent 16-byte loads in flight to cover the NVLink
// round trip. The per-element arithmetic is exactly the host fold's
// (hostreduce.cc), so the host oracle is bit-exact.
//
// Copy kernel: a flat tile space over up to 8 (src, dst, len) segments;
// every block takes 64 KiB tiles round-robin, so pulls from different peers
// proceed concurrently. One large copy within a GPU (a one-rank collective)
// runs on the stream copy kernel, or on the TMA bulk copy when its ends are
// only 16-byte aligned.
//
// Parity: replaces the reference's shim_reduce_write_vector /
// shim_reduce_write_tail (shim/nccl_collectives_shim.cu:772-851) and its
// copy-engine peer copies (:1156).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "kernels/fold.cuh"
#include "kernels/kernels.h"

namespace nb {
namespace {

using namespace kfold;

struct KReduceArgs {
  const void* src[kMaxRanks];
  void* dst[kMaxRanks];
  const void* dev_scalar[kMaxRanks];
  double scale[kMaxRanks];
  unsigned long long nvec;       // whole 16-byte vectors
  unsigned long long tail_elems; // trailing elements after the vectors
  int ndst;
  int op;
  int nranks;
};

struct KCopyArgs {
  const void* src[kMaxRanks];
  void* dst[kMaxRanks];
  unsigned long long len[kMaxRanks];
  unsigned long long tile_start[kMaxRanks + 1];  // prefix sums of tiles per segment
  int nseg;
};

constexpr int kTileBytes = 64 * 1024;

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_stream(void* p, uint4 v) {
  __stcs(reinterpret_cast<uint4*>(p), v);
}

template <typename T>
__device__ __forceinline__ typename Acc<T>::type load_scale(const KReduceArgs& a, int s) {
  using A = typename Acc<T>::type;
  if (a.dev_scalar[s]) return to_acc<T>(*reinterpret_cast<const T*>(a.dev_scalar[s]));
  return A(a.scale[s]);
}

// A VB-byte vector (16: ld/st.global.v4; 32: the sm_100 256-bit
// ld/st.global.v8, which halves the request count on NVLink).
template <int VB>
struct VecT {
  uint4 h[VB / 16];
};

template <int VB>
__device__ __forceinline__ VecT<VB> ldv(const VecT<VB>* p) {
  VecT<VB> v;
  if constexpr (VB == 32) {
    asm volatile("ld.global.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v.h[0].x), "=r"(v.h[0].y), "=r"(v.h[0].z), "=r"(v.h[0].w), "=r"(v.h[1].x),
                   "=r"(v.h[1].y), "=r"(v.h[1].z), "=r"(v.h[1].w)
                 : "l"(p));
  } else {
    v.h[0] = __ldcs(reinterpret_cast<const uint4*>(p));
  }
  return v;
}

template <int VB>
__device__ __forceinline__ void stv(VecT<VB>* p, const VecT<VB>& v) {
  if constexpr (VB == 32) {
    asm volatile("st.global.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.h[0].x),
                 "r"(v.h[0].y), "r"(v.h[0].z), "r"(v.h[0].w), "r"(v.h[1].x), "r"(v.h[1].y),
                 "r"(v.h[1].z), "r"(v.h[1].w)
                 : "memory");
  } else {
    __stcs(reinterpret_cast<uint4*>(p), v.h[0]);
  }
}

template <typename T, int NSRC, int VB>
__global__ void __launch_bounds__(512, VB == 32 ? 1 : 2) reduce_kernel(const __grid_constant__ KReduceArgs a) {
  using A = typename Acc<T>::type;
  using V = VecT<VB>;
  // About eight 16-byte loads in flight per thread.
  constexpr int U = (8 * 16 / VB / NSRC) > 0 ? (8 * 16 / VB / NSRC) : 1;
  A s[NSRC];
#pragma unroll
  for (int k = 0; k < NSRC; ++k) s[k] = load_scale<T>(a, k);
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  const unsigned long long tid = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (unsigned long long base = tid; base < a.nvec; base += stride * U) {
    V v[U][NSRC];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const unsigned long long idx = base + u * stride;
      if (idx < a.nvec) {
#pragma unroll
        for (int k = 0; k < NSRC; ++k) v[u][k] = ldv<VB>(static_cast<const V*>(a.src[k]) + idx);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const unsigned long long idx = base + u * stride;
      if (idx < a.nvec) {
        V out;
#pragma unroll
        for (int j = 0; j < VB / 16; ++j) {
          uint4 part[NSRC];
#pragma unroll
          for (int k = 0; k < NSRC; ++k) part[k] = v[u][k].h[j];
          out.h[j] = fold_vec<T, NSRC>(part, a.op, a.nranks, s);
        }
        for (int d = 0; d < a.ndst; ++d) stv<VB>(static_cast<V*>(a.dst[d]) + idx, out);
      }
    }
  }
  // Trailing elements that do not fill a vector.
  if (blockIdx.x == 0 && threadIdx.x < a.tail_elems) {
    const unsigned long long e = a.nvec * (VB / sizeof(T)) + threadIdx.x;
    A acc = first<T>(static_cast<const T*>(a.src[0])[e], a.op, s[0]);
#pragma unroll
    for (int k = 1; k < NSRC; ++k) acc = combine<T>(acc, static_cast<const T*>(a.src[k])[e], a.op, s[k]);
    const T out = finish<T>(acc, a.op, a.nranks);
    for (int d = 0; d < a.ndst; ++d) static_cast<T*>(a.dst[d])[e] = out;
  }
}

// Local bulk copy on the tensor memory accelerator: one thread per block
// streams 32 KiB chunks through four shared-memory stages with cp.async.bulk
// (global -> shared completing on an mbarrier, shared -> global in bulk
// groups), so 128 KiB per SM are in flight without occupying registers.
// Both buffers are this GPU's own memory (no peer memory, no cluster
// multicast). Every wait is bounded by %globaltimer; a wait that expires
// sets a status word in mapped host memory (tma_copy_status) and the block
// stops after its copies in flight have landed. That last wait is bounded
// too (twice the timeout): the loads in flight read this GPU's own memory
// and land within microseconds on a working GPU, so one still outstanding
// after seconds means the device itself is failing, which the status word
// already reports; every wait in this library has a bound.
constexpr int kTmaStages = 4;
constexpr unsigned kTmaChunk = 32768;
constexpr size_t kTmaCopySmem = size_t(kTmaStages) * kTmaChunk;

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_done(unsigned bar, unsigned parity) {
  unsigned done;
  asm volatile(
      "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

__global__ void __launch_bounds__(32, 1) tma_copy_kernel(const char* src, char* dst, unsigned long long len,
                                                         unsigned long long timeout_ns, unsigned* status) {
  extern __shared__ __align__(128) unsigned char stage[];
  __shared__ __align__(8) unsigned long long bars[kTmaStages];
  const unsigned long long body = len & ~15ull;
  const unsigned long long nchunks = (body + kTmaChunk - 1) / kTmaChunk;
  if (threadIdx.x == 0) {
    const unsigned smem = unsigned(__cvta_generic_to_shared(stage));
    const unsigned bar0 = unsigned(__cvta_generic_to_shared(bars));
    for (int i = 0; i < kTmaStages; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8u * unsigned(i)) : "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    // This block's chunks: blockIdx.x, blockIdx.x + gridDim.x, ...; the i-th
    // of them uses stage i % kTmaStages.
    unsigned long long mine = nchunks > blockIdx.x ? (nchunks - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    unsigned long long issued = 0, stored = 0;
    const unsigned long long t0 = now_ns();
    bool ok = true;
    auto chunk_off = [&](unsigned long long i) { return (blockIdx.x + i * gridDim.x) * (unsigned long long)kTmaChunk; };
    auto retire = [&]() {
      const unsigned st = unsigned(stored % kTmaStages);
      while (!mbar_done(bar0 + 8u * st, unsigned((stored / kTmaStages) & 1)))
        if (now_ns() - t0 > timeout_ns) return false;
      const unsigned long long off = chunk_off(stored);
      const unsigned size = unsigned(min((unsigned long long)kTmaChunk, body - off));
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst + off),
                   "r"(smem + st * kTmaChunk), "r"(size)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      ++stored;
      return true;
    };
    while (ok && issued < mine) {
      if (issued >= kTmaStages) {
        const unsigned long long j = issued - kTmaStages;  // the stage's previous chunk
        while (ok && stored <= j) ok = retire();
        // That chunk's store must have finished reading shared memory; the
        // stores issued after it may still be reading.
        switch (unsigned(stored - 1 - j)) {
          case 0: asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); break;
          case 1: asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); break;
          case 2: asm volatile("cp.async.bulk.wait_group.read 2;" ::: "memory"); break;
          default: asm volatile("cp.async.bulk.wait_group.read 3;" ::: "memory"); break;
        }
      }
      if (!ok) break;
      const unsigned st = unsigned(issued % kTmaStages);
      const unsigned long long off = chunk_off(issued);
      const unsigned size = unsigned(min((unsigned long long)kTmaChunk, body - off));
      const unsigned bar = bar0 + 8u * st;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(size) : "memory");
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              smem + st * kTmaChunk),
          "l"(src + off), "r"(size), "r"(bar)
          : "memory");
      ++issued;
      // Store every chunk whose load already landed, so stores start early.
      while (ok && stored < issued &&
             mbar_done(bar0 + 8u * unsigned(stored % kTmaStages), unsigned((stored / kTmaStages) & 1)))
        ok = retire();
    }
    while (ok && stored < issued) ok = retire();
    if (!ok) {
      *reinterpret_cast<volatile unsigned*>(status) = 1u;
      __threadfence_system();
    }
    // On a timeout, let loads still in flight land before the block exits.
    for (unsigned long long k = stored; !ok && k < issued; ++k)
      while (!mbar_done(bar0 + 8u * unsigned(k % kTmaStages), unsigned((k / kTmaStages) & 1)) &&
             now_ns() - t0 < 2 * timeout_ns) {
      }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  // Bytes after the last whole 16-byte unit.
  if (blockIdx.x == 0)
    for (unsigned long long i = body + threadIdx.x; i < len; i += blockDim.x) dst[i] = src[i];
}

// Local stream copy: one large copy within this GPU's memory, both ends
// 32-byte aligned. Every thread keeps 16 independent 32-byte loads in flight
// (512 bytes; 128 KiB per 256-thread block) before storing them, over a grid
// of four blocks per SM that strides through the buffer. Measured on B200 at
// 8 GiB this moves 6.69 TB/s (read + write), above a copy-engine copy
// (6.67 TB/s) and the TMA bulk pipeline (6.20 TB/s), which keeps fewer bytes
// in flight per SM. Loads skip L1 (each byte is read once).
constexpr int kStreamU = 16;
constexpr int kStreamThreads = 256;
constexpr int kStreamBlocksPerSm = 4;

struct Words8 {
  unsigned r[8];
};

__device__ __forceinline__ Words8 ld_once(const Words8* p) {
  Words8 v;
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.r[0]), "=r"(v.r[1]), "=r"(v.r[2]), "=r"(v.r[3]), "=r"(v.r[4]), "=r"(v.r[5]),
                 "=r"(v.r[6]), "=r"(v.r[7])
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_words8(Words8* p, const Words8& v) {
  asm volatile("st.global.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.r[0]), "r"(v.r[1]),
               "r"(v.r[2]), "r"(v.r[3]), "r"(v.r[4]), "r"(v.r[5]), "r"(v.r[6]), "r"(v.r[7])
               : "memory");
}

// Bytes after the last whole 32-byte vector (block 0 only).
__device__ __noinline__ void copy_byte_tail(const char* src, char* dst, unsigned long long from,
                                            unsigned long long len) {
  for (unsigned long long b = from + threadIdx.x; b < len; b += blockDim.x) dst[b] = src[b];
}

__global__ void stream_copy_kernel(const char* src, char* dst, unsigned long long len) {
  const unsigned long long nvec = len / 32;
  const Words8* s = reinterpret_cast<const Words8*>(src);
  Words8* d = reinterpret_cast<Words8*>(dst);
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long base = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; base < nvec;
       base += stride * kStreamU) {
    Words8 v[kStreamU];
#pragma unroll
    for (int u = 0; u < kStreamU; ++u) {
      const unsigned long long i = base + u * stride;
      if (i < nvec) v[u] = ld_once(s + i);
    }
#pragma unroll
    for (int u = 0; u < kStreamU; ++u) {
      const unsigned long long i = base + u * stride;
      if (i < nvec) st_words8(d + i, v[u]);
    }
  }
  if (blockIdx.x == 0 && nvec * 32 < len) copy_byte_tail(src, dst, nvec * 32, len);
}

// Tiles are interleaved across segments (tile t belongs to segment t % nseg)
// so that at any moment every source is being read: pulls from several peers
// spread over all their links instead of queueing on one peer at a time.
__global__ void __launch_bounds__(512) copy_kernel(const __grid_constant__ KCopyArgs a) {
  unsigned long long rounds = 0;
  for (int i = 0; i < a.nseg; ++i)
    rounds = max(rounds, a.tile_start[i + 1] - a.tile_start[i]);
  const unsigned long long tiles = rounds * (unsigned long long)a.nseg;
  for (unsigned long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int s = int(t % (unsigned long long)a.nseg);
    const unsigned long long round = t / (unsigned long long)a.nseg;
    if (round >= a.tile_start[s + 1] - a.tile_start[s]) continue;
    const unsigned long long lo = round * kTileBytes;
    const unsigned long long hi = min(lo + (unsigned long long)kTileBytes, a.len[s]);
    const char* src = static_cast<const char*>(a.src[s]) + lo;
    char* dst = static_cast<char*>(a.dst[s]) + lo;
    const unsigned long long n = hi - lo;
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 31) == 0) {
      using V = VecT<32>;
      const unsigned long long nvec = n / 32;
      constexpr int U = 4;
      for (unsigned long long base = threadIdx.x; base < nvec; base += blockDim.x * U) {
        V v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const unsigned long long i = base + u * blockDim.x;
          if (i < nvec) v[u] = ldv<32>(reinterpret_cast<const V*>(src) + i);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const unsigned long long i = base + u * blockDim.x;
          if (i < nvec) stv<32>(reinterpret_cast<V*>(dst) + i, v[u]);
        }
      }
      for (unsigned long long i = nvec * 32 + threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
    } else if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
      const unsigned long long nvec = n / 16;
      constexpr int U = 8;
      for (unsigned long long base = threadIdx.x; base < nvec; base += blockDim.x * U) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const unsigned long long i = base + u * blockDim.x;
          if (i < nvec) v[u] = ld_stream(reinterpret_cast<const uint4*>(src) + i);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const unsigned long long i = base + u * blockDim.x;
          if (i < nvec) st_stream(reinterpret_cast<uint4*>(dst) + i, v[u]);
        }
      }
      for (unsigned long long i = nvec * 16 + threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
    } else if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | n) & 3) == 0) {
      const unsigned long long nw = n / 4;
      for (unsigned long long i = threadIdx.x; i < nw; i += blockDim.x)
        reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
    } else {
      for (unsigned long long i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
    }
  }
}

using ReduceFn = void (*)(KReduceArgs);

template <typename T, int VB = 16>
ReduceFn reduce_for(int nsrc) {
  switch (nsrc) {
    case 1: return reduce_kernel<T, 1, VB>;
    case 2: return reduce_kernel<T, 2, VB>;
    case 3: return reduce_kernel<T, 3, VB>;
    case 4: return reduce_kernel<T, 4, VB>;
    case 5: return reduce_kernel<T, 5, VB>;
    case 6: return reduce_kernel<T, 6, VB>;
    case 7: return reduce_kernel<T, 7, VB>;
    case 8: return reduce_kernel<T, 8, VB>;
    default: return nullptr;
  }
}

// 32-byte vectors for the hot floating types when every operand allows it.
ReduceFn pick_reduce(DType t, int nsrc, bool wide) {
  switch (t) {
    case DType::F32: return wide ? reduce_for<float, 32>(nsrc) : reduce_for<float>(nsrc);
    case DType::F16: return wide ? reduce_for<__half, 32>(nsrc) : reduce_for<__half>(nsrc);
    case DType::BF16:
      return wide ? reduce_for<__nv_bfloat16, 32>(nsrc) : reduce_for<__nv_bfloat16>(nsrc);
    case DType::F64: return reduce_for<double>(nsrc);
    case DType::I8: return reduce_for<int8_t>(nsrc);
    case DType::U8: return reduce_for<uint8_t>(nsrc);
    case DType::I32: return reduce_for<int32_t>(nsrc);
    case DType::U32: return reduce_for<uint32_t>(nsrc);
    case DType::I64: return reduce_for<int64_t>(nsrc);
    case DType::U64: return reduce_for<uint64_t>(nsrc);
    default: return nullptr;
  }
}

}  // namespace

LaunchShape shape_for(size_t bytes, int sm_count, int blocks_per_sm, int threads) {
  LaunchShape s;
  s.threads = threads;
  const size_t per_block = size_t(threads) * 16 * 8;
  const size_t want = (bytes + per_block - 1) / per_block;
  const size_t cap = size_t(std::max(1, sm_count) * std::max(1, blocks_per_sm));
  s.blocks = int(std::max<size_t>(1, std::min(want, cap)));
  return s;
}

cudaError_t launch_reduce(const ReduceLaunch& r, LaunchShape shape, cudaStream_t stream) {
  const size_t es = elem_size(r.fold.dtype);
  if (!es || r.nsrc < 1 || r.nsrc > kMaxRanks || r.ndst < 1 || r.ndst > kMaxRanks ||
      r.bytes % es)
    return cudaErrorInvalidValue;
  if (r.bytes == 0) return cudaSuccess;
  // The kernel issues 16- or 32-byte vector accesses: refuse (never launch)
  // any operand that is not 16-byte aligned; use 32 when all are 32-aligned.
  uintptr_t any = 0;
  for (int i = 0; i < r.nsrc; ++i) any |= reinterpret_cast<uintptr_t>(r.src[i]);
  for (int i = 0; i < r.ndst; ++i) any |= reinterpret_cast<uintptr_t>(r.dst[i]);
  if (any % 16) return cudaErrorMisalignedAddress;
  const bool hot = r.fold.dtype == DType::F32 || r.fold.dtype == DType::BF16 || r.fold.dtype == DType::F16;
  const bool wide = hot && any % 32 == 0;
  const int vb = wide ? 32 : 16;
  const ReduceFn fn = pick_reduce(r.fold.dtype, r.nsrc, wide);
  if (!fn) return cudaErrorInvalidValue;
  KReduceArgs k{};
  for (int i = 0; i < r.nsrc; ++i) {
    k.src[i] = r.src[i];
    k.dev_scalar[i] = r.dev_scalar[i];
    k.scale[i] = r.fold.scalars[i];
  }
  for (int i = 0; i < r.ndst; ++i) k.dst[i] = r.dst[i];
  k.nvec = r.bytes / vb;
  k.tail_elems = (r.bytes - k.nvec * vb) / es;
  k.ndst = r.ndst;
  k.op = int(r.fold.op);
  k.nranks = r.fold.nranks;
  void* argv[] = {&k};
  return cudaLaunchKernel(reinterpret_cast<const void*>(fn), dim3(unsigned(shape.blocks)),
                          dim3(unsigned(shape.threads)), argv, 0, stream);
}

namespace {
std::mutex g_tma_status_mu;
unsigned* g_tma_status_host = nullptr;
unsigned* g_tma_status_dev = nullptr;

// The bulk copy's status word: pinned, mapped host memory (portable across
// devices), allocated once.
unsigned* tma_status_word() {
  std::lock_guard<std::mutex> lk(g_tma_status_mu);
  if (!g_tma_status_host) {
    unsigned* h = nullptr;
    unsigned* d = nullptr;
    if (cudaHostAlloc(reinterpret_cast<void**>(&h), sizeof(unsigned),
                      cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess)
      return nullptr;
    if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&d), h, 0) != cudaSuccess) {
      cudaFreeHost(h);
      return nullptr;
    }
    *h = 0;
    g_tma_status_host = h;
    g_tma_status_dev = d;
  }
  return g_tma_status_dev;
}
}  // namespace

bool tma_copy_prepare() { return tma_status_word() != nullptr; }

unsigned tma_copy_status() {
  std::lock_guard<std::mutex> lk(g_tma_status_mu);
  return g_tma_status_host ? *static_cast<volatile unsigned*>(g_tma_status_host) : 0u;
}

cudaError_t launch_copy(const CopyLaunch& c, LaunchShape shape, cudaStream_t stream) {
  if (c.nseg < 1 || c.nseg > kMaxRanks) return cudaErrorInvalidValue;
  const uintptr_t ends = reinterpret_cast<uintptr_t>(c.src[0]) | reinterpret_cast<uintptr_t>(c.dst[0]);
  const bool big_local = c.local && c.nseg == 1 && c.len[0] >= (4u << 20);
  // One large copy within this GPU's memory: the stream copy kernel when
  // both ends are 32-byte aligned (unless the TMA engine is asked for).
  if (big_local && (ends & 31) == 0 && !c.prefer_tma) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const char* src = static_cast<const char*>(c.src[0]);
    char* dst = static_cast<char*>(c.dst[0]);
    unsigned long long len = c.len[0];
    void* argv[] = {&src, &dst, &len};
    return cudaLaunchKernel(reinterpret_cast<const void*>(stream_copy_kernel),
                            dim3(unsigned(std::max(1, sms) * kStreamBlocksPerSm)), dim3(kStreamThreads), argv,
                            0, stream);
  }
  // Otherwise, 16-byte aligned: the TMA bulk copy.
  if (big_local && (ends & 15) == 0) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // The kernel's shared-memory opt-in, once per device (repeating it is harmless).
    static std::atomic<bool> opted[64];
    if (e == cudaSuccess && (dev >= 64 || !opted[dev].load(std::memory_order_acquire))) {
      e = cudaFuncSetAttribute(reinterpret_cast<const void*>(tma_copy_kernel),
                               cudaFuncAttributeMaxDynamicSharedMemorySize, int(kTmaCopySmem));
      if (e == cudaSuccess && dev < 64) opted[dev].store(true, std::memory_order_release);
    }
    if (e != cudaSuccess) return e;
    unsigned* status = tma_status_word();
    if (!status) return cudaErrorMemoryAllocation;
    const unsigned long long timeout_ns = 2000000000ull;
    const char* src = static_cast<const char*>(c.src[0]);
    char* dst = static_cast<char*>(c.dst[0]);
    unsigned long long len = c.len[0];
    void* argv[] = {&src, &dst, &len, const_cast<unsigned long long*>(&timeout_ns), &status};
    return cudaLaunchKernel(reinterpret_cast<const void*>(tma_copy_kernel), dim3(unsigned(sms)), dim3(32),
                            argv, kTmaCopySmem, stream);
  }
  KCopyArgs k{};
  k.nseg = c.nseg;
  unsigned long long tiles = 0;
  for (int i = 0; i < c.nseg; ++i) {
    k.src[i] = c.src[i];
    k.dst[i] = c.dst[i];
    k.len[i] = c.len[i];
    k.tile_start[i] = tiles;
    tiles += (c.len[i] + kTileBytes - 1) / kTileBytes;
  }
  k.tile_start[c.nseg] = tiles;
  if (!tiles) return cudaSuccess;
  const unsigned blocks = unsigned(std::min<unsigned long long>(tiles, (unsigned long long)shape.blocks));
  void* argv[] = {&k};
  return cudaLaunchKernel(reinterpret_cast<const void*>(copy_kernel), dim3(blocks),
                          dim3(unsigned(shape.threads)), argv, 0, stream);
}

}  // namespace nb
