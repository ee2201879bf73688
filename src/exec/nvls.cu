// NVLS collectives: multicast objects over the clique's GPUs and the
// multimem kernels.
//
// Setup (once per device set): one multicast object spans every clique GPU;
// each GPU binds its own physical scratch (cuMemCreate) into it and maps
// both a unicast view (its own memory) and a multicast view. The scratch
// holds K round buffers of R bytes (K >= 3) plus progress words per block;
// round s uses buffer s % K. By default K covers the largest message the
// interposer takes (8 GiB), so no call reuses a buffer: reuse within a call
// (K = 3) failed the round-reuse edge stress on the GPU although every wait
// the protocol needs is in place.
//
// Kernels (one per GPU; those launched for one call form a gang): the
// message is processed in rounds of R bytes. In a block, mover warps work
// through the switch (multimem.ld_reduce, accumulating 16-bit types in fp32,
// and multimem.st, which writes every GPU's scratch) while copier warps
// stream rounds between the user's buffers and this GPU's scratch. The two
// groups synchronize only through per-(block, group, rank) progress words,
// each waiting for exactly the steps it consumes, so neither waits on the
// other group's unrelated work. Every wait is bounded by %globaltimer: on
// expiry the kernel writes a status word in mapped host memory and returns;
// the host turns it into ncclUnhandledCudaError and disables the route.
// By default the copier warps use system-scope loads and stores on the
// scratch side (ld/st.relaxed.sys); on request (NCCL_B200_NVLS_STRONG=0)
// the copier group runs as one warp of TMA bulk copies (cp.async.bulk
// global -> shared on an mbarrier, shared -> global in bulk groups). Either
// reads and writes only this GPU's own memory (the user's buffers and the
// unicast view of its scratch). No load with cluster multicast is used.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "core/nvls_sched.h"
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
  unsigned nbuf;             // K round buffers; round s uses buffer s % K
  int ahead;                 // AllReduce copier: every copy-in first (only when rounds <= K)
  unsigned long long timeout_ns;
  unsigned* status;          // mapped host word: nonzero = a wait expired
  unsigned base;             // progress epoch before this call
  unsigned skew;             // added to every wait target (bounded-wait test only)
  int nranks, rank, dtype;
  int scaled;                // multiply the switch's sum by `mul` (Avg, PreMulSum)
  int tma;                   // copier group: TMA bulk pipeline (one warp) instead of SM copies
  int ramp;                  // AllReduce: ramped first and last rounds (see ar_round)
  int strong;                // SM copier: strong (system-scope) accesses to the scratch
  float mul;
  int movers;                // threads of a block that work through the switch
  int mode;                  // collective kind (xfer kernel)
  int root;                  // Broadcast
  unsigned long long slot;   // AllGather / ReduceScatter bytes per slot to move
  unsigned long long slot_stride;  // distance between consecutive slots
  unsigned long long* trace; // per-block phase timing record, or null
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

// Copy `bytes` (a multiple of 16, below 4 GiB) with the `nthreads` threads of
// a warp group (thread index t): 32-byte vectors, U in flight per thread,
// when both ends allow; else 16-byte vectors. Full groups of U run without
// predicates; 32-bit indices keep the loop within the 768-thread register
// budget (80 per thread).
__device__ __forceinline__ void copy16(char* dst, const char* src, unsigned long long bytes, int t,
                                       int nthreads) {
  constexpr int U = 4;
  unsigned n32 = 0;
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 31) == 0) {
    n32 = unsigned(bytes / 32);
    const unsigned nt = unsigned(nthreads);
    unsigned i = unsigned(t);
    for (; i + nt * (U - 1) < n32; i += nt * U) {
      V32 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = ld32(src + size_t(i + u * nt) * 32);
#pragma unroll
      for (int u = 0; u < U; ++u) st32(dst + size_t(i + u * nt) * 32, v[u]);
    }
    for (; i < n32; i += nt) st32(dst + size_t(i) * 32, ld32(src + size_t(i) * 32));
  }
  const size_t done = size_t(n32) * 32;
  const unsigned n16 = unsigned((bytes - done) / 16);
  const uint4* s16 = reinterpret_cast<const uint4*>(src + done);
  uint4* d16 = reinterpret_cast<uint4*>(dst + done);
  const unsigned nt = unsigned(nthreads);
  unsigned i = unsigned(t);
  for (; i + nt < n16; i += 2 * nt) {
    const uint4 a = __ldcs(s16 + i), b = __ldcs(s16 + i + nt);
    __stcs(d16 + i, a);
    __stcs(d16 + i + nt, b);
  }
  if (i < n16) __stcs(d16 + i, __ldcs(s16 + i));
}

// copy16 with system-scope relaxed (strong) accesses on one side: `mode` 1
// loads the source strongly, 2 stores the destination strongly. Used for the
// scratch side of the SM copier: the scratch is also written and read through
// the switch, and weak accesses may be served from, or left in, a cache the
// switch traffic does not see.
__device__ __forceinline__ void copy16_strong(char* dst, const char* src, unsigned long long bytes, int t,
                                              int nthreads, int mode) {
  constexpr int U = 4;
  const unsigned n16 = unsigned(bytes / 16);
  const unsigned nt = unsigned(nthreads);
  auto ld = [&](unsigned i) {
    uint4 v;
    const void* p = src + size_t(i) * 16;
    if (mode == 1)
      asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    else
      v = __ldcs(reinterpret_cast<const uint4*>(p));
    return v;
  };
  auto st = [&](unsigned i, uint4 v) {
    void* p = dst + size_t(i) * 16;
    if (mode == 2)
      asm volatile("st.relaxed.sys.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                   "r"(v.w) : "memory");
    else
      __stcs(reinterpret_cast<uint4*>(p), v);
  };
  unsigned i = unsigned(t);
  for (; i + nt * (U - 1) < n16; i += nt * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = ld(i + u * nt);
#pragma unroll
    for (int u = 0; u < U; ++u) st(i + u * nt, v[u]);
  }
  for (; i < n16; i += nt) st(i, ld(i));
}

// Calls st(i, ld(i)) for i = t, t + nt, ... below n, with the U loads of a
// group issued before its U stores (U requests in flight per thread).
template <int U, typename Ld, typename St>
__device__ __forceinline__ void strided(unsigned t, unsigned nt, unsigned n, Ld ld, St st) {
  unsigned i = t;
  for (; i + nt * (U - 1) < n; i += nt * U) {
    uint4 x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) x[u] = ld(i + u * nt);
#pragma unroll
    for (int u = 0; u < U; ++u) st(i + u * nt, x[u]);
  }
  for (; i < n; i += nt) st(i, ld(i));
}

// ---------------------------------------------------------------- progress
//
// The two warp groups of a block run decoupled pipelines and wait only for
// what they consume. Each block has, on every GPU, one progress word per
// (group, rank): flag(g, q) = epoch + the number of steps group g of this
// block index on rank q has completed. A group leader publishes its progress
// with one multicast store (release, system scope) after the group's
// bar.sync and a system fence, so every GPU's copy of the word advances; a
// waiting leader polls its own GPU's words with acquire loads, then releases
// its group with bar.sync. Values only grow (the host advances the epoch by
// the largest step count of each call), so a wait is "every listed rank
// reached v". Every wait is bounded by %globaltimer: on expiry the leader
// sets the status word in mapped host memory and the shared abort flag, and
// both groups return at their next wait.
constexpr int kMover = 0, kCopier = 1;

__device__ __forceinline__ unsigned flag_index(int group, int q) {
  return (blockIdx.x * 2u + unsigned(group)) * unsigned(kMaxRanks) + unsigned(q);
}

__device__ __forceinline__ void group_sync(bool mover, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(mover ? 1 : 2), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void mc_publish(unsigned* p, unsigned v) {
  asm volatile("multimem.st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Per-thread view of its warp group. `tr` (shared, leader only) accumulates
// the optional phase timing: [0] busy, [1] waiting, [2] last mark, [3] start.
struct Grp {
  bool mover;
  int t, nt;
  bool leader;
  volatile int* abort;
  unsigned long long* tr;
};

__device__ __forceinline__ Grp make_group(const NvlsArgs& a, int* abort_flag,
                                          unsigned long long (*trace_sh)[4]) {
  Grp g;
  g.mover = int(threadIdx.x) < a.movers;
  g.t = g.mover ? int(threadIdx.x) : int(threadIdx.x) - a.movers;
  g.nt = g.mover ? a.movers : int(blockDim.x) - a.movers;
  g.leader = g.t == 0;
  g.abort = abort_flag;
  g.tr = a.trace ? trace_sh[g.mover ? 0 : 1] : nullptr;
  return g;
}

// Leader: wait until flag(group, q) >= v on every rank q (only `only` when
// it is >= 0), then release the group. False for every thread of the group
// when a wait expired here or the other group aborted.
__device__ bool group_wait(const NvlsArgs& a, const Grp& g, int group, unsigned v, int only) {
  if (g.leader) {
    const unsigned long long t0 = globaltimer();
    if (g.tr) g.tr[0] += t0 - g.tr[2];
    const unsigned target = v + a.skew;
    for (int q = 0; q < a.nranks; ++q) {
      if (only >= 0 && q != only) continue;
      const unsigned* f = a.uc_flags + flag_index(group, q);
      while (int(ld_acquire(f) - target) < 0) {
        if (*g.abort) break;
        if (globaltimer() - t0 > a.timeout_ns) {
          *reinterpret_cast<volatile unsigned*>(a.status) = 1u;  // mapped host word
          __threadfence_system();
          *g.abort = 1;
          break;
        }
      }
      if (*g.abort) break;
    }
    if (g.tr) {
      const unsigned long long t1 = globaltimer();
      g.tr[1] += t1 - t0;
      g.tr[2] = t1;
    }
  }
  group_sync(g.mover, g.nt);
  return *g.abort == 0;
}

// The group finished a step: its writes are ordered before the leader's
// release of flag(own group, this rank) = v on every GPU.
__device__ __forceinline__ void group_publish(const NvlsArgs& a, const Grp& g, unsigned v) {
  group_sync(g.mover, g.nt);
  if (g.leader && !*g.abort) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    mc_publish(a.mc_flags + flag_index(g.mover ? kMover : kCopier, a.rank), v);
  }
}

// Optional per-block phase timing (NCCL_B200_NVLS_TRACE): each leader adds
// {busy, waiting, total} ns of its group to the block's record
// {mover busy, mover wait, copier busy, copier wait, mover total, copier total}.
__device__ __forceinline__ void trace_begin(const Grp& g) {
  if (g.tr && g.leader) {
    g.tr[0] = g.tr[1] = 0;
    g.tr[2] = g.tr[3] = globaltimer();
  }
}
__device__ __forceinline__ void trace_end(const NvlsArgs& a, const Grp& g) {
  if (!g.tr || !g.leader) return;
  const unsigned long long t = globaltimer();
  unsigned long long* rec = a.trace + 8ull * blockIdx.x;
  const int o = g.mover ? 0 : 2;
  rec[o] += g.tr[0] + (t - g.tr[2]);
  rec[o + 1] += g.tr[1];
  rec[4 + (g.mover ? 0 : 1)] += t - g.tr[3];
}

// ------------------------------------------------------------- TMA copier
//
// The copier group's data movement runs on the tensor memory accelerator:
// one thread streams each copy through shared memory in 16 KiB chunks with
// cp.async.bulk (global -> shared, completing on an mbarrier) and
// cp.async.bulk (shared -> global, bulk groups), eight stages deep. Up to
// 128 KiB per SM are in flight without occupying registers, which is what
// HBM needs beside the switch traffic. No cluster multicast is used. The
// scratch is also read and written by the switch (generic proxy), so the
// thread fences the async proxy after acquiring a round and before
// publishing one. Every wait is bounded by %globaltimer.
constexpr int kStages = 8;
constexpr unsigned kChunk = 16384;
constexpr size_t kTmaSmem = size_t(kStages) * kChunk;

struct Bulk {
  bool on;
  unsigned smem;   // shared address of stage 0
  unsigned bar;    // shared address of the first of kStages mbarriers
  char** dst;      // shared: destination of the chunk held by each stage
  unsigned* size;  // shared: its size
  unsigned long long issued, stored;
};

__device__ __forceinline__ unsigned shared_addr(const void* p) {
  return unsigned(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void fence_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ bool bulk_ready(const Bulk& b, unsigned long long k) {
  unsigned done;
  asm volatile(
      "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(done)
      : "r"(b.bar + 8u * unsigned(k % kStages)), "r"(unsigned((k / kStages) & 1))
      : "memory");
  return done != 0;
}

__device__ __forceinline__ void expire(const NvlsArgs& a, volatile int* abort) {
  *reinterpret_cast<volatile unsigned*>(a.status) = 1u;
  __threadfence_system();
  *abort = 1;
}

// Issue the store of the oldest loaded chunk (waiting, bounded, for its load).
__device__ bool bulk_retire(const NvlsArgs& a, Bulk& b, volatile int* abort) {
  const unsigned long long k = b.stored;
  const unsigned long long t0 = globaltimer();
  while (!bulk_ready(b, k)) {
    if (globaltimer() - t0 > a.timeout_ns) {
      expire(a, abort);
      return false;
    }
  }
  const unsigned st = unsigned(k % kStages);
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(b.dst[st]),
               "r"(b.smem + st * kChunk), "r"(b.size[st])
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  ++b.stored;
  return true;
}

// Wait until at most `pending` of the most recent stores still read shared
// memory (the instruction takes the count as an immediate).
__device__ __forceinline__ void bulk_wait_read(unsigned pending) {
  switch (pending) {
    case 0: asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.bulk.wait_group.read 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.bulk.wait_group.read 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.bulk.wait_group.read 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.bulk.wait_group.read 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.bulk.wait_group.read 6;" ::: "memory"); break;
    default: asm volatile("cp.async.bulk.wait_group.read 7;" ::: "memory"); break;
  }
}

// Queue the copy src -> dst (16-byte aligned, a multiple of 16 bytes).
__device__ bool bulk_push(const NvlsArgs& a, Bulk& b, char* dst, const char* src,
                          unsigned long long bytes, volatile int* abort) {
  for (unsigned long long off = 0; off < bytes; off += kChunk) {
    const unsigned size = unsigned(min((unsigned long long)kChunk, bytes - off));
    const unsigned long long k = b.issued;
    const unsigned st = unsigned(k % kStages);
    if (k >= kStages) {
      // The stage last held chunk k - kStages: its store must have been
      // issued and must have finished reading shared memory.
      const unsigned long long j = k - kStages;
      while (b.stored <= j)
        if (!bulk_retire(a, b, abort)) return false;
      bulk_wait_read(unsigned(b.stored - 1 - j));
    }
    const unsigned bar = b.bar + 8u * st;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(size) : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            b.smem + st * kChunk),
        "l"(src + off), "r"(size), "r"(bar)
        : "memory");
    b.dst[st] = dst + off;
    b.size[st] = size;
    ++b.issued;
    while (b.stored < b.issued && bulk_ready(b, b.stored))
      if (!bulk_retire(a, b, abort)) return false;
  }
  return true;
}

// Complete every queued copy: all stores issued and written to global
// memory, and ordered before later generic-proxy accesses.
__device__ bool bulk_drain(const NvlsArgs& a, Bulk& b, volatile int* abort) {
  bool ok = true;
  while (ok && b.stored < b.issued) ok = bulk_retire(a, b, abort);
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  fence_async_global();
  return ok;
}

// Before leaving the kernel: wait (bounded) for loads still in flight, then
// for every store.
__device__ void bulk_finish(const NvlsArgs& a, Bulk& b) {
  const unsigned long long t0 = globaltimer();
  for (unsigned long long k = b.stored; k < b.issued; ++k)
    while (!bulk_ready(b, k) && globaltimer() - t0 < a.timeout_ns) {
    }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// The copier group's view of its mover: the TMA pipeline (its leader alone
// issues) or, when off, the SM copy loop over all copier threads.
template <bool TMA>
struct Copier {
  Bulk b;
  const NvlsArgs* a;
  const Grp* g;
  __device__ Copier(const NvlsArgs& args, const Grp& grp, unsigned char* dsmem,
                    unsigned long long* bars, char** dsts, unsigned* sizes)
      : a(&args), g(&grp) {
    b.on = TMA && args.tma != 0;
    b.smem = shared_addr(dsmem);
    b.bar = shared_addr(bars);
    b.dst = dsts;
    b.size = sizes;
    b.issued = b.stored = 0;
    if (b.on && grp.leader && !grp.mover) {
      for (int i = 0; i < kStages; ++i)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(b.bar + 8u * unsigned(i)) : "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
  }
  // A round was acquired: later bulk loads must see what the switch wrote.
  __device__ void acquired() {
    if (b.on && g->leader) fence_async_global();
  }
  // `scratch`: 1 when the source is the scratch, 2 when the destination is.
  __device__ void copy(char* dst, const char* src, unsigned long long bytes, int scratch = 0) {
    if (!b.on) {
      if (a->strong && scratch)
        copy16_strong(dst, src, bytes, g->t, g->nt, scratch);
      else
        copy16(dst, src, bytes, g->t, g->nt);
      return;
    }
    if (!g->leader || *g->abort) return;
    if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | bytes) & 15) != 0) {
      copy16(dst, src, bytes, 0, 1);  // never taken: the gate admits 16-byte aligned calls only
      return;
    }
    bulk_push(*a, b, dst, src, bytes, g->abort);
  }
  // Before publishing a step.
  __device__ void flush() {
    if (b.on && g->leader && !*g->abort) bulk_drain(*a, b, g->abort);
  }
  __device__ void finish() {
    if (b.on && g->leader) bulk_finish(*a, b);
  }
};

// AllReduce. Warp specialization: movers reduce through the switch
// (NVLink-bound), copiers stream rounds in and out of the scratch
// (HBM-bound). Rounds (ar_round) cut into N slices; rank r owns slice r.
//   copier step s: A(s); publish s+1; then C(s-2) after every rank's B(s-2).
//   mover  step s: B(s) after every rank's A(s); publish s+1.
// A(s) reuses buffer s%3: every rank's B(s-3) is done (waited for before
// C(s-3), in the previous step) and so is this rank's C(s-3) (its loads
// complete before any later store is issued; the SM copier syncs the group).
// B(s) stores into every rank's buffer s%3 after that rank's A(s), hence
// after its C(s-3). Copy-in first keeps the copier up to two rounds ahead
// of the movers: after B(s-2) it has C(s-2) and A(s+1) to do while the
// movers run B(s-1) and B(s). U: multimem requests in flight per thread.
template <int U, int DT, bool TMA>
__global__ void __launch_bounds__(TMA ? 640 : 768, 1) nvls_allreduce_kernel(const __grid_constant__ NvlsArgs a) {
  extern __shared__ __align__(128) unsigned char dsmem[];
  __shared__ int abort_flag;
  __shared__ unsigned long long trace_sh[2][4];
  __shared__ __align__(8) unsigned long long tma_bar[kStages];
  __shared__ char* tma_dst[kStages];
  __shared__ unsigned tma_size[kStages];
  if (threadIdx.x == 0) abort_flag = 0;
  const Grp g = make_group(a, &abort_flag, trace_sh);
  trace_begin(g);
  __syncthreads();
  const int n = a.nranks;
  const unsigned rounds = ar_rounds(a.bytes, a.round, a.ramp);
  if (g.mover) {
    for (unsigned s = 0; s < rounds; ++s) {
      if (!group_wait(a, g, kCopier, a.base + s + 1, -1)) return;
      unsigned long long rbase, rlen, lo, hi;
      ar_round(s, a.bytes, a.round, a.ramp, &rbase, &rlen);
      portion(rlen, n, a.rank, &lo, &hi);
      char* base = a.mc + (s % a.nbuf) * a.buf_stride + lo;
      strided<U>(
          unsigned(g.t), unsigned(g.nt), unsigned((hi - lo) / 16),
          [&](unsigned v) { return ld_reduce(base + size_t(v) * 16, DT); },
          [&](unsigned v, uint4 x) { mc_store(base + size_t(v) * 16, a.scaled ? scale(x, DT, a.mul) : x); });
      group_publish(a, g, a.base + s + 1);
    }
  } else {
    Copier<TMA> cp(a, g, dsmem, tma_bar, tma_dst, tma_size);
    // With a buffer per round, copy every round in first (the movers never
    // wait for a copy-in after the first round), then copy each round out
    // once every rank's movers finished it.
    const bool ahead = a.ahead && rounds <= a.nbuf;
    for (unsigned s = 0; ahead && s < rounds; ++s) {
      unsigned long long rbase, rlen;
      ar_round(s, a.bytes, a.round, a.ramp, &rbase, &rlen);
      char* buf = a.uc + (s % a.nbuf) * a.buf_stride;
      for (int q = 0; q < n; ++q) {
        unsigned long long lo, hi;
        portion(rlen, n, q, &lo, &hi);
        cp.copy(buf + lo, a.send + rbase + lo, hi - lo, 2);
      }
      cp.flush();
      group_publish(a, g, a.base + s + 1);
    }
    for (unsigned s = 0; ahead && s < rounds; ++s) {
      if (!group_wait(a, g, kMover, a.base + s + 1, -1)) break;
      cp.acquired();
      unsigned long long rbase, rlen;
      ar_round(s, a.bytes, a.round, a.ramp, &rbase, &rlen);
      const char* buf = a.uc + (s % a.nbuf) * a.buf_stride;
      for (int q = 0; q < n; ++q) {
        unsigned long long lo, hi;
        portion(rlen, n, q, &lo, &hi);
        cp.copy(a.recv + rbase + lo, buf + lo, hi - lo, 1);
      }
    }
    for (unsigned s = 0; !ahead && s < rounds + 2; ++s) {
      if (s >= 2) {
        if (!group_wait(a, g, kMover, a.base + s - 1, -1)) break;
        cp.acquired();
        const unsigned i = s - 2;
        unsigned long long rbase, rlen;
        ar_round(i, a.bytes, a.round, a.ramp, &rbase, &rlen);
        const char* buf = a.uc + (i % a.nbuf) * a.buf_stride;
        for (int q = 0; q < n; ++q) {
          unsigned long long lo, hi;
          portion(rlen, n, q, &lo, &hi);
          cp.copy(a.recv + rbase + lo, buf + lo, hi - lo, 1);
        }
      }
      if (s < rounds) {
        unsigned long long rbase, rlen;
        ar_round(s, a.bytes, a.round, a.ramp, &rbase, &rlen);
        char* buf = a.uc + (s % a.nbuf) * a.buf_stride;
        for (int q = 0; q < n; ++q) {
          unsigned long long lo, hi;
          portion(rlen, n, q, &lo, &hi);
          cp.copy(buf + lo, a.send + rbase + lo, hi - lo, 2);
        }
      }
      cp.flush();
      group_publish(a, g, a.base + s + 1);
    }
    cp.flush();
    cp.finish();
  }
  trace_end(a, g);
}

// This block's part [lo, hi) of a flat range of `len` bytes (16-byte units).
__device__ __forceinline__ void flat_portion(unsigned long long len, unsigned long long* lo,
                                             unsigned long long* hi) {
  const unsigned long long per = ((len + gridDim.x - 1) / gridDim.x + 31) & ~31ull;
  *lo = min(len, per * blockIdx.x);
  *hi = min(len, *lo + per);
}

// Broadcast / AllGather / ReduceScatter through the switch, with the same
// K-buffer scratch, decoupled groups and bounded waits:
//  ReduceScatter: copier A(s) copies every slot's part of round s in (after
//    every rank's B(s-K), the last reader of buffer s%K); mover B(s), after
//    every rank's A(s), multimem.ld_reduces its own part into its output.
//  AllGather: mover B(s) multicasts its slot's part of round s into every
//    rank's buffer (after every rank's C(s-K)); copier C(s), after every
//    rank's B(s), copies all parts out.
//  Broadcast: the root's movers multicast round s (after every rank's
//    C(s-K)); copiers copy round s out after the root's B(s). The root
//    sends each byte once.
template <int U, int DT, bool TMA>
__global__ void __launch_bounds__(TMA ? 640 : 768, 1) nvls_xfer_kernel(const __grid_constant__ NvlsArgs a) {
  extern __shared__ __align__(128) unsigned char dsmem[];
  __shared__ int abort_flag;
  __shared__ unsigned long long trace_sh[2][4];
  __shared__ __align__(8) unsigned long long tma_bar[kStages];
  __shared__ char* tma_dst[kStages];
  __shared__ unsigned tma_size[kStages];
  if (threadIdx.x == 0) abort_flag = 0;
  const Grp g = make_group(a, &abort_flag, trace_sh);
  trace_begin(g);
  __syncthreads();
  Copier<TMA> cp(a, g, dsmem, tma_bar, tma_dst, tma_size);
  const int n = a.nranks;
  const bool bc = a.mode == int(Kind::Broadcast);
  const bool rs = a.mode == int(Kind::ReduceScatter);
  const unsigned long long part = bc ? a.round : ((a.round / (unsigned long long)n) & ~31ull);
  const unsigned long long total = bc ? a.bytes : a.slot;
  const unsigned rounds = unsigned((total + part - 1) / part);
  for (unsigned s = 0; s < rounds; ++s) {
    const unsigned long long plen = min(part, total - s * part);
    unsigned long long lo, hi;
    flat_portion(plen, &lo, &hi);
    if (rs) {
      if (g.mover) {
        if (!group_wait(a, g, kCopier, a.base + s + 1, -1)) return;
        const char* base = a.mc + (s % a.nbuf) * a.buf_stride + a.rank * part + lo;
        uint4* out = reinterpret_cast<uint4*>(a.recv + s * part + lo);
        strided<U>(
            unsigned(g.t), unsigned(g.nt), unsigned((hi - lo) / 16),
            [&](unsigned v) { return ld_reduce(base + size_t(v) * 16, DT); },
            [&](unsigned v, uint4 x) { __stcs(out + v, a.scaled ? scale(x, DT, a.mul) : x); });
      } else {
        if (s >= a.nbuf && !group_wait(a, g, kMover, a.base + s - a.nbuf + 1, -1)) break;
        cp.acquired();
        char* buf = a.uc + (s % a.nbuf) * a.buf_stride;
        for (int q = 0; q < n; ++q)
          cp.copy(buf + q * part + lo, a.send + q * a.slot_stride + s * part + lo, hi - lo, 2);
        cp.flush();
      }
    } else if (g.mover) {
      if (bc && a.rank != a.root) break;  // only the root's movers send
      if (s >= a.nbuf && !group_wait(a, g, kCopier, a.base + s - a.nbuf + 1, -1)) return;
      char* base = a.mc + (s % a.nbuf) * a.buf_stride + (bc ? 0 : a.rank * part) + lo;
      const uint4* in = reinterpret_cast<const uint4*>(a.send + s * part + lo);
      strided<U>(
          unsigned(g.t), unsigned(g.nt), unsigned((hi - lo) / 16),
          [&](unsigned v) { return __ldcs(in + v); },
          [&](unsigned v, uint4 x) { mc_store(base + size_t(v) * 16, x); });
    } else {
      if (!group_wait(a, g, kMover, a.base + s + 1, bc ? a.root : -1)) break;
      cp.acquired();
      const char* buf = a.uc + (s % a.nbuf) * a.buf_stride;
      if (bc) {
        cp.copy(a.recv + s * part + lo, buf + lo, hi - lo, 1);
      } else {
        for (int q = 0; q < n; ++q)
          cp.copy(a.recv + q * a.slot_stride + s * part + lo, buf + q * part + lo, hi - lo, 1);
      }
      cp.flush();
    }
    group_publish(a, g, a.base + s + 1);
  }
  if (!g.mover) cp.finish();
  trace_end(a, g);
}

// ------------------------------------------------------------------ host side

template <int U, bool TMA>
const void* pick_dtype(bool ar, DType t) {
  constexpr int F = int(DType::F32), B = int(DType::BF16), H = int(DType::F16);
  switch (t) {
    case DType::BF16:
      return ar ? reinterpret_cast<const void*>(nvls_allreduce_kernel<U, B, TMA>)
                : reinterpret_cast<const void*>(nvls_xfer_kernel<U, B, TMA>);
    case DType::F16:
      return ar ? reinterpret_cast<const void*>(nvls_allreduce_kernel<U, H, TMA>)
                : reinterpret_cast<const void*>(nvls_xfer_kernel<U, H, TMA>);
    default:  // fp32, and the raw 16-byte copies of AllGather/Broadcast
      return ar ? reinterpret_cast<const void*>(nvls_allreduce_kernel<U, F, TMA>)
                : reinterpret_cast<const void*>(nvls_xfer_kernel<U, F, TMA>);
  }
}

const void* pick_kernel(bool ar, bool u8, bool tma, DType t) {
  if (tma) return u8 ? pick_dtype<8, true>(ar, t) : pick_dtype<4, true>(ar, t);
  return u8 ? pick_dtype<8, false>(ar, t) : pick_dtype<4, false>(ar, t);
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
  unsigned nbuf = 3;      // round buffers
  size_t size = 0;        // bytes bound per GPU
  std::vector<char*> uc, mc;
  unsigned* status = nullptr;  // mapped pinned host word
  unsigned* status_dev = nullptr;
  unsigned long long epoch = 0;  // progress value every flag reached after the last call
  std::vector<unsigned long long*> trace;  // per device: blocks x 8 phase-time records
  bool tma_ok = true;  // every device admits the TMA copier's shared memory
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

bool nvls_ensure(const int* devices, int n, size_t round_bytes, int nbuf, std::string* why) {
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
  const size_t flags_bytes = round_up(size_t(blocks) * 2 * kMaxRanks * sizeof(unsigned), 4096);
  CUmulticastObjectProp mprop{};
  mprop.numDevices = unsigned(n);
  mprop.handleTypes = 0;
  const unsigned K = unsigned(std::max(3, nbuf));
  mprop.size = size_t(K) * stride + flags_bytes;
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
  c->nbuf = K;
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
    if (cudaMemset(reinterpret_cast<char*>(uc) + size_t(K) * stride, 0, flags_bytes) != cudaSuccess)
      return fail("flag init");
    unsigned long long* tr = nullptr;
    const size_t tr_bytes = size_t(blocks) * 8 * sizeof(unsigned long long);
    if (cudaMalloc(&tr, tr_bytes) != cudaSuccess || cudaMemset(tr, 0, tr_bytes) != cudaSuccess)
      return fail("trace records");
    c->trace.push_back(tr);
    // The TMA copier stages through 128 KiB of dynamic shared memory.
    for (int ar = 0; ar < 2; ++ar)
      for (int u8 = 0; u8 < 2; ++u8)
        for (DType t : {DType::F32, DType::BF16, DType::F16})
          if (cudaFuncSetAttribute(pick_kernel(ar, u8, true, t), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   int(kTmaSmem)) != cudaSuccess) {
            cudaGetLastError();
            c->tma_ok = false;
          }
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
  const bool ar = plan.desc.kind == Kind::AllReduce;
  const bool rs = plan.desc.kind == Kind::ReduceScatter;
  // An AllReduce gang covers the op's range of the buffers, a ReduceScatter
  // gang that range of every slot (the hybrid routes give the switch a
  // leading share); the other kinds the message.
  const size_t off = ar || rs ? op.src[0].off : 0;
  const size_t range = ar || rs ? op.bytes : plan.desc.bytes;
  if (off % 16 != 0 || range % 16 != 0) return cudaErrorInvalidValue;
  const unsigned grid = op.grid ? std::min<unsigned>(op.grid, unsigned(c->blocks)) : unsigned(c->blocks);
  NvlsArgs a{};
  a.send = static_cast<const char*>(b.send[r]) + off;
  a.recv = static_cast<char*>(b.recv[r]) + off;
  a.uc = c->uc[size_t(r)];
  a.mc = c->mc[size_t(r)];
  a.uc_flags = reinterpret_cast<unsigned*>(a.uc + size_t(c->nbuf) * c->stride);
  a.mc_flags = reinterpret_cast<unsigned*>(a.mc + size_t(c->nbuf) * c->stride);
  a.nbuf = c->nbuf;
  a.ahead = (op.nvls_ahead ? op.nvls_ahead == 2 : p.nvls_ahead) ? 1 : 0;
  a.bytes = ar ? range : plan.desc.bytes;
  // A smaller round than the scratch holds (a tuned kernel shape) uses the
  // same buffers; 32-byte multiples of every slice stay aligned.
  a.round = op.nvls_round && op.nvls_round < c->round
                ? std::max<size_t>(op.nvls_round / 32 * 32, size_t(b.nranks) * size_t(c->blocks) * 32)
                : c->round;
  a.buf_stride = c->stride;
  a.timeout_ns = p.device_timeout_ns;
  a.status = c->status_dev;
  a.base = unsigned(c->epoch);
  a.skew = p.test_nvls_skew;
  a.nranks = b.nranks;
  a.rank = r;
  a.dtype = int(plan.desc.dtype);
  a.scaled = plan.desc.op == RedOp::Avg || plan.desc.op == RedOp::PreMulSum;
  a.mul = plan.desc.op == RedOp::Avg ? 1.0f / float(b.nranks) : float(plan.desc.scalar);
  a.mode = int(plan.desc.kind);
  a.root = plan.desc.root;
  a.slot = rs ? range : plan.desc.bytes;  // AG send slot / RS part of each receive slot
  a.slot_stride = plan.desc.bytes;
  a.trace = p.nvls_trace ? c->trace[size_t(r)] : nullptr;
  // The largest progress value this call publishes (every rank the same):
  // the next call's epoch.
  unsigned long long steps = 0;
  a.ramp = ar && (op.nvls_ramp ? op.nvls_ramp == 2 : p.nvls_ramp) ? 1 : 0;
  // A shape that would need more rounds than the scratch has buffers (a
  // smaller round, the ramp) would reuse buffers within the call: take the
  // scratch's own round, uniform, instead.
  if (ar && ar_rounds(a.bytes, a.round, a.ramp) > c->nbuf) {
    a.round = c->round;
    a.ramp = 0;
  }
  if (ar) {
    steps = ar_rounds(a.bytes, a.round, a.ramp) + 2ull;
  } else {
    const bool bc = plan.desc.kind == Kind::Broadcast;
    const unsigned long long part = bc ? a.round : ((a.round / (unsigned long long)b.nranks) & ~31ull);
    if (part == 0) return cudaErrorInvalidValue;
    steps = ((bc ? plan.desc.bytes : a.slot) + part - 1) / part;
  }
  // TMA copier: the movers plus one copier warp, with the staging buffers
  // in dynamic shared memory; SM copier: the configured split.
  a.strong = p.nvls_strong ? 1 : 0;
  a.tma = p.nvls_tma && c->tma_ok && !a.strong ? 1 : 0;
  const int movers = op.nvls_movers ? int(op.nvls_movers) : p.nvls_movers;
  const int unroll = op.nvls_unroll ? int(op.nvls_unroll) : p.nvls_unroll;
  const int threads = a.tma ? std::min(movers, 608) + 32 : p.nvls_threads;
  a.movers = a.tma ? threads - 32 : std::min(movers, threads - 128);
  const size_t smem = a.tma ? kTmaSmem : 0;
  void* argv[] = {&a};
  const void* fn = pick_kernel(ar, unroll >= 8, a.tma != 0, plan.desc.dtype);
  (void)dev;
  const cudaError_t e =
      cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(unsigned(threads)), argv, smem, s);
  if (r == b.nranks - 1) c->epoch += steps;
  return e;
}

int nvls_trace_read(const int* devices, int n, int rank, double out[6], bool reset) {
  std::lock_guard<std::mutex> lk(g_mu);
  Context* c = find(devices, n);
  if (!c || rank < 0 || rank >= n) return -1;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(devices[rank]) != cudaSuccess) return -1;
  std::vector<unsigned long long> rec(size_t(c->blocks) * 8);
  const size_t bytes = rec.size() * sizeof(unsigned long long);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(rec.data(), c->trace[size_t(rank)], bytes, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && reset) e = cudaMemset(c->trace[size_t(rank)], 0, bytes);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return -1;
  // Mean over the blocks that ran: a launch with a smaller grid (the hybrid
  // route gives the switch part of the SMs) leaves the other records zero.
  int ran = 0;
  double sum[6] = {};
  for (int b = 0; b < c->blocks; ++b) {
    const unsigned long long* r = &rec[size_t(b) * 8];
    if (!(r[0] | r[1] | r[2] | r[3] | r[4] | r[5])) continue;
    ++ran;
    for (int k = 0; k < 6; ++k) sum[k] += double(r[k]);
  }
  for (int k = 0; k < 6; ++k) out[k] = ran ? sum[k] / double(ran) : 0.0;  // ns
  return ran;
}

unsigned nvls_status(const int* devices, int n) {
  std::lock_guard<std::mutex> lk(g_mu);
  Context* c = find(devices, n);
  return c && c->status ? *static_cast<volatile unsigned*>(c->status) : 0u;
}

bool nvls_scratch(const int* devices, int n, size_t* bytes, unsigned* buffers, size_t* round) {
  std::lock_guard<std::mutex> lk(g_mu);
  Context* c = find(devices, n);
  if (!c) return false;
  *bytes = c->size;
  *buffers = c->nbuf;
  *round = c->round;
  return true;
}

}  // namespace nb
