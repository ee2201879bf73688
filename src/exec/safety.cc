// Runtime safety checks run before a clique call is planned.
//
// Capture: the custom schedules use cross-device event dependencies and
// internal streams that a per-stream graph capture cannot represent, so a
// capturing caller stream (or one whose state cannot be read) falls back to
// NCCL.
//
// Buffers: the driver's facts about the first and the last byte (one batched
// pointer-attribute query each, plus the per-device access query for VMM
// memory) are classified by the pure rule table of core/bufclass.h; an
// ordinary buffer also needs every clique device to be peer-capable with its
// owner. Accepted buffers are remembered by allocation id (see VerdictKey).
//
// Parity: pair_capturing / supported_buffer of the reference
// (shim/nccl_collectives_shim.cu:1619-1705), which check a device pair's
// buffers by the same attributes.
#include <cuda.h>

#include "core/bufclass.h"
#include "exec/executor.h"

namespace nb {

bool stream_capturing(cudaStream_t s, int dev) {
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusActive;
  unsigned long long id = 0;
  const bool known = cudaSetDevice(dev) == cudaSuccess && cudaStreamGetCaptureInfo(s, &status, &id) == cudaSuccess;
  if (!known) cudaGetLastError();
  return !known || status != cudaStreamCaptureStatusNone;
}

namespace {

// Driver entry points, resolved once through the runtime (no link-time
// dependency on libcuda).
struct PointerApi {
  CUresult (*attributes)(unsigned, CUpointer_attribute*, void**, CUdeviceptr) = nullptr;
  CUresult (*access)(unsigned long long*, const CUmemLocation*, CUdeviceptr) = nullptr;
  bool ready() const { return attributes && access; }
};

template <typename Fn>
void resolve(const char* name, Fn& out) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    out = reinterpret_cast<Fn>(fn);
  else
    cudaGetLastError();
}

const PointerApi& pointer_api() {
  static const PointerApi api = [] {
    PointerApi a;
    resolve("cuPointerGetAttributes", a.attributes);
    resolve("cuMemGetAccess", a.access);
    return a;
  }();
  return api;
}

Access access_of(CUresult r, unsigned long long flags) {
  if (r == CUDA_ERROR_INVALID_VALUE) return Access::NoMapping;  // not a VMM mapping
  if (r != CUDA_SUCCESS) return Access::QueryFailed;
  if (flags == 0) return Access::NoFlags;
  return flags == CU_MEM_ACCESS_FLAGS_PROT_READWRITE ? Access::ReadWrite : Access::OtherFlags;
}

// Facts about the byte at p. The per-device access query matters only for
// VMM memory (not legacy-IPC capable): ordinary cudaMalloc memory has no
// per-device mapping to report, so for it the query is skipped and recorded
// as NoMapping, which saves N driver calls per endpoint on every call.
PointerFacts facts_at(const PointerApi& api, CUdeviceptr p, const int* devices, int n) {
  PointerFacts f;
  unsigned memtype = 0;
  int ordinal = -1, legacy = -1;
  CUmemoryPool pool = nullptr;
  uintptr_t start = 0, mstart = 0;
  size_t size = 0, msize = 0;
  CUpointer_attribute which[] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE,     CU_POINTER_ATTRIBUTE_DEVICE_ORDINAL,
                                 CU_POINTER_ATTRIBUTE_IS_LEGACY_CUDA_IPC_CAPABLE,
                                 CU_POINTER_ATTRIBUTE_MEMPOOL_HANDLE,  CU_POINTER_ATTRIBUTE_RANGE_START_ADDR,
                                 CU_POINTER_ATTRIBUTE_RANGE_SIZE,      CU_POINTER_ATTRIBUTE_MAPPING_BASE_ADDR,
                                 CU_POINTER_ATTRIBUTE_MAPPING_SIZE};
  void* out[] = {&memtype, &ordinal, &legacy, &pool, &start, &size, &mstart, &msize};
  // An address the driver does not know still answers CUDA_SUCCESS, with
  // memory type 0.
  if (api.attributes(unsigned(sizeof(which) / sizeof(which[0])), which, out, p) != CUDA_SUCCESS) return f;
  f.known = memtype != 0;
  f.device_memory = memtype == CU_MEMORYTYPE_DEVICE;
  f.device = ordinal;
  f.legacy_ipc = legacy;
  f.from_pool = pool != nullptr;
  f.range_start = start;
  f.range_size = size;
  f.mapping_start = mstart;
  f.mapping_size = msize;
  f.ndev = n;
  for (int i = 0; i < n; ++i) {
    if (f.legacy_ipc == 1) {
      f.access[i] = Access::NoMapping;
      continue;
    }
    CUmemLocation where{};
    where.type = CU_MEM_LOCATION_TYPE_DEVICE;
    where.id = devices[i];
    unsigned long long flags = 0;
    f.access[i] = access_of(api.access(&flags, &where, p), flags);
  }
  return f;
}

}  // namespace

namespace {

// Verdicts already reached, keyed by everything they depend on: the range,
// the owning device, the clique's devices, and the allocation's process-wide
// buffer id (a freed and re-made allocation at the same address gets a new
// id, so a stale verdict is never reused). A hit costs one attribute query
// instead of the full set; calls are serialized by the interposer's
// executor lock.
struct VerdictKey {
  uintptr_t ptr = 0;
  size_t bytes = 0;
  unsigned long long buffer_id = 0;
  int dev = -1, n = 0;
  int devices[kMaxRanks] = {};
  bool operator==(const VerdictKey& o) const {
    if (ptr != o.ptr || bytes != o.bytes || buffer_id != o.buffer_id || dev != o.dev || n != o.n) return false;
    for (int i = 0; i < n; ++i)
      if (devices[i] != o.devices[i]) return false;
    return true;
  }
};

constexpr size_t kVerdictSlots = 64;
VerdictKey g_verdicts[kVerdictSlots];
size_t g_verdict_next = 0;

bool verdict_known(const VerdictKey& k) {
  for (const VerdictKey& v : g_verdicts)
    if (v == k) return true;
  return false;
}

void remember_verdict(const VerdictKey& k) {
  g_verdicts[g_verdict_next] = k;
  g_verdict_next = (g_verdict_next + 1) % kVerdictSlots;
}

unsigned long long buffer_id_of(const PointerApi& api, CUdeviceptr p) {
  unsigned long long id = 0;
  CUpointer_attribute which[] = {CU_POINTER_ATTRIBUTE_BUFFER_ID};
  void* out[] = {&id};
  return api.attributes(1, which, out, p) == CUDA_SUCCESS ? id : 0;
}

}  // namespace

bool supported_buffer(const void* ptr, size_t bytes, int dev, const int* devices, int n) {
  const PointerApi& api = pointer_api();
  if (!api.ready() || bytes == 0 || n < 1 || n > kMaxRanks) return false;
  VerdictKey key;
  key.ptr = reinterpret_cast<uintptr_t>(ptr);
  key.bytes = bytes;
  key.dev = dev;
  key.n = n;
  for (int i = 0; i < n; ++i) key.devices[i] = devices[i];
  key.buffer_id = buffer_id_of(api, static_cast<CUdeviceptr>(key.ptr));
  if (key.buffer_id != 0 && verdict_known(key)) return true;
  const auto first = static_cast<CUdeviceptr>(reinterpret_cast<uintptr_t>(ptr));
  if (bytes - 1 > ~CUdeviceptr(0) - first) return false;
  const PointerFacts a = facts_at(api, first, devices, n);
  const PointerFacts b = facts_at(api, first + bytes - 1, devices, n);
  const BufferVerdict v = classify_buffer(a, b, first, bytes, dev);
  if (v.cls == BufferClass::Mapped) {
    if (key.buffer_id) remember_verdict(key);
    return true;
  }
  if (v.cls != BufferClass::Ordinary) return false;
  // Ordinary memory is reached through peer access, which setup enabled for
  // every pair that supports it.
  for (int i = 0; i < n; ++i) {
    int can = devices[i] == dev ? 1 : 0;
    if (!can && (cudaDeviceCanAccessPeer(&can, devices[i], dev) != cudaSuccess || !can)) {
      cudaGetLastError();
      return false;
    }
  }
  if (key.buffer_id) remember_verdict(key);
  return true;
}

}  // namespace nb
