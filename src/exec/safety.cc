// Runtime safety checks run before a clique call is planned.
//
// Capture: the custom schedules use cross-device event dependencies and
// internal streams that a per-stream graph capture cannot represent, so a
// capturing (or unknown-state) caller stream falls back to NCCL.
//
// Buffers: classified by queried properties, failing closed on any
// ambiguity: device memory of the expected device; one allocation covers
// both ends; not from a stream-ordered memory pool (pool memory is not made
// peer-accessible by cudaDeviceEnablePeerAccess); either VMM memory mapped
// READWRITE for every clique device, or ordinary cudaMalloc memory (legacy
// IPC capable) whose peers have peer access enabled.
//
// Parity: pair_capturing / supported_buffer of the reference
// (shim/nccl_collectives_shim.cu:1619-1705), for two fixed devices.
#include <cuda.h>

#include "exec/executor.h"

namespace nb {

bool stream_capturing(cudaStream_t s, int dev) {
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  if (cudaSetDevice(dev) != cudaSuccess || cudaStreamIsCapturing(s, &status) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return status != cudaStreamCaptureStatusNone;
}

namespace {

using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
using AttrFn = CUresult (*)(void*, CUpointer_attribute, CUdeviceptr);
using AccessFn = CUresult (*)(unsigned long long*, const CUmemLocation*, CUdeviceptr);

template <typename Fn>
Fn driver_fn(const char* name) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return reinterpret_cast<Fn>(fn);
}

}  // namespace

bool supported_buffer(const void* ptr, size_t bytes, int dev, const int* devices, int n) {
  cudaPointerAttributes attributes{};
  if (cudaPointerGetAttributes(&attributes, ptr) != cudaSuccess ||
      attributes.type != cudaMemoryTypeDevice || attributes.device != dev) {
    cudaGetLastError();
    return false;
  }
  static const RangeFn range = driver_fn<RangeFn>("cuMemGetAddressRange");
  static const AttrFn attribute = driver_fn<AttrFn>("cuPointerGetAttribute");
  static const AccessFn access = driver_fn<AccessFn>("cuMemGetAccess");
  if (!range || !attribute || !access || bytes == 0) return false;
  const auto address = static_cast<CUdeviceptr>(reinterpret_cast<uintptr_t>(ptr));
  if (bytes - 1 > UINTPTR_MAX - address) return false;
  const CUdeviceptr last = address + bytes - 1;
  CUdeviceptr base = 0, last_base = 0;
  size_t extent = 0, last_extent = 0;
  if (range(&base, &extent, address) != CUDA_SUCCESS || address < base ||
      address - base >= extent || bytes > extent - (address - base) ||
      range(&last_base, &last_extent, last) != CUDA_SUCCESS || last_base != base ||
      last_extent != extent)
    return false;
  bool vmm = true, ordinary = true;
  for (CUdeviceptr endpoint : {address, last}) {
    CUmemoryPool pool = nullptr;
    if (attribute(&pool, CU_POINTER_ATTRIBUTE_MEMPOOL_HANDLE, endpoint) != CUDA_SUCCESS || pool)
      return false;
    int legacy_ipc = 0;
    if (attribute(&legacy_ipc, CU_POINTER_ATTRIBUTE_IS_LEGACY_CUDA_IPC_CAPABLE, endpoint) != CUDA_SUCCESS)
      return false;
    if (legacy_ipc != 0) vmm = false;
    if (legacy_ipc != 1) ordinary = false;
    for (int i = 0; i < n; ++i) {
      CUmemLocation location{};
      location.type = CU_MEM_LOCATION_TYPE_DEVICE;
      location.id = devices[i];
      unsigned long long flags = 0;
      const CUresult result = access(&flags, &location, endpoint);
      if (result == CUDA_SUCCESS) {
        if (flags != CU_MEM_ACCESS_FLAGS_PROT_READWRITE) vmm = false;
        if (flags != 0 && flags != CU_MEM_ACCESS_FLAGS_PROT_READWRITE) ordinary = false;
      } else if (result == CUDA_ERROR_INVALID_VALUE) {
        vmm = false;
      } else {
        return false;
      }
    }
  }
  if (vmm) return true;
  if (!ordinary) return false;
  for (int i = 0; i < n; ++i) {
    if (devices[i] == dev) continue;
    int can = 0;
    if (cudaDeviceCanAccessPeer(&can, devices[i], dev) != cudaSuccess || !can) {
      cudaGetLastError();
      return false;
    }
  }
  return true;
}

}  // namespace nb
