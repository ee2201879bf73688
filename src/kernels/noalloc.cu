// Allocation-free staged AllReduce (see noalloc.h for who needs it, the
// limits and the sharing rules). This file has no counterpart in the
// reference.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "kernels/noalloc.h"

namespace {

constexpr unsigned long long kScratchBytes = 32ull << 20;
constexpr int kMaxRanks = 8;
constexpr int kMaxDevices = 64;

// The staging scratch: a file-scope device array, never cudaMalloc'd. In host
// code this name is only a host-side stand-in; the kernel receives the
// device address that cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch on the current device (looked up once per
// device, with that device current).
cudaError_t scratch_on_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

struct FoldArgs {
  const void* local;         // this rank's slice of its own input
  const unsigned char* scratch;  // staged slices of the other ranks
  unsigned long long stride; // bytes between staged slices
  void* dst[kMaxRanks];      // slice of every rank's output
  unsigned long long count;  // elements in the slice
  int nranks, rank;
};

template <typename T> __device__ __forceinline__ float to_f(T v) { return float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v) { return T(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// The staged fold with its sources in the static scratch: rank order, fp32
// accumulation, the result stored into every rank's output slice.
template <typename T>
__global__ void __launch_bounds__(512) staged_fold_noalloc_kernel(const __grid_constant__ FoldArgs a) {
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < a.count;
       i += stride) {
    float acc = 0.0f;
    int j = 0;
    for (int q = 0; q < a.nranks; ++q) {
      const T* src = q == a.rank ? static_cast<const T*>(a.local)
                                 : reinterpret_cast<const T*>(a.scratch + (unsigned long long)(j++) * a.stride);
      const float x = to_f<T>(src[i]);
      acc = q == 0 ? x : acc + x;
    }
    const T out = from_f<T>(acc);
    for (int q = 0; q < a.nranks; ++q) static_cast<T*>(a.dst[q])[i] = out;
  }
}

void set_err(char* err, size_t cap, const char* msg) {
  if (err && cap) std::snprintf(err, cap, "%s", msg);
}

}  // namespace

extern "C" uint64_t nb_noalloc_scratch_bytes() { return kScratchBytes; }

extern "C" int nb_staged_allreduce_noalloc(const void* const* sends, void* const* recvs, int nranks,
                                           uint64_t count, int dtype, void* stream, char* err,
                                           size_t errcap) {
  set_err(err, errcap, "");
  if (!sends || !recvs || nranks < 1 || nranks > kMaxRanks) {
    set_err(err, errcap, "bad arguments: 1..8 ranks with send and receive buffers");
    return -1;
  }
  size_t es = 0;
  const void* kernel = nullptr;
  switch (dtype) {
    case NB_NOALLOC_FLOAT16: es = 2; kernel = reinterpret_cast<const void*>(staged_fold_noalloc_kernel<__half>); break;
    case NB_NOALLOC_FLOAT32: es = 4; kernel = reinterpret_cast<const void*>(staged_fold_noalloc_kernel<float>); break;
    case NB_NOALLOC_BFLOAT16:
      es = 2;
      kernel = reinterpret_cast<const void*>(staged_fold_noalloc_kernel<__nv_bfloat16>);
      break;
    default:
      set_err(err, errcap, "bad arguments: dtype must be ncclFloat16, ncclFloat32 or ncclBfloat16");
      return -1;
  }
  // A count whose byte size wraps would pass the capacity check below.
  if (count > ~0ull / es) {
    set_err(err, errcap, "bad arguments: count * element size overflows 64 bits");
    return -1;
  }
  const unsigned long long bytes = count * es;
  // Slices on 32-byte boundaries, the last takes the remainder (the largest).
  const unsigned long long base = (bytes / (unsigned long long)nranks) & ~31ull;
  const unsigned long long largest = bytes - base * (unsigned long long)(nranks - 1);
  if ((unsigned long long)(nranks - 1) * largest > kScratchBytes) {
    char msg[160];
    std::snprintf(msg, sizeof msg,
                  "message of %llu bytes over %d ranks needs %llu bytes of staging scratch; the "
                  "static scratch holds %llu",
                  bytes, nranks, (unsigned long long)(nranks - 1) * largest, kScratchBytes);
    set_err(err, errcap, msg);
    return -2;
  }
  void* scratch = nullptr;
  cudaError_t e = scratch_on_current_device(&scratch);
  if (e != cudaSuccess) {
    set_err(err, errcap, "cudaGetSymbolAddress of the static scratch failed");
    return int(e);
  }
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) {
    set_err(err, errcap, "cannot query the current device's SM count");
    return int(e);
  }
  if (sms < 1) sms = 1;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int r = 0; r < nranks; ++r) {
    const unsigned long long off = base * (unsigned long long)r;
    const unsigned long long len = r == nranks - 1 ? bytes - off : base;
    if (!len) continue;
    int j = 0;
    for (int q = 0; q < nranks; ++q) {
      if (q == r) continue;
      e = cudaMemcpyAsync(static_cast<unsigned char*>(scratch) + (unsigned long long)(j++) * largest,
                          static_cast<const unsigned char*>(sends[q]) + off, len,
                          cudaMemcpyDeviceToDevice, s);
      if (e != cudaSuccess) {
        set_err(err, errcap, "cudaMemcpyAsync into the static scratch failed");
        return int(e);
      }
    }
    FoldArgs a{};
    a.local = static_cast<const unsigned char*>(sends[r]) + off;
    a.scratch = static_cast<const unsigned char*>(scratch);
    a.stride = largest;
    for (int q = 0; q < nranks; ++q) a.dst[q] = static_cast<unsigned char*>(recvs[q]) + off;
    a.count = len / es;
    a.nranks = nranks;
    a.rank = r;
    const unsigned long long want = (a.count + 511) / 512;
    const unsigned blocks = unsigned(want < (unsigned long long)(sms * 4) ? (want ? want : 1) : sms * 4);
    void* argv[] = {&a};
    e = cudaLaunchKernel(kernel, dim3(blocks), dim3(512), argv, 0, s);
    if (e != cudaSuccess) {
      set_err(err, errcap, "launch of the staged fold failed");
      return int(e);
    }
  }
  return 0;
}
