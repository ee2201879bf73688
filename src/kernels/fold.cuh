// Element folds shared by the sm_100a reduction kernels: fp32 accumulation
// for fp16/bf16/fp32 (fp64 for doubles, the type's own width with
// wrap-around for integers), sources folded in index (= rank) order, the
// op's finalization (average, pre-multiplied scalars) and the cast back.
// The arithmetic is exactly the host fold's (src/core/hostreduce.cc), so
// the host oracle is bit-exact.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "core/types.h"

namespace nb {
namespace kfold {

template <typename T>
struct Acc {
  using type = T;
};
template <> struct Acc<__half> { using type = float; };
template <> struct Acc<__nv_bfloat16> { using type = float; };
template <> struct Acc<float> { using type = float; };
template <> struct Acc<double> { using type = double; };

template <typename T> __device__ __forceinline__ typename Acc<T>::type to_acc(T v) { return v; }
template <> __device__ __forceinline__ float to_acc<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_acc<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_acc(typename Acc<T>::type v) { return T(v); }
template <> __device__ __forceinline__ __half from_acc<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T> struct IsFloat { static constexpr bool value = false; };
template <> struct IsFloat<__half> { static constexpr bool value = true; };
template <> struct IsFloat<__nv_bfloat16> { static constexpr bool value = true; };
template <> struct IsFloat<float> { static constexpr bool value = true; };
template <> struct IsFloat<double> { static constexpr bool value = true; };

template <typename T> struct Unsigned { using type = T; };
template <> struct Unsigned<int8_t> { using type = uint8_t; };
template <> struct Unsigned<int32_t> { using type = uint32_t; };
template <> struct Unsigned<int64_t> { using type = unsigned long long; };
template <> struct Unsigned<uint64_t> { using type = unsigned long long; };

// Same ordering rules as the host fold (hostreduce.cc fold_max/fold_min).
template <typename A>
__device__ __forceinline__ A fmax_ord(A a, A b) {
  if (a != a) return b;
  if (b != b) return a;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
template <typename A>
__device__ __forceinline__ A fmin_ord(A a, A b) {
  if (a != a) return b;
  if (b != b) return a;
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}

__device__ __forceinline__ float fma_rn(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fma_rn(double a, double b, double c) { return __fma_rn(a, b, c); }

template <typename T>
__device__ __forceinline__ typename Acc<T>::type combine(typename Acc<T>::type acc, T xv, int op,
                                                         typename Acc<T>::type s) {
  using A = typename Acc<T>::type;
  const A x = to_acc<T>(xv);
  if constexpr (IsFloat<T>::value) {
    switch (op) {
      case int(RedOp::Prod): return acc * x;
      case int(RedOp::Max): return fmax_ord(acc, x);
      case int(RedOp::Min): return fmin_ord(acc, x);
      case int(RedOp::PreMulSum): return fma_rn(x, s, acc);
      default: return acc + x;
    }
  } else {
    using U = typename Unsigned<T>::type;
    switch (op) {
      case int(RedOp::Prod): return T(U(acc) * U(x));
      case int(RedOp::Max): return acc > x ? acc : x;
      case int(RedOp::Min): return acc < x ? acc : x;
      default: return T(U(acc) + U(x));
    }
  }
}

template <typename T>
__device__ __forceinline__ T finish(typename Acc<T>::type acc, int op, int nranks) {
  using A = typename Acc<T>::type;
  if (op == int(RedOp::Avg)) {
    if constexpr (IsFloat<T>::value) acc = acc / A(nranks);
    else acc = T(T(acc) / T(nranks));
  }
  return from_acc<T>(acc);
}

template <typename T>
__device__ __forceinline__ typename Acc<T>::type first(T xv, int op, typename Acc<T>::type s) {
  using A = typename Acc<T>::type;
  A x = to_acc<T>(xv);
  if constexpr (IsFloat<T>::value) {
    if (op == int(RedOp::PreMulSum)) x = x * s;
  }
  return x;
}

// One 16-byte vector of every source -> folded vector.
template <typename T, int NSRC>
__device__ __forceinline__ uint4 fold_vec(const uint4 (&v)[NSRC], int op, int nranks,
                                          const typename Acc<T>::type (&s)[NSRC]) {
  using A = typename Acc<T>::type;
  constexpr int E = 16 / sizeof(T);
  uint4 out;
  const T* in0 = reinterpret_cast<const T*>(&v[0]);
  T* o = reinterpret_cast<T*>(&out);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    A acc = first<T>(in0[e], op, s[0]);
#pragma unroll
    for (int k = 1; k < NSRC; ++k) acc = combine<T>(acc, reinterpret_cast<const T*>(&v[k])[e], op, s[k]);
    o[e] = finish<T>(acc, op, nranks);
  }
  return out;
}

}  // namespace kfold
}  // namespace nb
