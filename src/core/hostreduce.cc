#include "core/hostreduce.h"

#include <cmath>
#include <cstring>
#include <thread>
#include <type_traits>
#include <vector>

namespace nb {

float half_to_float(uint16_t h) {
  const uint32_t sign = uint32_t(h & 0x8000) << 16;
  const uint32_t exp = (h >> 10) & 0x1f;
  uint32_t mant = h & 0x3ff;
  uint32_t bits;
  if (exp == 0x1f) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else {  // subnormal: normalize
      int e = -1;
      do {
        ++e;
        mant <<= 1;
      } while (!(mant & 0x400));
      bits = sign | uint32_t(127 - 15 - e) << 23 | (mant & 0x3ff) << 13;
    }
  } else {
    bits = sign | (exp + 127 - 15) << 23 | mant << 13;
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t float_to_half(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint16_t sign = uint16_t((x >> 16) & 0x8000);
  const uint32_t exp = (x >> 23) & 0xff;
  uint32_t mant = x & 0x7fffff;
  if (exp == 0xff) return uint16_t(sign | 0x7c00 | (mant ? (0x200 | (mant >> 13)) : 0));
  const int e = int(exp) - 127 + 15;
  if (e >= 31) return uint16_t(sign | 0x7c00);
  if (e <= 0) {
    if (e < -10) return sign;
    mant |= 0x800000;
    const int shift = 14 - e;
    uint32_t m = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (m & 1))) ++m;
    return uint16_t(sign | m);
  }
  uint32_t h = uint32_t(e) << 10 | (mant >> 13);
  const uint32_t rem = mant & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) ++h;  // carry may reach inf: correct
  return uint16_t(sign | h);
}

float bf16_to_float(uint16_t b) {
  const uint32_t bits = uint32_t(b) << 16;
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t float_to_bf16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7f800000u) == 0x7f800000u && (x & 0x7fffff)) return uint16_t((x >> 16) | 0x40);
  x += 0x7fffu + ((x >> 16) & 1);
  return uint16_t(x >> 16);
}

namespace {

// IEEE maxNum/minNum with a fixed order for signed zeros and NaNs, written
// the same way as the device code so both sides agree bit for bit.
template <typename A>
inline A fold_max(A a, A b) {
  if (a != a) return b;
  if (b != b) return a;
  if (a == b) return std::signbit(a) ? b : a;
  return a > b ? a : b;
}
template <typename A>
inline A fold_min(A a, A b) {
  if (a != a) return b;
  if (b != b) return a;
  if (a == b) return std::signbit(a) ? a : b;
  return a < b ? a : b;
}

template <typename S>
struct Storage {  // plain numeric storage
  using Acc = S;
  static Acc load(const void* p, size_t i) { return static_cast<const S*>(p)[i]; }
  static void store(void* p, size_t i, Acc v) { static_cast<S*>(p)[i] = v; }
};
struct HalfStorage {
  using Acc = float;
  static Acc load(const void* p, size_t i) { return half_to_float(static_cast<const uint16_t*>(p)[i]); }
  static void store(void* p, size_t i, Acc v) { static_cast<uint16_t*>(p)[i] = float_to_half(v); }
};
struct Bf16Storage {
  using Acc = float;
  static Acc load(const void* p, size_t i) { return bf16_to_float(static_cast<const uint16_t*>(p)[i]); }
  static void store(void* p, size_t i, Acc v) { static_cast<uint16_t*>(p)[i] = float_to_bf16(v); }
};

template <typename St>
void fold_float(const FoldParams& p, const void* const* srcs, int nsrc, void* dst, size_t lo,
                size_t hi) {
  using A = typename St::Acc;
  A s[kMaxRanks];
  for (int i = 0; i < nsrc; ++i) s[i] = A(p.scalars[i]);
  const A n = A(p.nranks);
  for (size_t e = lo; e < hi; ++e) {
    A acc = St::load(srcs[0], e);
    if (p.op == RedOp::PreMulSum) acc = acc * s[0];
    for (int i = 1; i < nsrc; ++i) {
      const A x = St::load(srcs[i], e);
      switch (p.op) {
        case RedOp::Prod: acc = acc * x; break;
        case RedOp::Max: acc = fold_max(acc, x); break;
        case RedOp::Min: acc = fold_min(acc, x); break;
        case RedOp::PreMulSum: acc = std::fma(x, s[i], acc); break;
        default: acc = acc + x; break;
      }
    }
    if (p.op == RedOp::Avg) acc = acc / n;
    St::store(dst, e, acc);
  }
}

template <typename T>
void fold_int(const FoldParams& p, const void* const* srcs, int nsrc, void* dst, size_t lo,
              size_t hi) {
  using U = std::make_unsigned_t<T>;
  for (size_t e = lo; e < hi; ++e) {
    T acc = static_cast<const T*>(srcs[0])[e];
    for (int i = 1; i < nsrc; ++i) {
      const T x = static_cast<const T*>(srcs[i])[e];
      switch (p.op) {
        case RedOp::Prod: acc = T(U(acc) * U(x)); break;
        case RedOp::Max: acc = acc > x ? acc : x; break;
        case RedOp::Min: acc = acc < x ? acc : x; break;
        default: acc = T(U(acc) + U(x)); break;
      }
    }
    if (p.op == RedOp::Avg) acc = T(acc / T(p.nranks));
    static_cast<T*>(dst)[e] = acc;
  }
}

void fold_range(const FoldParams& p, const void* const* srcs, int nsrc, void* dst, size_t lo,
                size_t hi) {
  switch (p.dtype) {
    case DType::F32: return fold_float<Storage<float>>(p, srcs, nsrc, dst, lo, hi);
    case DType::F64: return fold_float<Storage<double>>(p, srcs, nsrc, dst, lo, hi);
    case DType::F16: return fold_float<HalfStorage>(p, srcs, nsrc, dst, lo, hi);
    case DType::BF16: return fold_float<Bf16Storage>(p, srcs, nsrc, dst, lo, hi);
    case DType::I8: return fold_int<int8_t>(p, srcs, nsrc, dst, lo, hi);
    case DType::U8: return fold_int<uint8_t>(p, srcs, nsrc, dst, lo, hi);
    case DType::I32: return fold_int<int32_t>(p, srcs, nsrc, dst, lo, hi);
    case DType::U32: return fold_int<uint32_t>(p, srcs, nsrc, dst, lo, hi);
    case DType::I64: return fold_int<int64_t>(p, srcs, nsrc, dst, lo, hi);
    case DType::U64: return fold_int<uint64_t>(p, srcs, nsrc, dst, lo, hi);
    default: return;
  }
}

}  // namespace

void host_fold(const FoldParams& p, const void* const* srcs, int nsrc, void* dst, size_t bytes) {
  const size_t es = elem_size(p.dtype);
  if (!es || nsrc < 1) return;
  fold_range(p, srcs, nsrc, dst, 0, bytes / es);
}

void host_fold_parallel(const FoldParams& p, const void* const* srcs, int nsrc, void* dst,
                        size_t bytes, int threads) {
  const size_t es = elem_size(p.dtype);
  if (!es || nsrc < 1) return;
  const size_t n = bytes / es;
  if (threads <= 1 || n < (size_t(1) << 16)) return fold_range(p, srcs, nsrc, dst, 0, n);
  std::vector<std::thread> pool;
  pool.reserve(size_t(threads));
  // Chunk boundaries on 64-byte lines so no two threads share a cache line.
  const size_t per_line = 64 / es;
  const size_t chunk = ((n / size_t(threads) + per_line - 1) / per_line) * per_line;
  for (int t = 0; t < threads; ++t) {
    const size_t lo = size_t(t) * chunk;
    if (lo >= n) break;
    const size_t hi = std::min(n, lo + chunk);
    pool.emplace_back([&p, srcs, nsrc, dst, lo, hi] { fold_range(p, srcs, nsrc, dst, lo, hi); });
  }
  for (auto& t : pool) t.join();
}

}  // namespace nb
