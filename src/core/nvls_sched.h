// Round schedule of the NVLS AllReduce kernel, shared by the kernel, the
// host (progress steps of a call) and the CPU tests.
//
// Uniform rounds of R bytes; with `ramp` (and a message of at least 4R) the
// first four rounds are R/8, R/8, R/4, R/2 and the last four R/2, R/4, R/8,
// R/8 (q = R/8 rounded down to 32 bytes), so the switch starts after a short
// first copy-in and the kernel ends after a short last copy-out; the rounds
// between are R, the last of them partial. The rounds partition [0, bytes)
// in order; every round is at most R bytes.
#pragma once

#ifdef __CUDACC__
#define NB_HD __host__ __device__
#else
#define NB_HD
#endif

namespace nb {

NB_HD inline bool ar_ramped(unsigned long long bytes, unsigned long long R, int ramp) {
  return ramp && (R / 8 & ~31ull) > 0 && bytes >= 4 * R;
}

NB_HD inline unsigned ar_rounds(unsigned long long bytes, unsigned long long R, int ramp) {
  if (!ar_ramped(bytes, R, ramp)) return unsigned((bytes + R - 1) / R);
  const unsigned long long q = R / 8 & ~31ull;
  return 8u + unsigned((bytes - 16 * q + R - 1) / R);
}

NB_HD inline void ar_round(unsigned s, unsigned long long bytes, unsigned long long R, int ramp,
                           unsigned long long* base, unsigned long long* len) {
  if (!ar_ramped(bytes, R, ramp)) {
    *base = (unsigned long long)s * R;
    *len = bytes - *base < R ? bytes - *base : R;
    return;
  }
  const unsigned long long q = R / 8 & ~31ull;
  const unsigned long long mid = bytes - 16 * q;  // bytes of the uniform rounds
  const unsigned nmid = unsigned((mid + R - 1) / R);
  if (s < 4) {  // head: units of q at 0, 1, 2, 4; lengths 1, 1, 2, 4
    const unsigned long long off = s < 3 ? s : 4, n = s < 2 ? 1 : (s == 2 ? 2 : 4);
    *base = off * q;
    *len = n * q;
  } else if (s < 4 + nmid) {
    const unsigned long long at = (unsigned long long)(s - 4) * R;
    *base = 8 * q + at;
    *len = mid - at < R ? mid - at : R;
  } else {  // tail: units at 0, 4, 6, 7; lengths 4, 2, 1, 1
    const unsigned t = s - 4 - nmid;
    const unsigned long long off = t == 0 ? 0 : (t == 1 ? 4 : (t == 2 ? 6 : 7)), n = t == 0 ? 4 : (t == 1 ? 2 : 1);
    *base = 8 * q + mid + off * q;
    *len = n * q;
  }
}

}  // namespace nb
