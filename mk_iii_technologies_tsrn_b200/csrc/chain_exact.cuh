// chain_exact.cuh -- n successive fp32 additions of one addend, evaluated
// exactly (round to nearest, ties to even at every step) in a number of
// operations that grows with the binades the sum passes through, not with n.
//
// This is the carry of the tropical SSM recurrence through a stretch of time
// in which no input wins (h_t = fl(a + h_{t-1}), research/tsrn_dml.py:906-916):
// the chunk-parallel scan needs it for every chunk whose carry survives.
//
// Inside one binade [2^(e-1), 2^e) (one sign, spacing ulp = 2^(e-24)) a float
// is M * ulp with an integer significand M in [2^23, 2^24).  While the exact
// sum of a step stays in the binade, fl(M ulp + a) = (M + m) ulp with m the
// nearest integer to q = a / ulp -- or, when q lies exactly halfway, the even
// one of the two neighbours of M + q.  From an even M that even neighbour is
// M + m with m the even one of floor(q) and floor(q) + 1, so the increment is
// constant and s steps add s m.  A jump runs to the last step whose exact sum
// is still inside the binade; single additions cross binade edges, zeros,
// subnormals and the overflow end, and start a halfway run from an odd M.
// Significands and step counts are carried in double precision, where every
// quantity used is an exact integer or an exact fp32 value times a power of
// two.
//
// Header-only and usable from host code (the host test builds it with a C++
// compiler and compares it with step-by-step float32 additions).
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define TP_CHAIN_FN __host__ __device__ __forceinline__
#else
#define TP_CHAIN_FN static inline
#endif

namespace tp {

TP_CHAIN_FN uint32_t chain_f32_bits(float x) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(x);
#else
  uint32_t u;
  memcpy(&u, &x, sizeof(u));
  return u;
#endif
}

// 2^k as a double, -1022 <= k <= 1023
TP_CHAIN_FN double chain_pow2(int k) {
  const uint64_t bits = (uint64_t)(k + 1023) << 52;
#if defined(__CUDA_ARCH__)
  return __longlong_as_double((long long)bits);
#else
  double d;
  memcpy(&d, &bits, sizeof(d));
  return d;
#endif
}

// fl(...fl(fl(x + a) + a)... + a) with n additions (x for n <= 0)
TP_CHAIN_FN float chain_exact(float x, float a, int64_t n) {
  const double kLo = 8388608.0, kHi = 16777216.0;   // 2^23, 2^24: significands of a binade
  if (n <= 0) return x;
  // NaN, infinities and a zero addend settle after one addition
  if (x != x || a != a || a == 0.0f || isinf(x) || isinf(a)) return x + a;
  while (n > 0) {
    const int be = (int)((chain_f32_bits(x) >> 23) & 0xffu);    // biased exponent of x
    if (be < 2 || be > 252) {          // zero, subnormal or near overflow: one addition
      x = x + a;
      --n;
      if (isinf(x)) return x + a;      // an overflow (or NaN) settles
      continue;
    }
    const double inv_ulp = chain_pow2(150 - be);                // 1 / ulp of x's binade
    const double mag = fabs((double)x) * inv_ulp;                // M in [2^23, 2^24)
    const double sgn = x < 0.0f ? -1.0 : 1.0;
    const double q = sgn * (double)a * inv_ulp;                  // a / ulp, along x's sign
    const double s1 = mag + q;                                   // first exact sum, in ulps
    if (!(fabs(q) < kLo) || !(s1 >= kLo && s1 < kHi)) {         // the first step leaves the binade
      x = x + a;
      --n;
      continue;
    }
    const double fq = floor(q);
    double m;
    if (q - fq == 0.5) {               // halfway: ties to even
      if (fmod(mag, 2.0) != 0.0) {     // odd M: one addition makes it even
        x = x + a;
        --n;
        continue;
      }
      m = fmod(fq, 2.0) == 0.0 ? fq : fq + 1.0;
    } else {
      m = rint(q);
    }
    if (m == 0.0) return x;            // every addition rounds back to x
    // s additions whose exact sums s1 + (i - 1) m, i = 1..s, stay in [2^23, 2^24)
    double smax = m > 0.0 ? ceil((kHi - s1) / m) : floor((s1 - kLo) / -m) + 1.0;
    double s = (double)n < smax ? (double)n : smax;
    if (s < 1.0) s = 1.0;
    while (s > 1.0) {                  // the quotient's rounding can overshoot by one
      const double last = s1 + (s - 1.0) * m;
      if (last >= kLo && last < kHi) break;
      s -= 1.0;
    }
    x = (float)(sgn * (mag + s * m) * chain_pow2(be - 150));
    n -= (int64_t)s;
  }
  return x;
}

}  // namespace tp
