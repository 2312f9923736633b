// spec.cuh — the chunk summary behind the serial-order f64 folds (the plan oracle's s = ((0 + x0) + x1) + ... with
// one rounding to f32) that add runs of values out of order where no add of the fold can round.
//
// Every f32 is an integer multiple of its ulp, 2^(max(e,1) - 150) for exponent field e. If all the values added
// since the last inexact step are multiples of 2^q, so is every partial sum, and a partial sum below 2^(q+53) in
// magnitude has at most 53 significant bits: representable, so the add that made it did not round. While no add
// rounds, the serial fold is the exact sum, and any order of adding a run of values gives the same bits.
//
// A chunk of 64 consecutive values of a fold is summarised in three numbers: L = 2^(q + 53) for q the smallest ulp
// exponent of its nonzero values; T, its prefix sum in f64 in fold order; and H, the largest magnitude of those
// prefix sums, rounded up to f32. If H < L, no add of the prefix rounded (the first that did would have made a
// partial sum of magnitude at least L, since L is a power of two and rounding is monotone), so T and H are exact.
// Otherwise, or if T is a NaN or infinite, H is +inf. From a running sum s whose values so far are multiples of
// 2^q', the fold's partial sums inside the chunk are s + (a prefix), at most |s| + H in magnitude; below
// min(2^(q'+53), L) none of them rounds and s + T is exact. After a chunk is folded value by value, s is a multiple
// of 2^lowbit(s), and the limit restarts at 2^(lowbit(s) + 53) (spec_anchor).
#pragma once

#include <cstdint>

namespace up {

constexpr int kSpecChunk = 64;

__device__ __forceinline__ double pow2_biased(uint32_t e) { return __longlong_as_double((long long)e << 52); }
__device__ __forceinline__ double f64_inf() { return __longlong_as_double(0x7ff0000000000000ll); }

// 2^(lowbit(s) + 53) for a finite nonzero s, +inf otherwise.
__device__ __forceinline__ double spec_anchor(double s) {
  const uint64_t u = (uint64_t)__double_as_longlong(s);
  const uint32_t ex = (uint32_t)(u >> 52) & 0x7ffu;
  const uint64_t m = u & ((1ull << 52) - 1);
  if ((u << 1) == 0 || ex == 0x7ffu) return f64_inf();
  const uint64_t sig = ex ? (m | (1ull << 52)) : m;
  const uint32_t le = (ex ? ex : 1u) + (uint32_t)(__ffsll((long long)sig) - 1) + 1u;
  return pow2_biased(le < 2046u ? le : 2046u);
}

// One value into a chunk summary. mn keeps the minimum of (bits << 1) - 2: the sign drops out, and both zeros wrap
// to the top so they never count.
__device__ __forceinline__ void spec_acc(float v, double& pre, double& hi, uint32_t& mn) {
  pre += (double)v;
  hi = fmax(hi, fabs(pre));
  mn = min(mn, (__float_as_uint(v) << 1) - 2u);
}

// L and H of a chunk from its accumulators (T is the prefix itself).
__device__ __forceinline__ void spec_finish(double pre, double hi, uint32_t mn, double& lc, float& h) {
  lc = mn >= 0xfffffffeu ? f64_inf() : pow2_biased(max((mn + 2u) >> 24, 1u) + 926u);
  h = (hi < lc && pre - pre == 0.0) ? __double2float_ru(hi) : __int_as_float(0x7f800000);
}

}  // namespace up
