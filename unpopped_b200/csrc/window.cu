// window.cu — the Window lift (Access::Window, crates/unpopped/src/ir.rs:2206-2259) as 1-D pooling along one axis
// of a dense [outer, k_in, inner] input into [outer, k_out, inner], and the Im2Col lift (Access::Im2Col,
// ir.rs:2286-2324), the 2-D unfold of an NCHW input into [N, C·kh·kw, oH·oW].
//
// Window, as the oracle evaluates it (oracle/plan_window.rs:249-475): output o folds the taps
// p = o·stride − pad_lo + kk·dilation, kk = 0 .. size−1 ascending, skipping taps outside [0, k_in):
//  * f32 Sum/Mean fold in f64 and round once; Mean divides by `size` (count_include_pad) or by the valid taps;
//  * f32 Max/Min take the first tap, then a strictly better one, and keep the last NaN (its bits with the quiet bit
//    set, as the f32 -> f64 -> f32 conversions of the oracle leave them);
//  * i32 Sum wraps at 32 bits; i32 Max/Min are exact. i32 Mean is not defined (the oracle asserts against it).
// A window with no in-bounds tap is refused before launch (window_taps::check_window_taps; the reference's plan
// declines it, window_without_real_tap_declines.rs).
//
// Im2Col (plan_window.rs:483-535): output cell (n, c·kh·kw + ki·kw + kj, oh·oW + ow) copies the raw bits of
// input (n, c, oh·sh − ph + ki·dh, ow·sw − pw + kj·dw), or writes zero bytes where that falls outside the input.
#include "common.cuh"

#include <mutex>

namespace up {
namespace win {

constexpr int kThreads = 256;

// The window Mean's acc / d, correctly rounded in f64. For the full count d = SZ of a compile-time size it is
// Markstein's correction of acc * RN(1/d): the remainder acc - q d is exact by FMA, and RN(q + r * RN(1/d)) is the
// correctly rounded quotient for finite acc (P. Markstein, IBM J. Res. Develop. 34(1), 1990). Checked against IEEE
// division on 3e8 quotients (d = 2 .. 16; 2- and 3-term f64 sums of f32 values, random f64 values, integers), with
// no difference. Other counts and a non-finite acc take the division.
template <int SZ>
__device__ __forceinline__ double mean_div(double acc, int d) {
  if (SZ > 0 && d == SZ && acc - acc == 0.0) {  // finite: Inf - Inf and NaN compare unequal to 0
    constexpr double inv = 1.0 / (double)(SZ > 0 ? SZ : 1);
    const double q = acc * inv;
    return fma(fma(-q, (double)SZ, acc), inv, q);
  }
  return acc / (double)d;
}

// One output of a window: the fold of its in-bounds taps (src points at tap position 0 of the output's line;
// consecutive taps are `step` elements apart).
// SZ > 0 fixes the window size at compile time, so the tap loops unroll.
template <int OP, bool INCLUDE_PAD, int SZ>
__device__ __forceinline__ float window_f32_one(const float* __restrict__ src, int64_t step, int64_t p0, int64_t k_in,
                                                int size_rt, int dilation) {
  const int size = SZ > 0 ? SZ : size_rt;
  if (OP == UP_OP_SUM || OP == UP_OP_MEAN) {
    double acc = 0.0;
    int cnt = 0;
#pragma unroll
    for (int kk = 0; kk < size; ++kk) {
      const int64_t p = p0 + (int64_t)kk * dilation;
      if (p < 0 || p >= k_in) continue;
      acc += (double)src[p * step];
      ++cnt;
    }
    if (OP == UP_OP_MEAN) acc = mean_div<SZ>(acc, INCLUDE_PAD ? size : cnt);
    return __double2float_rn(acc);
  } else {
    if (p0 >= 0 && p0 + (int64_t)(size - 1) * dilation < k_in) {
      // an interior window: the first tap seeds a branch-free fold (as window_f32_row below)
      const int64_t tstep = (int64_t)dilation * step;
      const float* q = src + p0 * step;
      float b = *q;
      uint32_t nb = __float_as_uint(b);
      bool nan = b != b;
#pragma unroll
      for (int kk = 1; kk < size; ++kk) {
        q += tstep;
        const float v = *q;
        const bool vn = v != v;
        nb = vn ? __float_as_uint(v) : nb;
        nan = nan || vn;
        b = (OP == UP_OP_MAX ? v > b : v < b) ? v : b;
      }
      return __uint_as_float(nan ? (nb | 0x00400000u) : __float_as_uint(b));
    }
    uint32_t best = 0, nan_bits = 0;
    bool have = false, nan = false;
#pragma unroll
    for (int kk = 0; kk < size; ++kk) {
      const int64_t p = p0 + (int64_t)kk * dilation;
      if (p < 0 || p >= k_in) continue;
      const float v = src[p * step];
      if (v != v) {
        nan = true;
        nan_bits = __float_as_uint(v);
      } else if (!have || (OP == UP_OP_MAX ? v > __uint_as_float(best) : v < __uint_as_float(best))) {
        best = __float_as_uint(v);
      }
      have = have || v == v;
    }
    return __uint_as_float(nan ? (nan_bits | 0x00400000u) : best);
  }
}

template <int OP>
__device__ __forceinline__ int32_t window_i32_one(const int32_t* __restrict__ src, int64_t step, int64_t p0,
                                                  int64_t k_in, int size, int dilation) {
  uint32_t acc = 0;
  bool have = false;
  for (int kk = 0; kk < size; ++kk) {
    const int64_t p = p0 + (int64_t)kk * dilation;
    if (p < 0 || p >= k_in) continue;
    const int32_t v = src[p * step];
    if (OP == UP_OP_SUM) acc += (uint32_t)v;  // wraps at 32 bits
    else if (!have || (OP == UP_OP_MAX ? v > (int32_t)acc : v < (int32_t)acc)) acc = (uint32_t)v;
    have = true;
  }
  return (int32_t)acc;
}

// A "line" is one (b, o) pair: `inner` contiguous outputs whose taps are `inner` apart. With inner == 1 a CTA
// takes a row (b) and its threads the outputs o; with inner > 1 a CTA takes lines and its threads the inner index.
// No per-element division.
template <typename T, typename F>
__device__ __forceinline__ void window_walk(const T* __restrict__ x, int64_t outer, int64_t k_in, int64_t inner,
                                            int64_t k_out, int stride, int pad_lo, T* __restrict__ out, F one) {
  if (inner == 1) {
    for (int64_t b = blockIdx.x; b < outer; b += gridDim.x) {
      const T* row = x + b * k_in;
      T* orow = out + b * k_out;
      for (int64_t o = threadIdx.x; o < k_out; o += kThreads) orow[o] = one(row, 1, o * stride - pad_lo);
    }
  } else {
    // lines narrower than the CTA share it: lp lines per step, thread t on line t / inner, index t % inner
    const int64_t lines = outer * k_out;
    const int lp = inner < kThreads ? kThreads / (int)inner : 1;
    const int sub = inner < kThreads ? (int)threadIdx.x / (int)inner : 0;
    const int64_t i0 = inner < kThreads ? (int64_t)threadIdx.x - (int64_t)sub * inner : threadIdx.x;
    if (sub >= lp) return;  // the threads past lp whole lines
    // (b, o) of the line advance by a fixed step: one division per thread, not one per line
    const int64_t step = (int64_t)gridDim.x * lp;
    const int64_t db = step / k_out, dr = step - db * k_out;
    int64_t line = (int64_t)blockIdx.x * lp + sub;
    int64_t b = line / k_out, o = line - b * k_out;
    for (; line < lines; line += step) {
      const T* base = x + b * k_in * inner;
      T* orow = out + line * inner;
      for (int64_t i = i0; i < inner; i += kThreads) orow[i] = one(base + i, inner, o * stride - pad_lo);
      o += dr;
      b += db;
      if (o >= k_out) {
        o -= k_out;
        ++b;
      }
    }
  }
}

// The same fold over a row staged in shared memory, with 32-bit positions; an interior window (every tap inside the
// row) skips the bounds checks.
// SZ > 0 fixes the window size at compile time (the common pooling sizes), so the tap loops unroll.
template <int OP, bool INCLUDE_PAD, int SZ>
__device__ __forceinline__ float window_f32_row(const float* __restrict__ row, int p0, int k_in, int size_rt,
                                                int dilation) {
  const int size = SZ > 0 ? SZ : size_rt;
  const bool interior = p0 >= 0 && p0 + (size - 1) * dilation < k_in;
  if (OP == UP_OP_SUM || OP == UP_OP_MEAN) {
    double acc = 0.0;
    int cnt = 0;
    if (interior) {
#pragma unroll
      for (int kk = 0, p = p0; kk < size; ++kk, p += dilation) acc += (double)row[p];
      cnt = size;
    } else {
#pragma unroll
      for (int kk = 0, p = p0; kk < size; ++kk, p += dilation)
        if (p >= 0 && p < k_in) {
          acc += (double)row[p];
          ++cnt;
        }
    }
    if (OP == UP_OP_MEAN) acc = mean_div<SZ>(acc, INCLUDE_PAD ? size : cnt);
    return __double2float_rn(acc);
  } else {
    if (interior) {
      // Every tap is in bounds, so the first one seeds the fold. A NaN anywhere decides the result, so a NaN seed
      // needs no later non-NaN value, and a NaN tap never wins the comparison.
      float b = row[p0];
      uint32_t nb = __float_as_uint(b);  // the last NaN's bits, read only when there is one
      bool nan = b != b;
#pragma unroll
      for (int kk = 1, p = p0 + dilation; kk < size; ++kk, p += dilation) {
        const float v = row[p];
        const bool vn = v != v;
        nb = vn ? __float_as_uint(v) : nb;
        nan = nan || vn;
        b = (OP == UP_OP_MAX ? v > b : v < b) ? v : b;
      }
      return __uint_as_float(nan ? (nb | 0x00400000u) : __float_as_uint(b));
    }
    uint32_t best = 0, nan_bits = 0;
    bool have = false, nan = false;
#pragma unroll
    for (int kk = 0, p = p0; kk < size; ++kk, p += dilation) {
      if (p < 0 || p >= k_in) continue;
      const float v = row[p];
      if (v != v) {
        nan = true;
        nan_bits = __float_as_uint(v);
      } else if (!have || (OP == UP_OP_MAX ? v > __uint_as_float(best) : v < __uint_as_float(best))) {
        best = __float_as_uint(v);
      }
      have = have || v == v;
    }
    return __uint_as_float(nan ? (nan_bits | 0x00400000u) : best);
  }
}

// Windows along the innermost axis with rows that fit in shared memory: the row is staged once with cp.async
// (16-byte copies when the rows are 16-byte aligned, else 4-byte ones; no copy waits on a register, so every copy
// of the row is in flight together) and the taps are read from shared memory. One 32 KiB buffer (rows up to 8,192
// f32) keeps six CTAs on an SM, whose folds cover each other's staging: faster than 48 KiB (four CTAs) and than two
// buffers per CTA. Longer rows take the line path.
constexpr int64_t kRowStageBytes = 32 * 1024;
__device__ __forceinline__ void stage_copy16(void* smem, const void* gmem) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void stage_copy4(void* smem, const void* gmem) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sa), "l"(gmem) : "memory");
}
template <typename T, typename F>
__device__ __forceinline__ void window_rows_staged(const T* __restrict__ x, int64_t outer, int64_t k_in, int64_t k_out,
                                                   int stride, int pad_lo, T* __restrict__ out, F one) {
  static_assert(sizeof(T) == 4, "4-byte elements");
  __shared__ __align__(16) T srow[kRowStageBytes / sizeof(T)];
  const bool vec = ((uintptr_t)x & 15) == 0 && (k_in & 3) == 0;
  for (int64_t b = blockIdx.x; b < outer; b += gridDim.x) {
    const T* row = x + b * k_in;
    if (vec) {
      for (int i = threadIdx.x; i < (int)(k_in >> 2); i += kThreads) stage_copy16(srow + 4 * i, row + 4 * i);
    } else {
      for (int i = threadIdx.x; i < (int)k_in; i += kThreads) stage_copy4(srow + i, row + i);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    T* orow = out + b * k_out;
    // a 32-bit output index: a staged row's outputs are far below 2^31
    const int ko = (int)k_out;
    for (int o = threadIdx.x; o < ko; o += kThreads) orow[o] = one(srow, 1, (int64_t)o * stride - pad_lo);
    __syncthreads();  // the row is read before the next one is staged
  }
}

template <int OP, bool INCLUDE_PAD, int SZ>
__global__ void __launch_bounds__(kThreads) window_f32_staged_kernel(const float* __restrict__ x, int64_t outer,
                                                                      int64_t k_in, int64_t k_out, int size, int stride,
                                                                      int dilation, int pad_lo, float* __restrict__ out) {
  window_rows_staged<float>(x, outer, k_in, k_out, stride, pad_lo, out, [&](const float* src, int64_t, int64_t p0) {
    return window_f32_row<OP, INCLUDE_PAD, SZ>(src, (int)p0, (int)k_in, size, dilation);
  });
}

template <int OP, bool INCLUDE_PAD>
void launch_staged(const float* x, int64_t outer, int64_t k_in, int64_t k_out, int size, int stride, int dilation,
                   int pad_lo, float* out, int g, cudaStream_t s) {
  if (size == 2)
    window_f32_staged_kernel<OP, INCLUDE_PAD, 2><<<g, kThreads, 0, s>>>(x, outer, k_in, k_out, size, stride, dilation,
                                                                       pad_lo, out);
  else if (size == 3)
    window_f32_staged_kernel<OP, INCLUDE_PAD, 3><<<g, kThreads, 0, s>>>(x, outer, k_in, k_out, size, stride, dilation,
                                                                       pad_lo, out);
  else
    window_f32_staged_kernel<OP, INCLUDE_PAD, 0><<<g, kThreads, 0, s>>>(x, outer, k_in, k_out, size, stride, dilation,
                                                                       pad_lo, out);
}

template <int OP, bool INCLUDE_PAD, int SZ>
__global__ void __launch_bounds__(kThreads) window_f32_kernel(const float* __restrict__ x, int64_t outer, int64_t k_in,
                                                               int64_t inner, int64_t k_out, int size, int stride,
                                                               int dilation, int pad_lo, float* __restrict__ out) {
  window_walk<float>(x, outer, k_in, inner, k_out, stride, pad_lo, out, [&](const float* src, int64_t step, int64_t p0) {
    return window_f32_one<OP, INCLUDE_PAD, SZ>(src, step, p0, k_in, size, dilation);
  });
}

template <int OP, bool INCLUDE_PAD>
void launch_lines(const float* x, int64_t outer, int64_t k_in, int64_t inner, int64_t k_out, int size, int stride,
                  int dilation, int pad_lo, float* out, int g, cudaStream_t s) {
  if (size == 2)
    window_f32_kernel<OP, INCLUDE_PAD, 2><<<g, kThreads, 0, s>>>(x, outer, k_in, inner, k_out, size, stride, dilation,
                                                                pad_lo, out);
  else if (size == 3)
    window_f32_kernel<OP, INCLUDE_PAD, 3><<<g, kThreads, 0, s>>>(x, outer, k_in, inner, k_out, size, stride, dilation,
                                                                pad_lo, out);
  else
    window_f32_kernel<OP, INCLUDE_PAD, 0><<<g, kThreads, 0, s>>>(x, outer, k_in, inner, k_out, size, stride, dilation,
                                                                pad_lo, out);
}

template <int OP>
__global__ void __launch_bounds__(kThreads) window_i32_kernel(const int32_t* __restrict__ x, int64_t outer,
                                                               int64_t k_in, int64_t inner, int64_t k_out, int size,
                                                               int stride, int dilation, int pad_lo,
                                                               int32_t* __restrict__ out) {
  window_walk<int32_t>(x, outer, k_in, inner, k_out, stride, pad_lo, out,
                       [&](const int32_t* src, int64_t step, int64_t p0) {
                         return window_i32_one<OP>(src, step, p0, k_in, size, dilation);
                       });
}

// Windows along an outer or middle axis (inner > 1) whose inner extent is a multiple of 4 floats, with dilation 1
// and the common sizes and strides: a thread takes U = 2 consecutive outputs o of one (b, 4-float column) and loads
// every input line those outputs touch before folding either: L = STRIDE + SZ lines (5 for a 3/2 pool), so a line
// shared by the two outputs is read once and L 16-byte loads are in flight per thread, against one tap at a time on
// the line path. (Four outputs a thread, 9 lines, measured 1.17x slower: more registers, fewer warps per SM; one
// output, 1.10x; 8-byte columns, 1.2-1.4x.) The folds are the line path's, per float: the same taps in the same
// order.
template <int OP, bool INCLUDE_PAD, int SZ>
__device__ __forceinline__ float fold_taps(const float (&v)[SZ], const bool (&ok)[SZ]) {
  if (OP == UP_OP_SUM || OP == UP_OP_MEAN) {
    double acc = 0.0;
    int cnt = 0;
#pragma unroll
    for (int kk = 0; kk < SZ; ++kk)
      if (ok[kk]) {
        acc += (double)v[kk];
        ++cnt;
      }
    if (OP == UP_OP_MEAN) acc = mean_div<SZ>(acc, INCLUDE_PAD ? SZ : cnt);
    return __double2float_rn(acc);
  } else {
    uint32_t best = 0, nan_bits = 0;
    bool have = false, nan = false;
#pragma unroll
    for (int kk = 0; kk < SZ; ++kk) {
      if (!ok[kk]) continue;
      const float x = v[kk];
      if (x != x) {
        nan = true;
        nan_bits = __float_as_uint(x);
      } else if (!have || (OP == UP_OP_MAX ? x > __uint_as_float(best) : x < __uint_as_float(best))) {
        best = __float_as_uint(x);
      }
      have = have || x == x;
    }
    return __uint_as_float(nan ? (nan_bits | 0x00400000u) : best);
  }
}

template <int VEC>
struct FVec;
template <>
struct FVec<2> {
  using T = float2;
  static __device__ __forceinline__ float get(const float2& q, int c) { return c == 0 ? q.x : q.y; }
  static __device__ __forceinline__ float2 make(const float (&r)[2]) { return make_float2(r[0], r[1]); }
  static __device__ __forceinline__ float2 zero() { return make_float2(0.f, 0.f); }
};
template <>
struct FVec<4> {
  using T = float4;
  static __device__ __forceinline__ float get(const float4& q, int c) {
    return c == 0 ? q.x : c == 1 ? q.y : c == 2 ? q.z : q.w;
  }
  static __device__ __forceinline__ float4 make(const float (&r)[4]) { return make_float4(r[0], r[1], r[2], r[3]); }
  static __device__ __forceinline__ float4 zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
};

// VEC floats a thread per column (inner4 counts these vectors), U outputs a thread.
template <int OP, bool INCLUDE_PAD, int SZ, int STRIDE, int VEC, int U>
__device__ __forceinline__ void window_cols_body(const typename FVec<VEC>::T* __restrict__ x, int64_t outer,
                                                 int64_t k_in, int64_t inner4, int64_t k_out, int pad_lo,
                                                 typename FVec<VEC>::T* __restrict__ out) {
  using V = FVec<VEC>;
  using T = typename V::T;
  constexpr int L = (U - 1) * STRIDE + SZ;
  const int64_t groups = (k_out + U - 1) / U;  // output groups per b
  const int64_t rows = outer * groups;         // (b, group) pairs
  // rows narrower than the CTA share it: lp rows per step, thread t on row t / inner4, column t % inner4
  const int lp = inner4 < kThreads ? kThreads / (int)inner4 : 1;
  const int sub = inner4 < kThreads ? (int)threadIdx.x / (int)inner4 : 0;
  const int64_t c0 = inner4 < kThreads ? (int64_t)threadIdx.x - (int64_t)sub * inner4 : threadIdx.x;
  if (sub >= lp) return;  // the threads past lp whole rows
  for (int64_t r = (int64_t)blockIdx.x * lp + sub; r < rows; r += (int64_t)gridDim.x * lp) {
    const int64_t b = r / groups, g = r - b * groups;
    const int64_t p0 = g * U * STRIDE - pad_lo;  // input position of line 0
    const T* xb = x + b * k_in * inner4;
    T* ob = out + (b * k_out + g * U) * inner4;
    for (int64_t c = c0; c < inner4; c += kThreads) {
      T line[L];
      bool ok[L];
#pragma unroll
      for (int j = 0; j < L; ++j) {
        const int64_t p = p0 + j;
        ok[j] = p >= 0 && p < k_in;
        line[j] = ok[j] ? __ldg(xb + p * inner4 + c) : V::zero();
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (g * U + u >= k_out) break;
        bool tok[SZ];
#pragma unroll
        for (int kk = 0; kk < SZ; ++kk) tok[kk] = ok[u * STRIDE + kk];
        float res[VEC];
#pragma unroll
        for (int q = 0; q < VEC; ++q) {
          float v[SZ];
#pragma unroll
          for (int kk = 0; kk < SZ; ++kk) v[kk] = V::get(line[u * STRIDE + kk], q);
          res[q] = fold_taps<OP, INCLUDE_PAD, SZ>(v, tok);
        }
        ob[(int64_t)u * inner4 + c] = V::make(res);
      }
    }
  }
}

// A register cap of four CTAs per SM for Max/Min keeps more lines in flight per SM (1.05x). The f64 Sum/Mean folds
// spill under a cap of three and use up to 96 registers when told one CTA suffices, so they take the default bound.
template <int OP, bool INCLUDE_PAD, int SZ, int STRIDE, int VEC, int U>
__global__ void __launch_bounds__(kThreads, 4) window_f32_cols_ext_kernel(const typename FVec<VEC>::T* __restrict__ x,
                                                                           int64_t outer, int64_t k_in, int64_t inner4,
                                                                           int64_t k_out, int pad_lo,
                                                                           typename FVec<VEC>::T* __restrict__ out) {
  window_cols_body<OP, INCLUDE_PAD, SZ, STRIDE, VEC, U>(x, outer, k_in, inner4, k_out, pad_lo, out);
}
template <int OP, bool INCLUDE_PAD, int SZ, int STRIDE, int VEC, int U>
__global__ void __launch_bounds__(kThreads) window_f32_cols_sum_kernel(const typename FVec<VEC>::T* __restrict__ x,
                                                                        int64_t outer, int64_t k_in, int64_t inner4,
                                                                        int64_t k_out, int pad_lo,
                                                                        typename FVec<VEC>::T* __restrict__ out) {
  window_cols_body<OP, INCLUDE_PAD, SZ, STRIDE, VEC, U>(x, outer, k_in, inner4, k_out, pad_lo, out);
}

inline int grid_for(int64_t units);
constexpr int kColVec = 4, kColOutputs = 2;  // floats a thread per column, outputs a thread

// Launches the column kernel when it covers the shape; false leaves it to the line path.
template <int OP, bool INCLUDE_PAD>
bool launch_cols(const float* x, int64_t outer, int64_t k_in, int64_t inner, int64_t k_out, int size, int stride,
                 int dilation, int pad_lo, float* out, cudaStream_t s) {
  constexpr int VEC = kColVec, U = kColOutputs;
  if (inner < VEC || inner % VEC != 0 || dilation != 1 || !aligned(x, 4 * VEC) || !aligned(out, 4 * VEC)) return false;
  if (!((size == 2 || size == 3) && (stride == 1 || stride == 2))) return false;
  const int64_t inner4 = inner / VEC;
  const int64_t lp = inner4 < kThreads ? kThreads / inner4 : 1;
  const int64_t rows = outer * ((k_out + U - 1) / U);
  const int g = grid_for((rows + lp - 1) / lp);
  using T = typename FVec<VEC>::T;
  const T* x4 = reinterpret_cast<const T*>(x);
  T* o4 = reinterpret_cast<T*>(out);
#define UP_COLS(SZ, ST)                                                                                          \
  do {                                                                                                                  \
    if constexpr (OP == UP_OP_MAX || OP == UP_OP_MIN)                                                                   \
      window_f32_cols_ext_kernel<OP, INCLUDE_PAD, SZ, ST, VEC, U><<<g, kThreads, 0, s>>>(x4, outer, k_in, inner4,      \
                                                                                       k_out, pad_lo, o4);             \
    else                                                                                                                \
      window_f32_cols_sum_kernel<OP, INCLUDE_PAD, SZ, ST, VEC, U><<<g, kThreads, 0, s>>>(x4, outer, k_in, inner4,      \
                                                                                       k_out, pad_lo, o4);             \
  } while (0)
  if (size == 2 && stride == 1) UP_COLS(2, 1);
  else if (size == 2) UP_COLS(2, 2);
  else if (stride == 1) UP_COLS(3, 1);
  else UP_COLS(3, 2);
#undef UP_COLS
  return true;
}

// Windows along an outer or middle axis with 16-byte columns, staged: a CTA takes one (b, tile of TO outputs) item
// and copies every input line the tile touches into shared memory with cp.async (all of the tile's copies in flight
// together, no registers held by the loads), then folds each output from shared memory, a 16-byte read per tap.
// A 32 KiB buffer holds 2,048 16-byte columns: 64 lines of 128 floats, 31 outputs of a 3/2 pool. Any size, stride and
// dilation whose tile fits; the taps, their order and the folds are the line path's, per float.
constexpr int kLineStageVecs = 2048;  // 16-byte columns in the 32 KiB buffer
template <int OP, bool INCLUDE_PAD, int SZ>
__global__ void __launch_bounds__(kThreads) window_f32_lines_staged_kernel(const float4* __restrict__ x,
                                                                          int64_t outer, int64_t k_in, int inner4,
                                                                          int64_t k_out, int size_rt, int stride,
                                                                          int dilation, int pad_lo, int TO,
                                                                          float4* __restrict__ out) {
  __shared__ __align__(16) float4 stage[kLineStageVecs];
  const int size = SZ > 0 ? SZ : size_rt;
  const int64_t tiles = (k_out + TO - 1) / TO;
  const int64_t items = outer * tiles;
  // threads over (line or output, column): lp rows of inner4 columns a step, one division per thread
  const int lp = inner4 < kThreads ? kThreads / inner4 : 1;
  const int sub = inner4 < kThreads ? (int)threadIdx.x / inner4 : 0;
  const int c0 = inner4 < kThreads ? (int)threadIdx.x - sub * inner4 : (int)threadIdx.x;
  const int cstep = inner4 < kThreads ? inner4 : kThreads;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int64_t b = it / tiles, t = it - b * tiles;
    const int64_t o0 = t * TO;
    const int to = (int)(k_out - o0 < TO ? k_out - o0 : TO);
    const int64_t p_lo = o0 * stride - pad_lo;  // input position of staged line 0
    const int lines = (to - 1) * stride + (size - 1) * dilation + 1;
    // the staged lines that lie inside the axis: [j_lo, j_hi)
    const int j_lo = p_lo < 0 ? (int)-p_lo : 0;
    const int j_hi = p_lo + lines > k_in ? (int)(k_in - p_lo) : lines;
    if (sub < lp) {
      const int64_t base = (b * k_in + p_lo) * inner4;  // column 0 of staged line 0 (>= 0 for every line copied)
      for (int j = j_lo + sub; j < j_hi; j += lp)
        for (int c = c0; c < inner4; c += cstep)
          stage_copy16(&stage[j * inner4 + c], x + base + (int64_t)j * inner4 + c);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    if (sub < lp) {
      float4* ob = out + (b * k_out + o0) * inner4;
      for (int ol = sub; ol < to; ol += lp)
        for (int c = c0; c < inner4; c += cstep) {
          const int j0 = ol * stride;
          // every tap of the output inside the axis (all but the edge outputs): no range test per tap
          const bool interior = j0 >= j_lo && j0 + (size - 1) * dilation < j_hi;
          float res[4];
          if (OP == UP_OP_SUM || OP == UP_OP_MEAN) {
            double acc[4] = {0.0, 0.0, 0.0, 0.0};
            int cnt = 0;
            for (int kk = 0; kk < size; ++kk) {
              const int j = j0 + kk * dilation;
              if (!interior && (j < j_lo || j >= j_hi)) continue;
              const float4 v = stage[j * inner4 + c];
              acc[0] += (double)v.x;
              acc[1] += (double)v.y;
              acc[2] += (double)v.z;
              acc[3] += (double)v.w;
              ++cnt;
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const double a = OP == UP_OP_MEAN ? mean_div<SZ>(acc[q], INCLUDE_PAD ? size : cnt) : acc[q];
              res[q] = __double2float_rn(a);
            }
          } else if (interior) {
            // Max/Min branch-free from the first tap, the last NaN's bits tracked beside it (1.47x on a 3/2 pool)
            const float4 f4 = stage[j0 * inner4 + c];
            float bv[4] = {f4.x, f4.y, f4.z, f4.w};
            uint32_t nb[4];
            bool nan[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              nb[q] = __float_as_uint(bv[q]);
              nan[q] = bv[q] != bv[q];
            }
            for (int kk = 1; kk < size; ++kk) {
              const float4 v4 = stage[(j0 + kk * dilation) * inner4 + c];
              const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const bool vn = vv[q] != vv[q];
                nb[q] = vn ? __float_as_uint(vv[q]) : nb[q];
                nan[q] = nan[q] || vn;
                bv[q] = (OP == UP_OP_MAX ? vv[q] > bv[q] : vv[q] < bv[q]) ? vv[q] : bv[q];
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
              res[q] = __uint_as_float(nan[q] ? (nb[q] | 0x00400000u) : __float_as_uint(bv[q]));
          } else {
            uint32_t best[4] = {0u, 0u, 0u, 0u}, nan_bits[4] = {0u, 0u, 0u, 0u};
            bool have[4] = {false, false, false, false}, nan[4] = {false, false, false, false};
            for (int kk = 0; kk < size; ++kk) {
              const int j = j0 + kk * dilation;
              if (j < j_lo || j >= j_hi) continue;
              const float4 v4 = stage[j * inner4 + c];
              const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float v = vv[q];
                if (v != v) {
                  nan[q] = true;
                  nan_bits[q] = __float_as_uint(v);
                } else if (!have[q] ||
                           (OP == UP_OP_MAX ? v > __uint_as_float(best[q]) : v < __uint_as_float(best[q]))) {
                  best[q] = __float_as_uint(v);
                }
                have[q] = have[q] || v == v;
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) res[q] = __uint_as_float(nan[q] ? (nan_bits[q] | 0x00400000u) : best[q]);
          }
          ob[(int64_t)ol * inner4 + c] = make_float4(res[0], res[1], res[2], res[3]);
        }
    }
    __syncthreads();  // the tile is read before the next one is staged
  }
}

// Launches the staged kernel when a tile of at least 8 outputs fits the buffer; false leaves it to the other paths.
template <int OP, bool INCLUDE_PAD>
bool launch_lines_staged(const float* x, int64_t outer, int64_t k_in, int64_t inner, int64_t k_out, int size,
                         int stride, int dilation, int pad_lo, float* out, cudaStream_t s) {
  if (inner < 4 || inner % 4 != 0 || !aligned(x, 16) || !aligned(out, 16)) return false;
  const int64_t inner4 = inner / 4;
  if (inner4 > kLineStageVecs) return false;
  const int64_t lt = kLineStageVecs / inner4;  // lines the buffer holds
  const int64_t span = (int64_t)(size - 1) * dilation;
  if (lt - 1 - span < 0) return false;
  const int64_t to = (lt - 1 - span) / stride + 1;  // outputs a tile
  if (to < 8) return false;
  const int64_t items = outer * ((k_out + to - 1) / to);
  const int g = grid_for(items);
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float4* o4 = reinterpret_cast<float4*>(out);
#define UP_LS(SZ)                                                                                                   \
  window_f32_lines_staged_kernel<OP, INCLUDE_PAD, SZ><<<g, kThreads, 0, s>>>(x4, outer, k_in, (int)inner4, k_out, size, \
                                                                             stride, dilation, pad_lo, (int)to, o4)
  if (size == 2) UP_LS(2);
  else if (size == 3) UP_LS(3);
  else UP_LS(0);
#undef UP_LS
  return true;
}

// A CTA per output row (n, c, ki, kj), decoded once; its threads walk the row's oH·oW cells with 32-bit
// arithmetic (the row length fits: oH·oW < 2^31 is checked on the host).
template <typename T>
__global__ void __launch_bounds__(kThreads) im2col_kernel(const T* __restrict__ x, int64_t n, int64_t c, int64_t h,
                                                           int64_t w, int kh, int kw, int sh, int sw, int ph, int pw,
                                                           int dh, int dw, int64_t oh_n, int64_t ow_n,
                                                           T* __restrict__ out) {
  const int cols = (int)(oh_n * ow_n), own = (int)ow_n;
  const int64_t rows = n * c * kh * kw;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t patch = row % (c * kh * kw), nn = row / (c * kh * kw);
    const int64_t cc = patch / (kh * kw);
    const int kij = (int)(patch - cc * (kh * kw));
    const int ki = kij / kw, kj = kij - ki * kw;
    const T* plane = x + (nn * c + cc) * h * w;
    T* orow = out + row * cols;
    const int ih0 = ki * dh - ph, iw0 = kj * dw - pw;
    for (int col = threadIdx.x; col < cols; col += kThreads) {
      const int oh = col / own, ow = col - oh * own;
      const int ih = oh * sh + ih0, iw = ow * sw + iw0;
      T v{};
      if (ih >= 0 && ih < h && iw >= 0 && iw < w) v = __ldg(plane + (int64_t)ih * w + iw);
      orow[col] = v;
    }
  }
}

// A CTA per input plane (n, c) that fits in shared memory: the plane is staged once, coalesced, then the CTA writes
// the plane's kh·kw output rows from shared memory. With VEC > 1 (an output row width that is a multiple of VEC
// elements of 16 / sizeof(T)), a thread takes VEC consecutive cells of one output row and writes each of its kh·kw
// rows' cells with one 16-byte evict-first store: the output is the bulk of the traffic and is not read again.
constexpr int64_t kPlaneBytes = 96 * 1024;
template <typename T, int VEC>
__global__ void __launch_bounds__(kThreads) im2col_plane_kernel(const T* __restrict__ x, int64_t planes, int h, int w,
                                                                 int kh, int kw, int sh, int sw, int ph, int pw, int dh,
                                                                 int dw, int oh_n, int ow_n, T* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char plane_raw[];
  T* plane = reinterpret_cast<T*>(plane_raw);
  const int hw = h * w, cols = oh_n * ow_n;
  for (int64_t pl = blockIdx.x; pl < planes; pl += gridDim.x) {
    const T* src = x + pl * hw;
    const int bytes = hw * (int)sizeof(T);
    if ((((uintptr_t)src | (uintptr_t)bytes) & 15) == 0) {  // 16-byte cp.async: every copy of the plane in flight
      for (int i = threadIdx.x; i < bytes / 16; i += kThreads)
        stage_copy16(plane_raw + 16 * i, reinterpret_cast<const unsigned char*>(src) + 16 * i);
      asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    } else {
      for (int i = threadIdx.x; i < hw; i += kThreads) plane[i] = __ldg(src + i);
    }
    __syncthreads();
    // a thread decodes its cell (oh, ow) once and writes it in all kh·kw rows (each store coalesced across the warp)
    T* const orow = out + pl * kh * kw * (int64_t)cols;
    if constexpr (VEC > 1) {
      static_assert(VEC * sizeof(T) == 16, "one 16-byte store per vector of cells");
      for (int col = threadIdx.x * VEC; col < cols; col += kThreads * VEC) {
        const int oh = col / ow_n, ow = col - oh * ow_n;  // the VEC cells share oh: ow_n is a multiple of VEC
        const int ihb = oh * sh - ph, iwb = ow * sw - pw;
        T* o = orow + col;
        for (int ki = 0; ki < kh; ++ki) {
          const int ih = ihb + ki * dh;
          const bool in_h = ih >= 0 && ih < h;
          for (int kj = 0; kj < kw; ++kj, o += cols) {
            union {
              T e[VEC];
              uint4 v;
            } pk;
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
              const int iw = iwb + v * sw + kj * dw;
              pk.e[v] = (in_h && iw >= 0 && iw < w) ? plane[ih * w + iw] : T{};
            }
            st_cs_v4(o, pk.v);
          }
        }
      }
    } else {
      for (int col = threadIdx.x; col < cols; col += kThreads) {
        const int oh = col / ow_n, ow = col - oh * ow_n;
        const int ihb = oh * sh - ph, iwb = ow * sw - pw;
        T* o = orow + col;
        for (int ki = 0; ki < kh; ++ki) {
          const int ih = ihb + ki * dh;
          const bool in_h = ih >= 0 && ih < h;
          for (int kj = 0; kj < kw; ++kj, o += cols) {
            const int iw = iwb + kj * dw;
            *o = (in_h && iw >= 0 && iw < w) ? plane[ih * w + iw] : T{};
          }
        }
      }
    }
    __syncthreads();  // the plane is read before the next one is staged
  }
}

inline int grid_for(int64_t units) {  // one unit (a row or a line) per CTA at a time, up to 16 CTAs per SM
  const int64_t cap = (int64_t)sm_count() * 16;
  return (int)(units < cap ? (units > 0 ? units : 1) : cap);
}

}  // namespace win
}  // namespace up

using namespace up;

// True when every output window holds an in-bounds tap (window_taps::check_window_taps).
static bool every_window_has_a_tap(int64_t k_in, int64_t k_out, int size, int stride, int dilation, int pad_lo) {
  for (int64_t o = 0; o < k_out; ++o) {
    const int64_t p0 = o * stride - pad_lo;
    int64_t kk = p0 >= 0 ? 0 : (-p0 + dilation - 1) / dilation;  // the first tap at or after 0
    if (kk >= size || p0 + kk * dilation >= k_in) return false;
  }
  return true;
}

extern "C" int up_sm100_window(const void* x, int dtype, int64_t outer, int64_t k_in, int64_t inner, int op, int size,
                               int stride, int dilation, int pad_lo, int count_include_pad, void* out, int64_t k_out,
                               void* stream) {
  UP_CHECK_ARG(outer >= 0 && k_in >= 0 && inner >= 0 && k_out >= 0);
  if (size < 1 || stride < 1 || dilation < 1 || pad_lo < 0)
    return fail_with(UP_ERR_UNSUPPORTED, "window: size, stride and dilation >= 1, pad >= 0");
  if (dtype != UP_EK_F32 && dtype != UP_EK_I32) return fail_with(UP_ERR_UNSUPPORTED, "window: f32 or i32");
  if (op != UP_OP_SUM && op != UP_OP_MEAN && op != UP_OP_MAX && op != UP_OP_MIN)
    return fail_with(UP_ERR_UNSUPPORTED, "window: Sum, Mean, Max or Min (Prod is refused)");
  if (dtype == UP_EK_I32 && op == UP_OP_MEAN) return fail_with(UP_ERR_UNSUPPORTED, "window: an integer Mean");
  const int64_t total = outer * k_out * inner;
  if (total == 0) return UP_OK;
  if (!every_window_has_a_tap(k_in, k_out, size, stride, dilation, pad_lo))
    return fail_with(UP_ERR_UNSUPPORTED, "window: a window with no in-bounds tap");
  UP_CHECK_ARG(x != nullptr && out != nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t lp = inner > 1 && inner < win::kThreads ? win::kThreads / inner : 1;
  const int g = win::grid_for(inner == 1 ? outer : (outer * k_out + lp - 1) / lp);
  if (dtype == UP_EK_F32 && inner == 1 && k_in * 4 <= win::kRowStageBytes) {
    const float* xf = static_cast<const float*>(x);
    float* of = static_cast<float*>(out);
#define UP_WIN_S(OP, INC) win::launch_staged<OP, INC>(xf, outer, k_in, k_out, size, stride, dilation, pad_lo, of, g, s)
    switch (op) {
      case UP_OP_SUM: UP_WIN_S(UP_OP_SUM, false); break;
      case UP_OP_MEAN:
        if (count_include_pad) UP_WIN_S(UP_OP_MEAN, true);
        else UP_WIN_S(UP_OP_MEAN, false);
        break;
      case UP_OP_MAX: UP_WIN_S(UP_OP_MAX, false); break;
      default: UP_WIN_S(UP_OP_MIN, false); break;
    }
#undef UP_WIN_S
  } else if (dtype == UP_EK_F32) {
    const float* xf = static_cast<const float*>(x);
    float* of = static_cast<float*>(out);
#define UP_WIN_F32(OP, INC)                                                                                      \
  (void)(win::launch_lines_staged<OP, INC>(xf, outer, k_in, inner, k_out, size, stride, dilation, pad_lo, of, s) || \
         win::launch_cols<OP, INC>(xf, outer, k_in, inner, k_out, size, stride, dilation, pad_lo, of, s) ||         \
         (win::launch_lines<OP, INC>(xf, outer, k_in, inner, k_out, size, stride, dilation, pad_lo, of, g, s), true))
    switch (op) {
      case UP_OP_SUM: UP_WIN_F32(UP_OP_SUM, false); break;
      case UP_OP_MEAN:
        if (count_include_pad) UP_WIN_F32(UP_OP_MEAN, true);
        else UP_WIN_F32(UP_OP_MEAN, false);
        break;
      case UP_OP_MAX: UP_WIN_F32(UP_OP_MAX, false); break;
      default: UP_WIN_F32(UP_OP_MIN, false); break;
    }
#undef UP_WIN_F32
  } else {
    const int32_t* xi = static_cast<const int32_t*>(x);
    int32_t* oi = static_cast<int32_t*>(out);
    if (op == UP_OP_SUM)
      win::window_i32_kernel<UP_OP_SUM><<<g, win::kThreads, 0, s>>>(xi, outer, k_in, inner, k_out, size, stride, dilation, pad_lo, oi);
    else if (op == UP_OP_MAX)
      win::window_i32_kernel<UP_OP_MAX><<<g, win::kThreads, 0, s>>>(xi, outer, k_in, inner, k_out, size, stride, dilation, pad_lo, oi);
    else
      win::window_i32_kernel<UP_OP_MIN><<<g, win::kThreads, 0, s>>>(xi, outer, k_in, inner, k_out, size, stride, dilation, pad_lo, oi);
  }
  note_launch();
  return check_launch();
}

extern "C" int up_sm100_im2col(const void* x, int elem_bytes, int64_t n, int64_t c, int64_t h, int64_t w, int kh,
                               int kw, int sh, int sw, int ph, int pw, int dh, int dw, void* out, void* stream) {
  UP_CHECK_ARG(n >= 0 && c >= 0 && h >= 0 && w >= 0);
  if (kh < 1 || kw < 1 || sh < 1 || sw < 1 || dh < 1 || dw < 1 || ph < 0 || pw < 0)
    return fail_with(UP_ERR_UNSUPPORTED, "im2col: kernel, stride and dilation >= 1, pad >= 0");
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8) return UP_ERR_UNSUPPORTED;
  const int64_t oh = (h + 2 * (int64_t)ph - (int64_t)dh * (kh - 1) - 1) / sh + 1;
  const int64_t ow = (w + 2 * (int64_t)pw - (int64_t)dw * (kw - 1) - 1) / sw + 1;
  if (oh <= 0 || ow <= 0) return fail_with(UP_ERR_UNSUPPORTED, "im2col: the window is larger than the padded input");
  const int64_t total = n * c * kh * kw * oh * ow;
  if (total == 0) return UP_OK;
  // 32-bit cell loops step by up to kThreads * 16 cells past the row's end: keep that headroom below 2^31
  if (oh * ow > 0x7fffffffLL - 16 * win::kThreads || h > 0x7fffffffLL || w > 0x7fffffffLL) return UP_ERR_UNSUPPORTED;
  UP_CHECK_ARG(x != nullptr && out != nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int g = win::grid_for(n * c * kh * kw);
  const int64_t plane_bytes = h * w * (int64_t)elem_bytes;
  if (plane_bytes <= win::kPlaneBytes && oh * ow <= 0x7fffffffLL && kh * kw <= 0x7fff) {
    const int mx = (int)win::kPlaneBytes;
    // 16-byte stores of 16 / elem_bytes cells when every output row holds whole vectors
    const bool vec = ow % (16 / elem_bytes) == 0 && aligned(out, 16);
    const int gp = win::grid_for(n * c);
    cudaError_t e = cudaSuccess;
#define UP_I2P(T, V)                                                                                                 \
  do {                                                                                                               \
    e = ensure_smem_attr((const void*)win::im2col_plane_kernel<T, V>, mx);                                          \
    if (e == cudaSuccess)                                                                                            \
      win::im2col_plane_kernel<T, V><<<gp, win::kThreads, (size_t)plane_bytes, s>>>(                                \
          static_cast<const T*>(x), n * c, (int)h, (int)w, kh, kw, sh, sw, ph, pw, dh, dw, (int)oh, (int)ow,       \
          static_cast<T*>(out));                                                                                     \
  } while (0)
    switch (elem_bytes) {
      case 1: if (vec) UP_I2P(uint8_t, 16); else UP_I2P(uint8_t, 1); break;
      case 2: if (vec) UP_I2P(uint16_t, 8); else UP_I2P(uint16_t, 1); break;
      case 4: if (vec) UP_I2P(uint32_t, 4); else UP_I2P(uint32_t, 1); break;
      default: if (vec) UP_I2P(unsigned long long, 2); else UP_I2P(unsigned long long, 1); break;
    }
#undef UP_I2P
    if (e != cudaSuccess) return cuda_status(e);
    note_launch();
    return check_launch();
  }
#define UP_I2C(T) \
  win::im2col_kernel<T><<<g, win::kThreads, 0, s>>>(static_cast<const T*>(x), n, c, h, w, kh, kw, sh, sw, ph, pw, dh, dw, oh, ow, static_cast<T*>(out))
  switch (elem_bytes) {
    case 1: UP_I2C(uint8_t); break;
    case 2: UP_I2C(uint16_t); break;
    case 4: UP_I2C(uint32_t); break;
    default: UP_I2C(unsigned long long); break;
  }
#undef UP_I2C
  note_launch();
  return check_launch();
}

UP_DEFINE_REVISION(window)
