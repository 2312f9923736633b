// reduce2d.cu — the breadth of the reduction lift on a rank-2 [rows, cols] input reduced over one axis: f32 Mean,
// Max and Min, and i32 Sum, Prod, Max, Min, And, Or and Xor, over the last axis (axis 1, out[rows]) or the outer
// axis (axis 0, out[cols]). f32 Sum over the last axis is reduce.cu's row sum; Mean over the last axis reuses it.
//
// Semantics: eval_reduction (crates/unpopped/src/oracle/plan_eval.rs:501-651) with fold_step, extremum_fold and
// bit_fold (oracle/plan_contract.rs:146-245):
//  * i32 Sum and Prod wrap at 32 bits (the oracle's i128 fold wrapped at 64 bits, stored at the dtype's width);
//    Max/Min exact; And/Or/Xor seeded by the first element; an empty fold stores 0, or 1 for Prod. Every one of
//    these is associative and commutative, so any combine order gives the oracle's bits.
//  * f32 Max/Min keep the first element and replace it by a NaN or by a strictly better value: the result is the
//    row's last NaN if it has one (widened through f64 and back, so with the quiet bit set), else the first
//    element of the extreme value (so the first zero's sign when +0 and -0 tie). The kernels reduce a packed
//    (order key, inverted index) word and a last-NaN index, both order-independent, then copy that element's bits.
//  * f32 Sum/Mean over the outer axis fold each column in the serial order in f64 (one thread per column: the
//    order is the oracle's, not a tree), one rounding; Mean divides by the row count, so an empty Mean is 0/0.
#include "common.cuh"

namespace up {
namespace r2 {

constexpr int kThreads = 256;

template <int OP>
__device__ __forceinline__ int32_t ident() {
  if (OP == UP_OP_PROD) return 1;
  if (OP == UP_OP_MAX) return INT32_MIN;
  if (OP == UP_OP_MIN) return INT32_MAX;
  if (OP == UP_OP_AND) return -1;
  return 0;  // Sum, Or, Xor
}

template <int OP>
__device__ __forceinline__ int32_t comb(int32_t a, int32_t b) {
  if (OP == UP_OP_SUM) return (int32_t)((uint32_t)a + (uint32_t)b);
  if (OP == UP_OP_PROD) return (int32_t)((uint32_t)a * (uint32_t)b);
  if (OP == UP_OP_MAX) return a > b ? a : b;
  if (OP == UP_OP_MIN) return a < b ? a : b;
  if (OP == UP_OP_AND) return a & b;
  if (OP == UP_OP_OR) return a | b;
  return a ^ b;
}

template <int OP>
__device__ __forceinline__ int32_t comb4(int32_t a, uint4 v) {
  a = comb<OP>(a, (int32_t)v.x);
  a = comb<OP>(a, (int32_t)v.y);
  a = comb<OP>(a, (int32_t)v.z);
  return comb<OP>(a, (int32_t)v.w);
}

template <int OP>
__device__ __forceinline__ int32_t block_comb(int32_t a, int32_t* part) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = comb<OP>(a, __shfl_xor_sync(0xffffffffu, a, o));
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = a;
  __syncthreads();
  int32_t t = part[0];
#pragma unroll
  for (int i = 1; i < kThreads / 32; ++i) t = comb<OP>(t, part[i]);
  __syncthreads();
  return t;
}

// ---- i32, last axis: one CTA per row, 16-byte loads when the rows allow ----
template <int OP, bool VEC>
__global__ void __launch_bounds__(kThreads) row_fold_i32_kernel(const int32_t* __restrict__ x, int64_t rows,
                                                                 int64_t cols, int64_t stride,
                                                                 int32_t* __restrict__ out) {
  __shared__ int32_t part[kThreads / 32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int32_t* row = x + r * stride;
    int32_t acc = ident<OP>();
    if (VEC) {
      const uint4* rv = reinterpret_cast<const uint4*>(row);
      const int64_t nv = cols / 4;
      int64_t i = threadIdx.x;
      for (; i + 3 * kThreads < nv; i += 4 * kThreads) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = ld_nc_na_v4(rv + i + u * kThreads);
#pragma unroll
        for (int u = 0; u < 4; ++u) acc = comb4<OP>(acc, v[u]);
      }
      for (; i < nv; i += kThreads) acc = comb4<OP>(acc, ld_nc_na_v4(rv + i));
    } else {
      for (int64_t c = threadIdx.x; c < cols; c += kThreads) acc = comb<OP>(acc, __ldg(row + c));
    }
    acc = block_comb<OP>(acc, part);
    if (threadIdx.x == 0) out[r] = cols > 0 ? acc : (OP == UP_OP_PROD ? 1 : 0);
  }
}

// ---- i32, outer axis: a thread per column (coalesced across the row), rows split over gridDim.y; the splits
// combine into out with atomics (out holds the identity first). ----
template <int OP>
__global__ void col_init_i32_kernel(int32_t* __restrict__ out, int64_t cols) {
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += (int64_t)gridDim.x * blockDim.x)
    out[c] = ident<OP>();
}

template <int OP>
__global__ void __launch_bounds__(kThreads) col_fold_i32_kernel(const int32_t* __restrict__ x, int64_t rows,
                                                                 int64_t cols, int64_t stride, int64_t per_split,
                                                                 int32_t* __restrict__ out) {
  const int64_t c = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  const int64_t r0 = (int64_t)blockIdx.y * per_split;
  const int64_t r1 = r0 + per_split < rows ? r0 + per_split : rows;
  int32_t acc = ident<OP>();
  int64_t r = r0;
  for (; r + 3 < r1; r += 4) {
    int32_t v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldg(x + (r + u) * stride + c);
#pragma unroll
    for (int u = 0; u < 4; ++u) acc = comb<OP>(acc, v[u]);
  }
  for (; r < r1; ++r) acc = comb<OP>(acc, __ldg(x + r * stride + c));
  int32_t* o = out + c;
  if (OP == UP_OP_SUM) atomicAdd(o, acc);
  else if (OP == UP_OP_MAX) atomicMax(o, acc);
  else if (OP == UP_OP_MIN) atomicMin(o, acc);
  else if (OP == UP_OP_AND) atomicAnd(o, acc);
  else if (OP == UP_OP_OR) atomicOr(o, acc);
  else if (OP == UP_OP_XOR) atomicXor(o, acc);
  else {  // Prod: no atomic multiply; a compare-and-swap loop (each retry sees a newer value, so it ends)
    int32_t old = *reinterpret_cast<volatile int32_t*>(o), seen;
    do {
      seen = old;
      old = atomicCAS(o, seen, comb<OP>(seen, acc));
    } while (old != seen);
  }
}

// ---- f32 Max/Min ----
// Order key of a non-NaN f32 (-0 counted as +0); MIN ranks by the inverted key. The packed word puts the key above
// the inverted index, so the greatest word is the best value at its first index; 0 means "no element".
template <bool MAX>
__device__ __forceinline__ uint64_t ext_pack(uint32_t u, uint32_t idx) {
  if (u == 0x80000000u) u = 0;
  const uint32_t key = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((uint64_t)(MAX ? key : ~key) << 32) | (uint64_t)(0xffffffffu - idx);
}

__device__ __forceinline__ bool f32_isnan_bits(uint32_t u) { return (u & 0x7fffffffu) > 0x7f800000u; }

template <bool MAX>
__device__ __forceinline__ void ext_take(uint32_t u, uint32_t idx, uint64_t& best, int64_t& nan_idx) {
  if (f32_isnan_bits(u)) {
    nan_idx = (int64_t)idx > nan_idx ? (int64_t)idx : nan_idx;
  } else {
    const uint64_t p = ext_pack<MAX>(u, idx);
    best = p > best ? p : best;
  }
}

// the result's bits from the fold's state: the last NaN (quiet bit set), else the best element, else 0 (empty)
__device__ __forceinline__ uint32_t ext_result(const float* base, int64_t step, uint64_t best, int64_t nan_idx) {
  if (nan_idx >= 0) return __float_as_uint(base[nan_idx * step]) | 0x00400000u;
  if (best == 0) return 0u;
  return __float_as_uint(base[(int64_t)(0xffffffffu - (uint32_t)best) * step]);
}

template <bool MAX, bool VEC>
__global__ void __launch_bounds__(kThreads) row_extremum_f32_kernel(const float* __restrict__ x, int64_t rows,
                                                                     int64_t cols, int64_t stride,
                                                                     float* __restrict__ out) {
  __shared__ uint64_t sbest[kThreads / 32];
  __shared__ int64_t snan[kThreads / 32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* row = x + r * stride;
    uint64_t best = 0;
    int64_t nan_idx = -1;
    if (VEC) {
      const int64_t nv = cols / 4;
      for (int64_t i = threadIdx.x; i < nv; i += kThreads) {
        const float4 f = ld_nc_na_f4(row + 4 * i);
        const uint32_t c = (uint32_t)(4 * i);
        ext_take<MAX>(__float_as_uint(f.x), c, best, nan_idx);
        ext_take<MAX>(__float_as_uint(f.y), c + 1, best, nan_idx);
        ext_take<MAX>(__float_as_uint(f.z), c + 2, best, nan_idx);
        ext_take<MAX>(__float_as_uint(f.w), c + 3, best, nan_idx);
      }
    } else {
      for (int64_t c = threadIdx.x; c < cols; c += kThreads)
        ext_take<MAX>(__float_as_uint(__ldg(row + c)), (uint32_t)c, best, nan_idx);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t b = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t n = __shfl_xor_sync(0xffffffffu, nan_idx, o);
      best = b > best ? b : best;
      nan_idx = n > nan_idx ? n : nan_idx;
    }
    if ((threadIdx.x & 31) == 0) {
      sbest[threadIdx.x >> 5] = best;
      snan[threadIdx.x >> 5] = nan_idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int i = 1; i < kThreads / 32; ++i) {
        best = sbest[i] > best ? sbest[i] : best;
        nan_idx = snan[i] > nan_idx ? snan[i] : nan_idx;
      }
      best = sbest[0] > best ? sbest[0] : best;
      nan_idx = snan[0] > nan_idx ? snan[0] : nan_idx;
      out[r] = __uint_as_float(ext_result(row, 1, best, nan_idx));
    }
    __syncthreads();
  }
}

// f32 over the outer axis, one thread per column folding the rows in order: Sum/Mean in f64 (the serial order),
// Max/Min by the packed rule.
template <int OP>
__global__ void __launch_bounds__(kThreads) col_f32_kernel(const float* __restrict__ x, int64_t rows, int64_t cols,
                                                            int64_t stride, float* __restrict__ out) {
  const int64_t c = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  if (OP == UP_OP_SUM || OP == UP_OP_MEAN) {
    double acc = 0.0;
    int64_t r = 0;
    for (; r + 3 < rows; r += 4) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldg(x + (r + u) * stride + c);
#pragma unroll
      for (int u = 0; u < 4; ++u) acc += (double)v[u];
    }
    for (; r < rows; ++r) acc += (double)__ldg(x + r * stride + c);
    out[c] = __double2float_rn(OP == UP_OP_MEAN ? acc / (double)rows : acc);
  } else {
    constexpr bool MAX = OP == UP_OP_MAX;
    uint64_t best = 0;
    int64_t nan_idx = -1;
    for (int64_t r = 0; r < rows; ++r) ext_take<MAX>(__float_as_uint(__ldg(x + r * stride + c)), (uint32_t)r, best, nan_idx);
    out[c] = __uint_as_float(ext_result(x + c, stride, best, nan_idx));
  }
}

template <int OP>
int launch_i32(const int32_t* x, int64_t rows, int64_t cols, int64_t stride, int axis, int32_t* out, cudaStream_t s) {
  const int sms = sm_count();
  if (axis == 1) {
    int64_t g = rows < (int64_t)sms * 8 ? rows : (int64_t)sms * 8;
    const bool vec = aligned(x, 16) && cols % 4 == 0 && stride % 4 == 0;
    if (vec) row_fold_i32_kernel<OP, true><<<(int)g, kThreads, 0, s>>>(x, rows, cols, stride, out);
    else row_fold_i32_kernel<OP, false><<<(int)g, kThreads, 0, s>>>(x, rows, cols, stride, out);
    note_launch();
    return check_launch();
  }
  const int64_t gx = (cols + kThreads - 1) / kThreads;
  col_init_i32_kernel<OP><<<(int)(gx < 4096 ? gx : 4096), kThreads, 0, s>>>(out, cols);
  note_launch();
  if (rows == 0) {  // an empty fold stores 0 (1 for Prod): overwrite the identity
    if (OP != UP_OP_PROD) cudaMemsetAsync(out, 0, sizeof(int32_t) * (size_t)cols, s);
    return check_launch();
  }
  int64_t splits = ((int64_t)sms * 4 + gx - 1) / gx;
  const int64_t max_splits = (rows + 63) / 64;
  if (splits > max_splits) splits = max_splits;
  if (splits > 65535) splits = 65535;
  if (splits < 1) splits = 1;
  const int64_t per = (rows + splits - 1) / splits;
  splits = (rows + per - 1) / per;
  col_fold_i32_kernel<OP><<<dim3((unsigned)gx, (unsigned)splits), kThreads, 0, s>>>(x, rows, cols, stride, per, out);
  note_launch();
  return check_launch();
}

}  // namespace r2
}  // namespace up

using namespace up;
using namespace up::r2;

extern "C" int up_sm100_reduce2d_i32(const int32_t* x, int64_t rows, int64_t cols, int64_t row_stride, int axis,
                                     int op, int32_t* out, void* stream) {
  UP_CHECK_ARG(rows >= 0 && cols >= 0 && row_stride >= cols && (axis == 0 || axis == 1));
  UP_CHECK_ARG(out != nullptr || (axis == 1 ? rows : cols) == 0);
  if ((axis == 1 ? rows : cols) == 0) return UP_OK;
  UP_CHECK_ARG(x != nullptr || (axis == 1 ? cols : rows) == 0);
  if (rows > 65535LL * 0x7fffffffLL || cols > 0x7fffffffLL * kThreads) return UP_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (op) {
    case UP_OP_SUM: return launch_i32<UP_OP_SUM>(x, rows, cols, row_stride, axis, out, s);
    case UP_OP_PROD: return launch_i32<UP_OP_PROD>(x, rows, cols, row_stride, axis, out, s);
    case UP_OP_MAX: return launch_i32<UP_OP_MAX>(x, rows, cols, row_stride, axis, out, s);
    case UP_OP_MIN: return launch_i32<UP_OP_MIN>(x, rows, cols, row_stride, axis, out, s);
    case UP_OP_AND: return launch_i32<UP_OP_AND>(x, rows, cols, row_stride, axis, out, s);
    case UP_OP_OR: return launch_i32<UP_OP_OR>(x, rows, cols, row_stride, axis, out, s);
    case UP_OP_XOR: return launch_i32<UP_OP_XOR>(x, rows, cols, row_stride, axis, out, s);
    default: return UP_ERR_UNSUPPORTED;
  }
}

extern "C" int up_sm100_reduce2d_f32(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int axis, int op,
                                     int accum, int block, float* out, void* stream) {
  UP_CHECK_ARG(rows >= 0 && cols >= 0 && row_stride >= cols && (axis == 0 || axis == 1));
  if (op != UP_OP_SUM && op != UP_OP_MEAN && op != UP_OP_MAX && op != UP_OP_MIN) return UP_ERR_UNSUPPORTED;
  UP_CHECK_ARG(out != nullptr || (axis == 1 ? rows : cols) == 0);
  if ((axis == 1 ? rows : cols) == 0) return UP_OK;
  UP_CHECK_ARG(x != nullptr || (axis == 1 ? cols : rows) == 0);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (axis == 1) {
    if (op == UP_OP_SUM) return up_sm100_row_sum_f32(x, rows, cols, row_stride, out, accum, block, stream);
    if (op == UP_OP_MEAN) {
      // the documented f64 order of the Auto row sum, divided by the extent before the one rounding
      if (accum != UP_ACCUM_AUTO) return fail_with(UP_ERR_UNSUPPORTED, "reduce2d_f32: Mean is lowered for Auto");
      return row_mean_f32_auto(x, rows, cols, row_stride, block, out, stream);
    }
    if (cols > 0xfffffffeLL) return UP_ERR_UNSUPPORTED;  // indices are packed in 32 bits
    const int g = (int)(rows < (int64_t)sm_count() * 8 ? rows : (int64_t)sm_count() * 8);
    const bool vec = aligned(x, 16) && cols % 4 == 0 && row_stride % 4 == 0;
    if (op == UP_OP_MAX) {
      if (vec) row_extremum_f32_kernel<true, true><<<g, kThreads, 0, s>>>(x, rows, cols, row_stride, out);
      else row_extremum_f32_kernel<true, false><<<g, kThreads, 0, s>>>(x, rows, cols, row_stride, out);
    } else {
      if (vec) row_extremum_f32_kernel<false, true><<<g, kThreads, 0, s>>>(x, rows, cols, row_stride, out);
      else row_extremum_f32_kernel<false, false><<<g, kThreads, 0, s>>>(x, rows, cols, row_stride, out);
    }
    note_launch();
    return check_launch();
  }
  // axis 0: the serial order per column (Sum/Mean), so the accumulation policy must be Auto
  if ((op == UP_OP_SUM || op == UP_OP_MEAN) && accum != UP_ACCUM_AUTO)
    return fail_with(UP_ERR_UNSUPPORTED, "reduce2d_f32: an outer-axis Sum/Mean is lowered for Auto");
  if (rows > 0xfffffffeLL) return UP_ERR_UNSUPPORTED;
  const int64_t gx = (cols + kThreads - 1) / kThreads;
  if (gx > 0x7fffffff) return UP_ERR_UNSUPPORTED;
  switch (op) {
    case UP_OP_SUM: col_f32_kernel<UP_OP_SUM><<<(int)gx, kThreads, 0, s>>>(x, rows, cols, row_stride, out); break;
    case UP_OP_MEAN: col_f32_kernel<UP_OP_MEAN><<<(int)gx, kThreads, 0, s>>>(x, rows, cols, row_stride, out); break;
    case UP_OP_MAX: col_f32_kernel<UP_OP_MAX><<<(int)gx, kThreads, 0, s>>>(x, rows, cols, row_stride, out); break;
    default: col_f32_kernel<UP_OP_MIN><<<(int)gx, kThreads, 0, s>>>(x, rows, cols, row_stride, out); break;
  }
  note_launch();
  return check_launch();
}
