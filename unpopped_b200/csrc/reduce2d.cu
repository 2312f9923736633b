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
//    element of the extreme value (so the first zero's sign when +0 and -0 tie). The kernels keep the best value
//    with its first index and the last NaN's index; merging those by value (ties to the lower index) is
//    order-independent.
//  * f32 Sum/Mean over the outer axis fold each column in the serial order in f64, one rounding (the kernels add
//    runs of values out of order only where no add of the serial fold can round); Mean divides by the row count,
//    so an empty Mean is 0/0.
#include "common.cuh"
#include "spec.cuh"

#include <cooperative_groups.h>
#include <mutex>

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
  if (VEC && cols / 4 <= 8 * kThreads) {
    // rows of at most 8 int4 per thread: the next row's loads are issued before this row is folded
    const int64_t nv = cols / 4;
    uint4 f[8];
    auto load = [&](int64_t rr) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t i = threadIdx.x + (int64_t)u * kThreads;
        if (rr < rows && i < nv) f[u] = ld_nc_na_v4(x + rr * stride + 4 * i);
      }
    };
    int64_t r = blockIdx.x;
    load(r);
    for (; r < rows; r += gridDim.x) {
      uint4 cur[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) cur[u] = f[u];
      load(r + gridDim.x);
      int32_t acc = ident<OP>();
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (threadIdx.x + (int64_t)u * kThreads < nv) acc = comb4<OP>(acc, cur[u]);
      acc = block_comb<OP>(acc, part);
      if (threadIdx.x == 0) out[r] = cols > 0 ? acc : (OP == UP_OP_PROD ? 1 : 0);
    }
    return;
  }
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
__global__ void col_init_i32_kernel(int32_t* __restrict__ out, int64_t cols, int64_t ob) {
  out += (int64_t)blockIdx.z * ob;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += (int64_t)gridDim.x * blockDim.x)
    out[c] = ident<OP>();
}

// A split's partial into out[c] with the op's atomic.
template <int OP>
__device__ __forceinline__ void col_combine_out(int32_t* o, int32_t acc) {
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

template <int OP>
__global__ void __launch_bounds__(kThreads) col_fold_i32_kernel(const int32_t* __restrict__ x, int64_t rows,
                                                                 int64_t cols, int64_t stride, int64_t per_split,
                                                                 int32_t* __restrict__ out, int64_t xb, int64_t ob) {
  x += (int64_t)blockIdx.z * xb;  // batch z of a middle-axis reduction
  out += (int64_t)blockIdx.z * ob;
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
  col_combine_out<OP>(out + c, acc);
}

// ---- f32 Max/Min ----
// The fold's state: the best value so far with its first index (idx = kNone: no non-NaN element yet) and the last
// NaN's index. A thread takes its elements in ascending index order and replaces only on a strictly better value,
// so it keeps the first of equal values (and of +0/-0). The value is the element itself, bits and all, so the
// result needs no re-read unless it is a NaN. Two states combine by value, ties to the lower index.
constexpr uint32_t kNone = 0xffffffffu;

template <bool MAX>
struct ExtState {
  float m;
  uint32_t idx;
  int32_t nan_idx;
  __device__ __forceinline__ void init() {
    m = MAX ? -__int_as_float(0x7f800000) : __int_as_float(0x7f800000);
    idx = kNone;
    nan_idx = -1;
  }
  __device__ __forceinline__ void take(float v, uint32_t i) {  // i ascending within a thread
    const bool is_nan = v != v;
    const bool take_v = !is_nan && ((MAX ? v > m : v < m) || idx == kNone);
    m = take_v ? v : m;
    idx = take_v ? i : idx;
    nan_idx = is_nan ? (int32_t)i : nan_idx;
  }
  __device__ __forceinline__ void merge(float om, uint32_t oidx, int32_t onan) {
    nan_idx = onan > nan_idx ? onan : nan_idx;
    if (oidx == kNone) return;
    const bool better = idx == kNone || (MAX ? om > m : om < m) || (om == m && oidx < idx);
    m = better ? om : m;
    idx = better ? oidx : idx;
  }
  __device__ __forceinline__ void warp_merge() {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
      const int32_t on = __shfl_xor_sync(0xffffffffu, nan_idx, o);
      merge(om, oi, on);
    }
  }
  // the result's bits: the last NaN (quiet bit set), else the best element, else 0 (empty)
  __device__ __forceinline__ uint32_t result(const float* base, int64_t step) const {
    if (nan_idx >= 0) return __float_as_uint(base[(int64_t)nan_idx * step]) | 0x00400000u;
    return idx == kNone ? 0u : __float_as_uint(m);
  }
};

// max.NaN / min.NaN: the larger (smaller) operand, NaN if either is NaN, so one tree over a chunk both finds the
// chunk's extreme value and shows whether the chunk holds a NaN.
template <bool MAX>
__device__ __forceinline__ float pick_nan(float a, float b) {
  float d;
  if (MAX)
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  else
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// Folds U float4s (elements base[u] .. base[u] + 3, ascending in u; ok[u] false for a float4 outside the row) into
// the state in index order, with the serial rule's result: the chunk's extreme value is found by one max.NaN tree;
// a chunk with a NaN takes the serial path element by element; otherwise the state changes only when the chunk's
// value is strictly better (or the state is empty), and then to the chunk's first element equal to it, so the first
// of equal values (and of +0/-0) is kept. About 1.1 operations per element instead of the serial rule's seven.
template <bool MAX, int U>
__device__ __forceinline__ void fold_chunk(ExtState<MAX>& st, const float4 (&f)[U], const uint32_t (&base)[U],
                                           const bool (&ok)[U]) {
  const float fill = MAX ? -__int_as_float(0x7f800000) : __int_as_float(0x7f800000);
  float q[U];
#pragma unroll
  for (int u = 0; u < U; ++u)
    q[u] = ok[u] ? pick_nan<MAX>(pick_nan<MAX>(f[u].x, f[u].y), pick_nan<MAX>(f[u].z, f[u].w)) : fill;
#pragma unroll
  for (int h = 1; h < U; h <<= 1)
#pragma unroll
    for (int u = 0; u + h < U; u += 2 * h) q[u] = pick_nan<MAX>(q[u], q[u + h]);
  const float cm = q[0];
  if (cm != cm) {
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (ok[u]) {
        st.take(f[u].x, base[u]);
        st.take(f[u].y, base[u] + 1);
        st.take(f[u].z, base[u] + 2);
        st.take(f[u].w, base[u] + 3);
      }
  } else if (st.idx == kNone || (MAX ? cm > st.m : cm < st.m)) {
    bool found = false;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float4 c = f[u];
      if (!found && ok[u] && (c.x == cm || c.y == cm || c.z == cm || c.w == cm)) {
        found = true;
        st.idx = c.x == cm ? base[u] : c.y == cm ? base[u] + 1 : c.z == cm ? base[u] + 2 : base[u] + 3;
        st.m = c.x == cm ? c.x : c.y == cm ? c.y : c.z == cm ? c.z : c.w;
      }
    }
  }
}

// An order-preserving integer key of a non-NaN float, with +0 and -0 equal (ties between them go to the lower
// index, as equal values do).
__device__ __forceinline__ int32_t ext_key(float m) {
  const int32_t b = m == 0.0f ? 0 : __float_as_int(m);
  return b >= 0 ? b : (b ^ 0x7fffffff);
}

// Merges the 32 lanes' states into every lane with the warp's integer reductions: the best key, the lowest index
// holding it, the last NaN; the value's bits come from the lane that holds the winning index.
template <bool MAX>
__device__ __forceinline__ void warp_reduce_ext(ExtState<MAX>& st) {
  const int32_t none = MAX ? (int32_t)0x80000000 : 0x7fffffff;
  const int32_t k = st.idx == kNone ? none : ext_key(st.m);
  const int32_t wk = MAX ? __reduce_max_sync(0xffffffffu, k) : __reduce_min_sync(0xffffffffu, k);
  const uint32_t wi = __reduce_min_sync(0xffffffffu, (st.idx != kNone && k == wk) ? st.idx : kNone);
  const unsigned own = __ballot_sync(0xffffffffu, wi != kNone && st.idx == wi);
  const float wm = __shfl_sync(0xffffffffu, st.m, own ? __ffs(own) - 1 : 0);
  st.nan_idx = __reduce_max_sync(0xffffffffu, st.nan_idx);
  st.m = wm;
  st.idx = wi;
}

// f32 Max/Min over the last axis, a CTA per row (grid-stride). Rows of at most 8 float4 per thread keep the whole
// share in registers and issue the next row's loads before folding this one; longer rows fold 4 float4 per step.
// The block merge is one barrier per row: the warps' states go to a double-buffered slot and warp 0 merges them.
template <bool MAX, bool VEC>
__global__ void __launch_bounds__(kThreads) row_extremum_f32_kernel(const float* __restrict__ x, int64_t rows,
                                                                     int64_t cols, int64_t stride,
                                                                     float* __restrict__ out) {
  constexpr int kW = kThreads / 32;
  __shared__ float sm[2][kW];
  __shared__ uint32_t si[2][kW];
  __shared__ int32_t sn[2][kW];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int par = 0;
  // the warp-merged state of this row to the slot; warp 0 merges the slots and writes the result
  auto finish = [&](ExtState<MAX>& st, int64_t r) {
    warp_reduce_ext<MAX>(st);
    if (lane == 0) {
      sm[par][w] = st.m;
      si[par][w] = st.idx;
      sn[par][w] = st.nan_idx;
    }
    __syncthreads();
    if (w == 0) {
      ExtState<MAX> b;
      b.init();
      if (lane < kW) {
        b.m = sm[par][lane];
        b.idx = si[par][lane];
        b.nan_idx = sn[par][lane];
      }
      warp_reduce_ext<MAX>(b);
      if (lane == 0) out[r] = __uint_as_float(b.result(x + r * stride, 1));
    }
    par ^= 1;  // the next row writes the other slot; this one is read before the next row's barrier
  };
  if (VEC && cols / 4 <= 8 * kThreads) {
    const int64_t nv = cols / 4;
    uint32_t base[8];
    bool ok[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t i = threadIdx.x + (int64_t)u * kThreads;
      ok[u] = i < nv;
      base[u] = (uint32_t)(4 * i);
    }
    float4 f[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) f[u] = make_float4(0.f, 0.f, 0.f, 0.f);  // a float4 outside the row is never folded
    auto load = [&](int64_t rr) {
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (rr < rows && ok[u]) f[u] = ld_nc_na_f4(x + rr * stride + base[u]);
    };
    int64_t r = blockIdx.x;
    load(r);
    for (; r < rows; r += gridDim.x) {
      float4 cur[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) cur[u] = f[u];
      load(r + gridDim.x);
      ExtState<MAX> st;
      st.init();
      fold_chunk<MAX, 8>(st, cur, base, ok);
      finish(st, r);
    }
    return;
  }
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* row = x + r * stride;
    ExtState<MAX> st;
    st.init();
    if (VEC) {
      const int64_t nv = cols / 4;
      for (int64_t i = threadIdx.x; i < nv; i += 4 * kThreads) {
        float4 f[4];
        uint32_t base[4];
        bool ok[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t j = i + (int64_t)u * kThreads;
          ok[u] = j < nv;
          base[u] = (uint32_t)(4 * j);
          f[u] = ok[u] ? ld_nc_na_f4(row + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        fold_chunk<MAX, 4>(st, f, base, ok);
      }
    } else {
      for (int64_t c = threadIdx.x; c < cols; c += kThreads) st.take(__ldg(row + c), (uint32_t)c);
    }
    finish(st, r);
  }
}

// f32 Max/Min over the outer axis: a CTA takes 32 columns (one per lane, coalesced across the row) and its 16 warps
// split the rows (warp w folds rows w, w + 16, ... in order); the 16 partials of a column merge by value.
constexpr int kColWarps = 16;
template <bool MAX>
__global__ void __launch_bounds__(32 * kColWarps) col_extremum_f32_kernel(const float* __restrict__ x, int64_t rows,
                                                                          int64_t cols, int64_t stride,
                                                                          float* __restrict__ out, int64_t xb, int64_t ob) {
  x += (int64_t)blockIdx.z * xb;  // batch z of a middle-axis reduction
  out += (int64_t)blockIdx.z * ob;
  __shared__ float sm[kColWarps][32];
  __shared__ uint32_t si[kColWarps][32];
  __shared__ int32_t sn[kColWarps][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  ExtState<MAX> st;
  st.init();
  if (c < cols) {
    int64_t r = w;
    for (; r + 3 * kColWarps < rows; r += 4 * kColWarps) {
      float v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = __ldg(x + (r + k * kColWarps) * stride + c);
#pragma unroll
      for (int k = 0; k < 4; ++k) st.take(v[k], (uint32_t)(r + k * kColWarps));
    }
    for (; r < rows; r += kColWarps) st.take(__ldg(x + r * stride + c), (uint32_t)r);
  }
  sm[w][lane] = st.m;
  si[w][lane] = st.idx;
  sn[w][lane] = st.nan_idx;
  __syncthreads();
  if (w == 0 && c < cols) {
    for (int k = 1; k < kColWarps; ++k) st.merge(sm[k][lane], si[k][lane], sn[k][lane]);
    out[c] = __uint_as_float(st.result(x + c, stride));
  }
}

// f32 Max/Min over the outer axis, 16-byte loads: a CTA takes a strip of 128 columns (a float4 per lane, 512 B of
// each row per warp) and a cluster of 8 CTAs splits the rows into 8 ranges; warp w of a CTA folds rows w, w + 8, ...
// of its range in order. Each lane folds a batch of 4 rows per column with one max.NaN tree and searches the batch
// only when its value is strictly better (the serial rule as in fold_chunk). The 8 warps merge through shared
// memory and the cluster's 8 CTAs through distributed shared memory into rank 0, which writes the strip.
constexpr int kColStrip = 128, kColCluster = 8, kColVecWarps = 8;
template <bool MAX>
__device__ __forceinline__ void fold_col_batch(ExtState<MAX>& st, float a0, float a1, float a2, float a3,
                                               uint32_t r, uint32_t step) {
  const float cm = pick_nan<MAX>(pick_nan<MAX>(a0, a1), pick_nan<MAX>(a2, a3));
  if (cm != cm) {
    st.take(a0, r);
    st.take(a1, r + step);
    st.take(a2, r + 2 * step);
    st.take(a3, r + 3 * step);
  } else if (st.idx == kNone || (MAX ? cm > st.m : cm < st.m)) {
    st.idx = a0 == cm ? r : a1 == cm ? r + step : a2 == cm ? r + 2 * step : r + 3 * step;
    st.m = a0 == cm ? a0 : a1 == cm ? a1 : a2 == cm ? a2 : a3;
  }
}

template <bool MAX>
__global__ void __cluster_dims__(1, kColCluster, 1) __launch_bounds__(32 * kColVecWarps)
    col_extremum_f32_vec_kernel(const float* __restrict__ x, int64_t rows, int64_t cols, int64_t stride,
                                float* __restrict__ out, int64_t xb, int64_t ob) {
  x += (int64_t)blockIdx.z * xb;  // batch z of a middle-axis reduction
  out += (int64_t)blockIdx.z * ob;
  namespace cg = cooperative_groups;
  __shared__ float sm[kColVecWarps][kColStrip];
  __shared__ uint32_t si[kColVecWarps][kColStrip];
  __shared__ int32_t sn[kColVecWarps][kColStrip];
  __shared__ float cm_[kColStrip];
  __shared__ uint32_t ci_[kColStrip];
  __shared__ int32_t cn_[kColStrip];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c0 = (int64_t)blockIdx.x * kColStrip + 4 * lane;
  const int64_t per = (rows + kColCluster - 1) / kColCluster;
  const int64_t r0 = (int64_t)blockIdx.y * per;
  const int64_t r1 = r0 + per < rows ? r0 + per : rows;
  ExtState<MAX> st[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) st[j].init();
  if (c0 < cols) {
    const float* base = x + c0;
    int64_t r = r0 + w;
    constexpr int S = kColVecWarps;
    for (; r + 7 * S < r1; r += 8 * S) {  // eight rows in flight, folded as two batches in row order
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = ld_nc_na_f4(base + (r + u * S) * stride);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t rh = (uint32_t)(r + 4 * h * S);
        fold_col_batch<MAX>(st[0], v[4 * h].x, v[4 * h + 1].x, v[4 * h + 2].x, v[4 * h + 3].x, rh, S);
        fold_col_batch<MAX>(st[1], v[4 * h].y, v[4 * h + 1].y, v[4 * h + 2].y, v[4 * h + 3].y, rh, S);
        fold_col_batch<MAX>(st[2], v[4 * h].z, v[4 * h + 1].z, v[4 * h + 2].z, v[4 * h + 3].z, rh, S);
        fold_col_batch<MAX>(st[3], v[4 * h].w, v[4 * h + 1].w, v[4 * h + 2].w, v[4 * h + 3].w, rh, S);
      }
    }
    for (; r + 3 * S < r1; r += 4 * S) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = ld_nc_na_f4(base + (r + u * S) * stride);
      fold_col_batch<MAX>(st[0], v[0].x, v[1].x, v[2].x, v[3].x, (uint32_t)r, S);
      fold_col_batch<MAX>(st[1], v[0].y, v[1].y, v[2].y, v[3].y, (uint32_t)r, S);
      fold_col_batch<MAX>(st[2], v[0].z, v[1].z, v[2].z, v[3].z, (uint32_t)r, S);
      fold_col_batch<MAX>(st[3], v[0].w, v[1].w, v[2].w, v[3].w, (uint32_t)r, S);
    }
    for (; r < r1; r += S) {
      const float4 v = ld_nc_na_f4(base + r * stride);
      st[0].take(v.x, (uint32_t)r);
      st[1].take(v.y, (uint32_t)r);
      st[2].take(v.z, (uint32_t)r);
      st[3].take(v.w, (uint32_t)r);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sm[w][4 * lane + j] = st[j].m;
    si[w][4 * lane + j] = st[j].idx;
    sn[w][4 * lane + j] = st[j].nan_idx;
  }
  __syncthreads();
  const int t = threadIdx.x;  // the strip's column t (threads 0 .. 127)
  if (t < kColStrip) {
    ExtState<MAX> a;
    a.m = sm[0][t];
    a.idx = si[0][t];
    a.nan_idx = sn[0][t];
    for (int k = 1; k < kColVecWarps; ++k) a.merge(sm[k][t], si[k][t], sn[k][t]);
    cm_[t] = a.m;
    ci_[t] = a.idx;
    cn_[t] = a.nan_idx;
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();  // every CTA's strip states are visible to rank 0
  if (cluster.block_rank() == 0 && t < kColStrip) {
    ExtState<MAX> a;
    a.m = cm_[t];
    a.idx = ci_[t];
    a.nan_idx = cn_[t];
    for (unsigned q = 1; q < (unsigned)kColCluster; ++q)
      a.merge(*cluster.map_shared_rank(&cm_[t], q), *cluster.map_shared_rank(&ci_[t], q),
              *cluster.map_shared_rank(&cn_[t], q));
    const int64_t c = (int64_t)blockIdx.x * kColStrip + t;
    if (c < cols) out[c] = __uint_as_float(a.result(x + c, stride));
  }
  cluster.sync();  // rank 0 has read the other CTAs' shared memory before they exit
}

// f32 Sum/Mean over the outer axis in the serial order per column: s = (((0 + x0) + x1) + ...) in f64, one rounding
// to f32 (plan_eval.rs:566-645). Folded directly, each column is a chain of 8,192 dependent f64 adds with the
// loads in front of them. The kernels below get the same bits with a short chain:
//  * Exactness. Every f32 is an integer multiple of its ulp, 2^(max(e,1) - 150) for exponent field e. If all the
//    values added since the last inexact step are multiples of 2^q, so is every partial sum, and a partial sum
//    below 2^(q+53) in magnitude is a multiple of 2^q with at most 53 significant bits: representable, so the add
//    that made it did not round. While no add rounds, the serial fold is the exact sum, and any order of adding a
//    run of values gives the same bits.
//  * Chunks. Producer warps read each column in chunks of 64 rows and summarise a chunk in three numbers: L =
//    2^(q + 53) for q the smallest ulp exponent of its nonzero values; T, its prefix sum in f64 in row order; and
//    H, the largest magnitude of those prefix sums, rounded up to f32. If H < L, no add of the prefix rounded (the
//    first that did would have made a partial sum of magnitude at least L, since L is a power of two and rounding
//    is monotone), so T and H are exact. Otherwise, or if T is a NaN or infinite, H is +inf.
//  * The chain walks a column's chunks in order with the running sum s and lim, the minimum of the L seen since the
//    last anchor. The serial fold's partial sums inside a chunk are s + (a prefix), at most |s| + H in magnitude,
//    so if |s| + H < lim each is a multiple of 2^q below 2^(q+53): the chunk adds no rounding, and s + T is
//    exact. Otherwise the chunk is re-read and folded value by
//    value in f64, as the serial fold does; s then anchors lim at 2^(lowbit(s) + 53), lowbit(s) the place of its
//    lowest set bit. A NaN or infinite s fails the comparison, so the rest of such a column takes the serial fold
//    too (NaN payloads propagate as they do there).
// On N(0,1) data about 0.002 % of chunks take the serial fold and on U[0,1) about 0.04 %; on data whose exponents
// spread over 30 binades or more nearly all do, and the kernels then run at about the speed of the plain fold.
// The serial fold of chunk rows [r0, r0 + 64) for every lane of the warp with `slow` set (chunks that may round),
// and the anchor after it. The whole warp loads each such column's chunk, two rows a lane, so its 64 loads are in
// flight together, and passes the values to the owning lane in row order. col_of(f) is lane f's column base. Every
// lane of the warp calls this with the same r0.
template <class ColOf>
__device__ __forceinline__ void spec_serial_chunks_warp(bool slow, ColOf col_of, int64_t r0, int64_t rows,
                                                        int64_t stride, double& s, double& lim) {
  const int lane = threadIdx.x & 31;
  unsigned m = __ballot_sync(0xffffffffu, slow);
  while (m) {
    const int f = __ffs(m) - 1;
    m &= m - 1;
    const float* __restrict__ xc = col_of(f);
    const float a = r0 + lane < rows ? __ldg(xc + (r0 + lane) * stride) : 0.f;
    const float b = r0 + 32 + lane < rows ? __ldg(xc + (r0 + 32 + lane) * stride) : 0.f;
    double acc = s;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const float v = __shfl_sync(0xffffffffu, a, k);
      if (r0 + k < rows) acc += (double)v;
    }
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const float v = __shfl_sync(0xffffffffu, b, k);
      if (r0 + 32 + k < rows) acc += (double)v;
    }
    if (lane == f) {
      s = acc;
      lim = spec_anchor(acc);
    }
  }
}

// The form for any row alignment: a CTA takes 32 columns (lane l: column 32·blockIdx.x + l); warps 1..8 summarise
// segments of 16 chunks, warp 0 walks them, and a segment's summaries are double-buffered in shared memory so the
// chain walks segment i - 1 while the producers summarise segment i. The chain adds a segment's chunks
// speculatively and checks all of them beside it; a lane with a failed check goes back to the segment's start.
constexpr int kSpecSeg = 16, kSpecProducers = 8;

template <bool MEAN>
__global__ void __launch_bounds__(32 * (kSpecProducers + 1), 2)
    col_sum_f32_serial_spec_kernel(const float* __restrict__ x, int64_t rows, int64_t cols, int64_t stride,
                                   float* __restrict__ out, int64_t xb, int64_t ob) {
  x += (int64_t)blockIdx.z * xb;  // batch z of a middle-axis reduction
  out += (int64_t)blockIdx.z * ob;
  __shared__ double s_t[2][kSpecSeg][32], s_l[2][kSpecSeg][32];
  __shared__ float s_h[2][kSpecSeg][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.x * 32 + lane;
  const bool cok = col < cols;
  const float* __restrict__ xc = x + (cok ? col : 0);
  const int64_t nseg = (rows + kSpecChunk * kSpecSeg - 1) / (kSpecChunk * kSpecSeg);
  double s = 0.0, lim = f64_inf();  // the chain's state (warp 0)
  for (int64_t i = 0; i <= nseg; ++i) {
    if (warp > 0) {
      if (i < nseg) {
        const int bb = (int)(i & 1);
        for (int j = warp - 1; j < kSpecSeg; j += kSpecProducers) {
          const int64_t r0 = (i * kSpecSeg + j) * kSpecChunk;
          float v[kSpecChunk];
          if (cok && r0 + kSpecChunk <= rows) {
#pragma unroll
            for (int k = 0; k < kSpecChunk; ++k) v[k] = __ldg(xc + (r0 + k) * stride);
          } else {
#pragma unroll
            for (int k = 0; k < kSpecChunk; ++k) v[k] = (cok && r0 + k < rows) ? __ldg(xc + (r0 + k) * stride) : 0.f;
          }
          double pre = 0.0, hi = 0.0;
          uint32_t mn = 0xffffffffu;
#pragma unroll
          for (int k = 0; k < kSpecChunk; ++k) spec_acc(v[k], pre, hi, mn);
          double lc;
          float h;
          spec_finish(pre, hi, mn, lc, h);
          s_t[bb][j][lane] = pre;
          s_l[bb][j][lane] = lc;
          s_h[bb][j][lane] = h;
        }
      }
    } else if (i > 0) {
      const int bb = (int)((i - 1) & 1);
      const double s0 = s, l0 = lim;
      bool ok = true;
#pragma unroll
      for (int j = 0; j < kSpecSeg; ++j) {
        lim = fmin(lim, s_l[bb][j][lane]);
        ok &= fabs(s) + (double)s_h[bb][j][lane] < lim;
        s += s_t[bb][j][lane];
      }
      if (__any_sync(0xffffffffu, !ok)) {  // the lanes with a failed check walk the segment again
        if (!ok) {
          s = s0;
          lim = l0;
        }
        const float* xb0 = x + (int64_t)blockIdx.x * 32;
        for (int j = 0; j < kSpecSeg; ++j) {
          bool slow = false;
          if (!ok) {
            lim = fmin(lim, s_l[bb][j][lane]);
            if (fabs(s) + (double)s_h[bb][j][lane] < lim)
              s += s_t[bb][j][lane];
            else
              slow = true;
          }
          spec_serial_chunks_warp(slow, [&](int f) { return xb0 + f; }, ((i - 1) * kSpecSeg + j) * kSpecChunk, rows,
                                  stride, s, lim);
        }
      }
    }
    __syncthreads();  // segment i is summarised and segment i - 1 walked before either buffer is reused
  }
  if (warp == 0 && cok) out[col] = __double2float_rn(MEAN ? s / (double)rows : s);
}

// The form for 16-byte aligned rows whose width is a multiple of 4, which reads 512 bytes of a row per warp (a float4
// per lane): a CTA takes a strip of 128 columns and a cluster of kStripCluster CTAs splits the rows. Chunks go in
// rounds of kStripCluster · kStripCap; in each round rank k summarises its share of the round's chunks into shared
// memory (all 8 warps, a lane's 4 columns at once). Then, one column per lane of warps 0..3:
//  1. each rank adds its own chunks' T in order (SL) and takes the minimum of their L (ML), the largest |partial
//     sum| of SL (MX) and the largest H (HM);
//  2. rank k starts from the round's carry plus SL of ranks 0..k-1 (read through distributed shared memory), with
//     lim the minimum of the carry's and their ML. From a start s, every partial sum of the serial fold over the
//     rank's rows is at most |s| + MX + HM in magnitude (the partial sums at chunk starts are s + a partial sum of
//     SL), so if that bound (taken with upward-rounded adds) is below min(lim, ML), no add of the rank's rows
//     rounds and s + SL is exact: one test for the whole rank. Otherwise the rank walks its chunks with the checks;
//  3. if every rank's test held and every SL used was exact, each start was the serial fold's own, and
//     rank kStripCluster-1's result is the next carry. Otherwise the ranks go in order: rank k takes the carry from
//     rank k-1 and keeps its own result if its speculative start equals that carry bit for bit; else it tries the
//     one test from the carry, and only then walks from the carry (re-reading any chunk that may round).
constexpr int kStripCols = 128, kStripCluster = 4, kStripCap = 32, kStripWarps = 8, kStripSub = 16;
constexpr int kStripSmem = kStripCap * kStripCols * (8 + 8 + 4) + 4 * kStripCols * 8 + 16;

template <bool MEAN>
__global__ void __cluster_dims__(1, kStripCluster, 1) __launch_bounds__(32 * kStripWarps, 2)
    col_sum_f32_serial_strip_kernel(const float* __restrict__ x, int64_t rows, int64_t cols, int64_t stride,
                                    float* __restrict__ out, int64_t xb, int64_t ob) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  x += (int64_t)blockIdx.z * xb;  // batch z of a middle-axis reduction
  out += (int64_t)blockIdx.z * ob;
  extern __shared__ __align__(16) unsigned char strip_smem[];
  double* s_t = reinterpret_cast<double*>(strip_smem);  // [kStripCap][128] chunk sums T
  double* s_l = s_t + kStripCap * kStripCols;            // [kStripCap][128] chunk limits L
  double* s_carry = s_l + kStripCap * kStripCols;        // [2][128]: s and lim handed to this rank
  double* s_part = s_carry + 2 * kStripCols;             // [2][128]: this rank's SL and ML
  float* s_h = reinterpret_cast<float*>(s_part + 2 * kStripCols);  // [kStripCap][128] prefix bounds H
  int* s_fail = reinterpret_cast<int*>(s_h + kStripCap * kStripCols);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c0 = (int64_t)blockIdx.x * kStripCols;
  const bool pok = c0 + 4 * lane < cols;  // a producer lane's 4 columns (cols is a multiple of 4)
  const int ccol = 32 * warp + lane;      // a chain lane's column (warps 0..3)
  const bool cok = warp < 4 && c0 + ccol < cols;
  if (threadIdx.x < kStripCols) {
    s_carry[threadIdx.x] = 0.0;
    s_carry[kStripCols + threadIdx.x] = f64_inf();
  }
  cluster.sync();  // every CTA of the cluster runs and holds its initial carry before any hand-off
  const float* __restrict__ xp = x + c0 + 4 * lane;
  const int64_t nchunks = (rows + kSpecChunk - 1) / kSpecChunk;
  const int64_t per_round = (int64_t)kStripCluster * kStripCap;
  for (int64_t g0 = 0; g0 < nchunks; g0 += per_round) {
    const int64_t nch = min(per_round, nchunks - g0);
    const int64_t share = (nch + kStripCluster - 1) / kStripCluster;
    const int64_t mb = g0 + min(nch, (int64_t)rank * share);  // this rank's first chunk
    const int me = (int)(g0 + min(nch, (int64_t)(rank + 1) * share) - mb);
    for (int j = warp; j < me; j += kStripWarps) {
      const int64_t r0 = (mb + j) * kSpecChunk;
      double pre[4] = {0.0, 0.0, 0.0, 0.0}, hi[4] = {0.0, 0.0, 0.0, 0.0};
      uint32_t mn[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
      for (int sb = 0; sb < kSpecChunk; sb += kStripSub) {
        float4 v[kStripSub];
        const bool full = pok && r0 + sb + kStripSub <= rows;
#pragma unroll
        for (int k = 0; k < kStripSub; ++k) {
          const int64_t r = r0 + sb + k;
          v[k] = (full || (pok && r < rows)) ? ld_nc_na_f4(xp + r * stride) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < kStripSub; ++k) {
          spec_acc(v[k].x, pre[0], hi[0], mn[0]);
          spec_acc(v[k].y, pre[1], hi[1], mn[1]);
          spec_acc(v[k].z, pre[2], hi[2], mn[2]);
          spec_acc(v[k].w, pre[3], hi[3], mn[3]);
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int at = j * kStripCols + 4 * lane + c;
        double lc;
        float h;
        spec_finish(pre[c], hi[c], mn[c], lc, h);
        s_t[at] = pre[c];
        s_l[at] = lc;
        s_h[at] = h;
      }
    }
    __syncthreads();
    // 1. this rank's SL and ML
    double si = 0.0, li = 0.0, so = 0.0, lo = 0.0;  // the speculative start and result
    double sl = 0.0, ml = f64_inf(), mx = 0.0, hm = 0.0;
    bool exact = true, wok = true;                  // SL exact (or unused); the rank's test or walk held
    if (cok) {
      float h = 0.f;
#pragma unroll 4
      for (int j = 0; j < me; ++j) {
        ml = fmin(ml, s_l[j * kStripCols + ccol]);
        h = fmaxf(h, s_h[j * kStripCols + ccol]);
        sl += s_t[j * kStripCols + ccol];
        mx = fmax(mx, fabs(sl));
      }
      hm = (double)h;
      s_part[ccol] = sl;
      s_part[kStripCols + ccol] = ml;
      exact = rank == kStripCluster - 1 || mx < ml;  // SL is used by later ranks only
    }
    // the whole rank from start s without a rounding add (see 2. above)
    auto rank_exact = [&](double s, double lim) {
      return __dadd_ru(__dadd_ru(fabs(s), mx), hm) < fmin(lim, ml);
    };
    // The chunk-by-chunk walk from (s, lim) for lanes with `act`, 8 chunks at a time without branches; with FOLD,
    // a block with a failed check is walked again chunk by chunk and folds the chunks that may round. Every lane of
    // the warp calls it. Returns whether every check held.
    auto walk = [&](double& s, double& lim, bool act, bool fold) {
      bool good = true;
      const float* xw = x + c0 + 32 * warp;
      for (int j0 = 0; j0 < me; j0 += 8) {
        double s1 = s, l1 = lim;
        bool okb = true;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (j0 + u < me) {
            const int at = (j0 + u) * kStripCols + ccol;
            l1 = fmin(l1, s_l[at]);
            okb &= fabs(s1) + (double)s_h[at] < l1;
            s1 += s_t[at];
          }
        }
        if (act && (okb || !fold)) {
          s = s1;
          lim = l1;
        }
        good &= okb;
        const bool redo = fold && act && !okb;
        if (__any_sync(0xffffffffu, redo)) {
          for (int u = 0; u < 8 && j0 + u < me; ++u) {
            bool slow = false;
            if (redo) {
              const int at = (j0 + u) * kStripCols + ccol;
              lim = fmin(lim, s_l[at]);
              if (fabs(s) + (double)s_h[at] < lim)
                s += s_t[at];
              else
                slow = true;
            }
            spec_serial_chunks_warp(slow, [&](int f) { return xw + f; }, (mb + j0 + u) * kSpecChunk, rows, stride, s,
                                    lim);
          }
        }
      }
      return good;
    };
    cluster.sync();
    // 2. the speculative start and the checked walk
    if (cok) {
      const double* c0r = cluster.map_shared_rank(s_carry, 0);
      double s = c0r[ccol], lim = c0r[kStripCols + ccol];
      for (int q = 0; q < rank; ++q) {
        const double* pr = cluster.map_shared_rank(s_part, q);
        s += pr[ccol];
        lim = fmin(lim, pr[kStripCols + ccol]);
      }
      si = s;
      li = lim;
      const bool whole = rank_exact(s, lim);
      if (whole) {
        s += sl;
        lim = fmin(lim, ml);
      }
      so = s;
      lo = lim;
      wok = whole;
    }
    if (warp < 4 && __any_sync(0xffffffffu, cok && !wok)) {
      const bool act = cok && !wok;
      double s = si, lim = li;
      const bool good = walk(s, lim, act, false);
      if (act) {
        so = s;
        lo = lim;
        wok = good;
      }
    }
    const int fail = __syncthreads_or(cok && !(exact && wok));
    if (threadIdx.x == 0) *s_fail = fail;
    cluster.sync();
    bool any = false;
    for (int q = 0; q < kStripCluster; ++q) any |= *cluster.map_shared_rank(s_fail, q) != 0;
    if (!any) {
      // 3. every start was the serial fold's own: the last rank's result carries
      if (rank == kStripCluster - 1 && cok) {
        double* dst = cluster.map_shared_rank(s_carry, 0);
        dst[ccol] = so;
        dst[kStripCols + ccol] = lo;
      }
      cluster.sync();
    } else {
      for (int p = 0; p < kStripCluster; ++p) {
        if (rank == p && warp < 4) {
          double s = s_carry[ccol], lim = s_carry[kStripCols + ccol];
          // a lane whose speculative start was the carry keeps its result; the others take the rank's test from the
          // carry, and walk from it if that fails
          bool again = cok && !(wok && __double_as_longlong(s) == __double_as_longlong(si) &&
                                __double_as_longlong(lim) == __double_as_longlong(li));
          if (again && rank_exact(s, lim)) {
            so = s + sl;
            lo = fmin(lim, ml);
            again = false;
          }
          if (__any_sync(0xffffffffu, again)) {
            walk(s, lim, again, true);
            if (again) {
              so = s;
              lo = lim;
            }
          }
          if (cok) {
            double* dst = cluster.map_shared_rank(s_carry, (p + 1) % kStripCluster);
            dst[ccol] = so;
            dst[kStripCols + ccol] = lo;
          }
        }
        cluster.sync();  // the hand-off is visible before the next rank reads it
      }
    }
  }
  if (rank == 0 && cok) {
    const double s = s_carry[ccol];
    out[c0 + ccol] = __double2float_rn(MEAN ? s / (double)rows : s);
  }
}

// f32 Sum/Mean over the outer axis in the launched lift's documented order for a logical block of B threads
// (kernel_lift/block_reduce.rs:13-30): logical thread t of column c folds rows t, t+B, t+2B, ... ascending into an
// f64; then acc[t] += acc[t+s] for s = B/2 .. 1; Mean divides by the row count; one rounding. A CTA takes 32
// columns (one per lane) and 16 warps; warp w holds logical threads w, w+16, ... (B/16 accumulators; B <= 256),
// so each step loads B/16 rows per thread, all coalesced across the 32 columns. The tree runs in shared memory.
constexpr int kDocWarps = 16, kDocMaxB = 256;
template <bool MEAN>
__global__ void __launch_bounds__(32 * kDocWarps) col_sum_f32_doc_kernel(const float* __restrict__ x, int64_t rows,
                                                                         int64_t cols, int64_t stride, int B,
                                                                         float* __restrict__ out, int64_t xb, int64_t ob) {
  x += (int64_t)blockIdx.z * xb;  // batch z of a middle-axis reduction
  out += (int64_t)blockIdx.z * ob;
  extern __shared__ double sacc[];  // [B][32]
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  const int J = B > kDocWarps ? B / kDocWarps : (w < B ? 1 : 0);  // logical threads of this warp
  double acc[kDocMaxB / kDocWarps];
#pragma unroll
  for (int j = 0; j < kDocMaxB / kDocWarps; ++j) acc[j] = 0.0;
  if (c < cols && J > 0) {
    for (int64_t r0 = 0; r0 < rows; r0 += B) {
      float v[kDocMaxB / kDocWarps];
#pragma unroll
      for (int j = 0; j < kDocMaxB / kDocWarps; ++j) {
        const int64_t r = r0 + w + (int64_t)kDocWarps * j;
        v[j] = (j < J && r < rows) ? __ldg(x + r * stride + c) : 0.0f;
      }
#pragma unroll
      for (int j = 0; j < kDocMaxB / kDocWarps; ++j)
        if (j < J && r0 + w + (int64_t)kDocWarps * j < rows) acc[j] += (double)v[j];
    }
  }
#pragma unroll
  for (int j = 0; j < kDocMaxB / kDocWarps; ++j)
    if (j < J) sacc[(w + kDocWarps * j) * 32 + lane] = acc[j];
  __syncthreads();
  for (int sh = B >> 1; sh > 0; sh >>= 1) {
    for (int i = threadIdx.x; i < sh * 32; i += 32 * kDocWarps) {
      const int t = i >> 5, l = i & 31;
      sacc[t * 32 + l] = sacc[t * 32 + l] + sacc[(t + sh) * 32 + l];
    }
    __syncthreads();
  }
  if (w == 0 && c < cols) out[c] = __double2float_rn(MEAN ? sacc[lane] / (double)rows : sacc[lane]);
}

// The documented order with 16-byte loads, for B = 64, 128 or 256: a strip of 128 columns (a float4 per lane) per
// CTA and a cluster of 8 CTAs per strip. Logical thread t = k + 8w + 64i lives in CTA rank k, warp w, slot i
// (I = B/64 slots per lane), so each warp reads 512 B of every row it touches. The tree's levels s >= 64 pair
// slots of one thread, s = 32, 16, 8 pair warps of one CTA (through shared memory) and s = 4, 2, 1 pair CTAs of the
// cluster (rank 0 reads the other ranks' values through distributed shared memory), each as acc[t] + acc[t+s].
//
// Occupancy sets the wave count: 8,192 columns are 512 CTAs, so the CTAs an SM holds decide whether they run as one
// wave. With four slots a lane (B = 256) the kernel keeps four rows in flight under a cap of four CTAs per SM (64
// registers, a few spilled): one wave, 1.09x faster than eight rows at two CTAs per SM (110 registers, 1.7 waves).
template <bool MEAN, int I>
__device__ __forceinline__ void col_sum_doc_vec_body(const float* __restrict__ x, int64_t rows, int64_t cols,
                                                     int64_t stride, float* __restrict__ out, int64_t xb, int64_t ob) {
  x += (int64_t)blockIdx.z * xb;  // batch z of a middle-axis reduction
  out += (int64_t)blockIdx.z * ob;
  namespace cg = cooperative_groups;
  constexpr int B = 64 * I, U = I == 4 ? 1 : 8 / I;  // U steps of I rows in flight per lane
  __shared__ double sw[8][kColStrip];
  __shared__ double cs[kColStrip];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int k = (int)blockIdx.y;
  const int64_t c0 = (int64_t)blockIdx.x * kColStrip + 4 * lane;
  double acc[I][4];
#pragma unroll
  for (int i = 0; i < I; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
  if (c0 < cols) {
    const float* base = x + c0;
    const int64_t M = (rows + B - 1) / B;
    auto add = [&](int i, int64_t r, const float4 v) {
      if (r < rows) {
        acc[i][0] += (double)v.x;
        acc[i][1] += (double)v.y;
        acc[i][2] += (double)v.z;
        acc[i][3] += (double)v.w;
      }
    };
    int64_t m = 0;
    for (; m + U <= M; m += U) {
      float4 v[U][I];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int i = 0; i < I; ++i) {
          const int64_t r = k + 8 * w + 64 * i + B * (m + u);
          v[u][i] = r < rows ? ld_nc_na_f4(base + r * stride) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int i = 0; i < I; ++i) add(i, k + 8 * w + 64 * i + B * (m + u), v[u][i]);
    }
    for (; m < M; ++m) {
#pragma unroll
      for (int i = 0; i < I; ++i) {
        const int64_t r = k + 8 * w + 64 * i + B * m;
        if (r < rows) add(i, r, ld_nc_na_f4(base + r * stride));
      }
    }
  }
#pragma unroll
  for (int h = I / 2; h >= 1; h >>= 1)  // levels s = 64h
#pragma unroll
    for (int i = 0; i < h; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = acc[i][j] + acc[i + h][j];
#pragma unroll
  for (int j = 0; j < 4; ++j) sw[w][4 * lane + j] = acc[0][j];
  __syncthreads();
  const int t = threadIdx.x;  // the strip's column t (threads 0 .. 127)
  if (t < kColStrip) {
    double v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = sw[q][t];
#pragma unroll
    for (int h = 4; h >= 1; h >>= 1)  // levels s = 8h: warp q and q + h
#pragma unroll
      for (int q = 0; q < h; ++q) v[q] = v[q] + v[q + h];
    cs[t] = v[0];
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();  // every CTA's values are visible to rank 0
  if (cluster.block_rank() == 0 && t < kColStrip) {
    double v[8];
    v[0] = cs[t];
#pragma unroll
    for (unsigned q = 1; q < 8; ++q) v[q] = *cluster.map_shared_rank(&cs[t], q);
#pragma unroll
    for (int h = 4; h >= 1; h >>= 1)  // levels s = h: rank q and q + h
#pragma unroll
      for (int q = 0; q < h; ++q) v[q] = v[q] + v[q + h];
    const int64_t c = (int64_t)blockIdx.x * kColStrip + t;
    if (c < cols) out[c] = __double2float_rn(MEAN ? v[0] / (double)rows : v[0]);
  }
  cluster.sync();  // rank 0 has read the other CTAs' shared memory before they exit
}

template <bool MEAN, int I>
__global__ void __cluster_dims__(1, kColCluster, 1) __launch_bounds__(256)
    col_sum_f32_doc_vec_kernel(const float* __restrict__ x, int64_t rows, int64_t cols, int64_t stride,
                               float* __restrict__ out, int64_t xb, int64_t ob) {
  col_sum_doc_vec_body<MEAN, I>(x, rows, cols, stride, out, xb, ob);
}
template <bool MEAN>
__global__ void __cluster_dims__(1, kColCluster, 1) __launch_bounds__(256, 4)
    col_sum_f32_doc_vec4_kernel(const float* __restrict__ x, int64_t rows, int64_t cols, int64_t stride,
                                float* __restrict__ out, int64_t xb, int64_t ob) {
  col_sum_doc_vec_body<MEAN, 4>(x, rows, cols, stride, out, xb, ob);
}

// The same with 16-byte loads (a thread takes 4 adjacent columns, a CTA 1024 columns, 4 KB of each row).
template <int OP>
__global__ void __launch_bounds__(kThreads) col_fold_i32_vec_kernel(const int32_t* __restrict__ x, int64_t rows,
                                                                     int64_t cols, int64_t stride, int64_t per_split,
                                                                     int32_t* __restrict__ out, int64_t xb, int64_t ob) {
  x += (int64_t)blockIdx.z * xb;  // batch z of a middle-axis reduction
  out += (int64_t)blockIdx.z * ob;
  const int64_t c = ((int64_t)blockIdx.x * kThreads + threadIdx.x) * 4;
  if (c >= cols) return;
  const int64_t r0 = (int64_t)blockIdx.y * per_split;
  const int64_t r1 = r0 + per_split < rows ? r0 + per_split : rows;
  int32_t a[4] = {ident<OP>(), ident<OP>(), ident<OP>(), ident<OP>()};
  int64_t r = r0;
  for (; r + 3 < r1; r += 4) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = ld_nc_na_v4(x + (r + u) * stride + c);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      a[0] = comb<OP>(a[0], (int32_t)v[u].x);
      a[1] = comb<OP>(a[1], (int32_t)v[u].y);
      a[2] = comb<OP>(a[2], (int32_t)v[u].z);
      a[3] = comb<OP>(a[3], (int32_t)v[u].w);
    }
  }
  for (; r < r1; ++r) {
    const uint4 v = ld_nc_na_v4(x + r * stride + c);
    a[0] = comb<OP>(a[0], (int32_t)v.x);
    a[1] = comb<OP>(a[1], (int32_t)v.y);
    a[2] = comb<OP>(a[2], (int32_t)v.z);
    a[3] = comb<OP>(a[3], (int32_t)v.w);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) col_combine_out<OP>(out + c + j, a[j]);
}

template <int OP>
int launch_i32_rows(const int32_t* x, int64_t rows, int64_t cols, int64_t stride, int32_t* out, cudaStream_t s) {
  const int sms = sm_count();
  const bool vec = aligned(x, 16) && cols % 4 == 0 && stride % 4 == 0;
  // rows held in registers with the next row's loads in flight need only two CTAs per SM (measured best)
  const int64_t per_sm = vec && cols / 4 <= 8 * kThreads ? 2 : 8;
  const int64_t g = rows < (int64_t)sms * per_sm ? rows : (int64_t)sms * per_sm;
  if (vec) row_fold_i32_kernel<OP, true><<<(int)g, kThreads, 0, s>>>(x, rows, cols, stride, out);
  else row_fold_i32_kernel<OP, false><<<(int)g, kThreads, 0, s>>>(x, rows, cols, stride, out);
  note_launch();
  return check_launch();
}

constexpr int64_t kMaxGridZ = 65535;

// The middle axis of [outer, rows, cols] (outer 1: axis 0 of [rows, cols]) into out[outer][cols] (row stride ob);
// batch b reads x + b * xb. Batches ride on gridDim.z, in chunks of at most 65535.
template <int OP>
int launch_i32_cols(const int32_t* x, int64_t outer, int64_t rows, int64_t cols, int64_t xb, int64_t stride,
                    int32_t* out, int64_t ob, cudaStream_t s) {
  const int sms = sm_count();
  const bool vec = aligned(x, 16) && cols % 4 == 0 && stride % 4 == 0 && xb % 4 == 0;
  const int64_t gx = vec ? (cols + 4 * kThreads - 1) / (4 * kThreads) : (cols + kThreads - 1) / kThreads;
  for (int64_t b0 = 0; b0 < outer; b0 += kMaxGridZ) {
    const int64_t nb = outer - b0 < kMaxGridZ ? outer - b0 : kMaxGridZ;
    const int32_t* xs = x + b0 * xb;
    int32_t* os = out + b0 * ob;
    col_init_i32_kernel<OP><<<dim3((unsigned)(gx < 4096 ? gx : 4096), 1, (unsigned)nb), kThreads, 0, s>>>(os, cols, ob);
    note_launch();
    if (rows == 0) {  // an empty fold stores 0 (1 for Prod): overwrite the identity
      if (OP != UP_OP_PROD) {
        const cudaError_t e = cudaMemset2DAsync(os, sizeof(int32_t) * (size_t)ob, 0, sizeof(int32_t) * (size_t)cols,
                                                (size_t)nb, s);
        if (e != cudaSuccess) return cuda_status(e);
      }
      continue;
    }
    int64_t splits = ((int64_t)sms * 4 + gx * nb - 1) / (gx * nb);
    const int64_t max_splits = (rows + 63) / 64;
    if (splits > max_splits) splits = max_splits;
    if (splits > 65535) splits = 65535;
    if (splits < 1) splits = 1;
    const int64_t per = (rows + splits - 1) / splits;
    splits = (rows + per - 1) / per;
    const dim3 grid((unsigned)gx, (unsigned)splits, (unsigned)nb);
    if (vec)
      col_fold_i32_vec_kernel<OP><<<grid, kThreads, 0, s>>>(xs, rows, cols, stride, per, os, xb, ob);
    else
      col_fold_i32_kernel<OP><<<grid, kThreads, 0, s>>>(xs, rows, cols, stride, per, os, xb, ob);
    note_launch();
    const int st = check_launch();
    if (st != UP_OK) return st;
  }
  return check_launch();
}

template <int OP>
int launch_i32(const int32_t* x, int64_t outer, int64_t rows, int64_t cols, int64_t xb, int64_t stride, int axis,
               int32_t* out, int64_t ob, cudaStream_t s) {
  if (axis == 1 && outer == 1) return launch_i32_rows<OP>(x, rows, cols, stride, out, s);
  return launch_i32_cols<OP>(x, outer, rows, cols, xb, stride, out, ob, s);
}

// f32 over the middle axis of [outer, rows, cols] (outer 1: axis 0), as launch_i32_cols.
int launch_f32_cols(const float* x, int64_t outer, int64_t rows, int64_t cols, int64_t xb, int64_t row_stride,
                    int op, int accum, int block, float* out, int64_t ob, cudaStream_t s) {
  const bool summing = op == UP_OP_SUM || op == UP_OP_MEAN;
  // Sum/Mean in the serial order (block 1) or the documented order of a logical block of up to 256
  if (summing && accum != UP_ACCUM_AUTO)
    return fail_with(UP_ERR_UNSUPPORTED, "reduce2d_f32: an outer-axis Sum/Mean is lowered for Auto");
  if (summing && block > 1 && (block > kDocMaxB || (block & (block - 1)) != 0))
    return fail_with(UP_ERR_UNSUPPORTED, "reduce2d_f32: an outer-axis block is a power of two up to 256");
  if (rows > 0x7fffffffLL) return UP_ERR_UNSUPPORTED;
  const int64_t gx = (cols + kThreads - 1) / kThreads;
  if (gx > 0x7fffffff) return UP_ERR_UNSUPPORTED;
  const bool vec = aligned(x, 16) && cols % 4 == 0 && row_stride % 4 == 0 && xb % 4 == 0;
  if (summing && block == 1 && vec) {
    cudaError_t e = ensure_smem_attr((const void*)col_sum_f32_serial_strip_kernel<true>, kStripSmem);
    if (e == cudaSuccess) e = ensure_smem_attr((const void*)col_sum_f32_serial_strip_kernel<false>, kStripSmem);
    if (e != cudaSuccess) return cuda_status(e);
  }
  if (summing && block > 1 && !(block >= 64 && vec)) {
    const int bytes = (int)((size_t)kDocMaxB * 32 * sizeof(double));
    cudaError_t e = ensure_smem_attr((const void*)col_sum_f32_doc_kernel<true>, bytes);
    if (e == cudaSuccess) e = ensure_smem_attr((const void*)col_sum_f32_doc_kernel<false>, bytes);
    if (e != cudaSuccess) return cuda_status(e);
  }
  const bool mean = op == UP_OP_MEAN;
  for (int64_t b0 = 0; b0 < outer; b0 += kMaxGridZ) {
    const unsigned nb = (unsigned)(outer - b0 < kMaxGridZ ? outer - b0 : kMaxGridZ);
    const float* xs = x + b0 * xb;
    float* os = out + b0 * ob;
    if (summing && block > 1 && block >= 64 && vec) {
      const dim3 grid((unsigned)((cols + kColStrip - 1) / kColStrip), kColCluster, nb);
      if (block == 64)
        mean ? col_sum_f32_doc_vec_kernel<true, 1><<<grid, 256, 0, s>>>(xs, rows, cols, row_stride, os, xb, ob)
             : col_sum_f32_doc_vec_kernel<false, 1><<<grid, 256, 0, s>>>(xs, rows, cols, row_stride, os, xb, ob);
      else if (block == 128)
        mean ? col_sum_f32_doc_vec_kernel<true, 2><<<grid, 256, 0, s>>>(xs, rows, cols, row_stride, os, xb, ob)
             : col_sum_f32_doc_vec_kernel<false, 2><<<grid, 256, 0, s>>>(xs, rows, cols, row_stride, os, xb, ob);
      else
        mean ? col_sum_f32_doc_vec4_kernel<true><<<grid, 256, 0, s>>>(xs, rows, cols, row_stride, os, xb, ob)
             : col_sum_f32_doc_vec4_kernel<false><<<grid, 256, 0, s>>>(xs, rows, cols, row_stride, os, xb, ob);
    } else if (summing && block > 1) {
      const size_t smem = (size_t)block * 32 * sizeof(double);
      const dim3 grid((unsigned)((cols + 31) / 32), 1, nb);
      if (mean)
        col_sum_f32_doc_kernel<true><<<grid, 32 * kDocWarps, smem, s>>>(xs, rows, cols, row_stride, block, os, xb, ob);
      else
        col_sum_f32_doc_kernel<false><<<grid, 32 * kDocWarps, smem, s>>>(xs, rows, cols, row_stride, block, os, xb, ob);
    } else if (summing && vec) {
      const dim3 grid((unsigned)((cols + kStripCols - 1) / kStripCols), kStripCluster, nb);
      if (mean)
        col_sum_f32_serial_strip_kernel<true><<<grid, 32 * kStripWarps, kStripSmem, s>>>(xs, rows, cols, row_stride,
                                                                                      os, xb, ob);
      else
        col_sum_f32_serial_strip_kernel<false><<<grid, 32 * kStripWarps, kStripSmem, s>>>(xs, rows, cols, row_stride,
                                                                                       os, xb, ob);
    } else if (summing) {
      const dim3 grid((unsigned)((cols + 31) / 32), 1, nb);
      if (mean)
        col_sum_f32_serial_spec_kernel<true><<<grid, 32 * (kSpecProducers + 1), 0, s>>>(xs, rows, cols, row_stride, os,
                                                                                       xb, ob);
      else
        col_sum_f32_serial_spec_kernel<false><<<grid, 32 * (kSpecProducers + 1), 0, s>>>(xs, rows, cols, row_stride,
                                                                                        os, xb, ob);
    } else if (vec) {
      const dim3 grid((unsigned)((cols + kColStrip - 1) / kColStrip), kColCluster, nb);
      if (op == UP_OP_MAX)
        col_extremum_f32_vec_kernel<true><<<grid, 32 * kColVecWarps, 0, s>>>(xs, rows, cols, row_stride, os, xb, ob);
      else
        col_extremum_f32_vec_kernel<false><<<grid, 32 * kColVecWarps, 0, s>>>(xs, rows, cols, row_stride, os, xb, ob);
    } else {
      const dim3 grid((unsigned)((cols + 31) / 32), 1, nb);
      if (op == UP_OP_MAX)
        col_extremum_f32_kernel<true><<<grid, 32 * kColWarps, 0, s>>>(xs, rows, cols, row_stride, os, xb, ob);
      else
        col_extremum_f32_kernel<false><<<grid, 32 * kColWarps, 0, s>>>(xs, rows, cols, row_stride, os, xb, ob);
    }
    note_launch();
    const int st = check_launch();
    if (st != UP_OK) return st;
  }
  return UP_OK;
}

}  // namespace r2
}  // namespace up

using namespace up;
using namespace up::r2;

static int reduce_i32(const int32_t* x, int64_t outer, int64_t rows, int64_t cols, int64_t xb, int64_t row_stride,
                      int axis, int op, int32_t* out, int64_t ob, cudaStream_t s) {
  if (rows > 65535LL * 0x7fffffffLL || cols > 0x7fffffffLL * kThreads) return UP_ERR_UNSUPPORTED;
  switch (op) {
    case UP_OP_SUM: return launch_i32<UP_OP_SUM>(x, outer, rows, cols, xb, row_stride, axis, out, ob, s);
    case UP_OP_PROD: return launch_i32<UP_OP_PROD>(x, outer, rows, cols, xb, row_stride, axis, out, ob, s);
    case UP_OP_MAX: return launch_i32<UP_OP_MAX>(x, outer, rows, cols, xb, row_stride, axis, out, ob, s);
    case UP_OP_MIN: return launch_i32<UP_OP_MIN>(x, outer, rows, cols, xb, row_stride, axis, out, ob, s);
    case UP_OP_AND: return launch_i32<UP_OP_AND>(x, outer, rows, cols, xb, row_stride, axis, out, ob, s);
    case UP_OP_OR: return launch_i32<UP_OP_OR>(x, outer, rows, cols, xb, row_stride, axis, out, ob, s);
    case UP_OP_XOR: return launch_i32<UP_OP_XOR>(x, outer, rows, cols, xb, row_stride, axis, out, ob, s);
    default: return UP_ERR_UNSUPPORTED;
  }
}

extern "C" int up_sm100_reduce2d_i32(const int32_t* x, int64_t rows, int64_t cols, int64_t row_stride, int axis,
                                     int op, int32_t* out, void* stream) {
  UP_CHECK_ARG(rows >= 0 && cols >= 0 && row_stride >= cols && (axis == 0 || axis == 1));
  UP_CHECK_ARG(out != nullptr || (axis == 1 ? rows : cols) == 0);
  if ((axis == 1 ? rows : cols) == 0) return UP_OK;
  UP_CHECK_ARG(x != nullptr || (axis == 1 ? cols : rows) == 0);
  return reduce_i32(x, 1, rows, cols, 0, row_stride, axis, op, out, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int up_sm100_reduce3d_i32(const int32_t* x, int64_t outer, int64_t rows, int64_t cols,
                                     int64_t outer_stride, int64_t row_stride, int op, int32_t* out,
                                     int64_t out_stride, void* stream) {
  UP_CHECK_ARG(outer >= 0 && rows >= 0 && cols >= 0 && row_stride >= cols && out_stride >= cols);
  UP_CHECK_ARG(outer <= 1 || outer_stride >= rows * row_stride);
  if (outer == 0 || cols == 0) return UP_OK;
  UP_CHECK_ARG(out != nullptr && (x != nullptr || rows == 0));
  return reduce_i32(x, outer, rows, cols, outer_stride, row_stride, 0, op, out, out_stride,
                    static_cast<cudaStream_t>(stream));
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
    if (cols > 0x7fffffffLL) return UP_ERR_UNSUPPORTED;  // indices are 32-bit
    const bool vec = aligned(x, 16) && cols % 4 == 0 && row_stride % 4 == 0;
    const int64_t per_sm = vec && cols / 4 <= 8 * kThreads ? 2 : 8;  // as for the i32 fold (measured best)
    const int g = (int)(rows < (int64_t)sm_count() * per_sm ? rows : (int64_t)sm_count() * per_sm);
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
  return launch_f32_cols(x, 1, rows, cols, 0, row_stride, op, accum, block, out, 0, s);
}

extern "C" int up_sm100_reduce3d_f32(const float* x, int64_t outer, int64_t rows, int64_t cols, int64_t outer_stride,
                                     int64_t row_stride, int op, int accum, int block, float* out, int64_t out_stride,
                                     void* stream) {
  UP_CHECK_ARG(outer >= 0 && rows >= 0 && cols >= 0 && row_stride >= cols && out_stride >= cols);
  UP_CHECK_ARG(outer <= 1 || outer_stride >= rows * row_stride);
  if (op != UP_OP_SUM && op != UP_OP_MEAN && op != UP_OP_MAX && op != UP_OP_MIN) return UP_ERR_UNSUPPORTED;
  if (outer == 0 || cols == 0) return UP_OK;
  UP_CHECK_ARG(out != nullptr && (x != nullptr || rows == 0));
  return launch_f32_cols(x, outer, rows, cols, outer_stride, row_stride, op, accum, block, out, out_stride,
                         static_cast<cudaStream_t>(stream));
}

UP_DEFINE_REVISION(reduce2d)
