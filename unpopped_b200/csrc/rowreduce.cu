// rowreduce.cu — the launched RowReduce lift (Access::RowReduce; crates/unpopped/src/kernel_lift/
// row_reduce_launched.rs:1-24) for its named forms over f32 rows:
//   softmax          stage 0 Max(x), stage 1 Sum(exp(x - r0)),     epilogue exp(x - r0) / r1
//   RMS norm         stage 0 Mean(x * x),                          epilogue x / sqrt(r0 + eps)
//   centred quotient stage 0 Mean(x), stage 1 Max(x - r0),         epilogue (x - r0) / r1
// (the forms of crates/unpopped/tests/kernel_parallel_row_reduce_agrees.rs:99-131).
//
// Numerics, as the launched lift defines them for a logical block of B threads:
//  * Every expression is evaluated in f64 from the f32 inputs and the f32 stage values (the kernel interpreter
//    evaluates in f64 and rounds when a value is stored; oracle/expr_eval.rs, kernel_eval.rs).
//  * A Sum/Mean stage folds logical thread t's elements t, t+B, t+2B, ... ascending into an f64, then
//    acc[t] += acc[t+s] for s = B/2 .. 1 (kernel_lift/block_reduce.rs:13-23); Mean divides by the row length.
//  * A Max stage is NaN-keeping and order-independent (plan_contract.rs:300-315).
//  * Thread 0 rounds each stage value once to f32; later stages and the epilogue read that f32 value
//    (row_reduce_launched.rs:86-120); the epilogue rounds once on the store.
// exp and sqrt are CUDA's f64 functions (sqrt is correctly rounded; exp is within an ulp of f64), so results are
// within the reference's stated few-ulp band of its serial lift and, after the f32 rounding, almost always
// bit-equal to the CPU restatement.
//
// Layout: a row group of G = min(B, 256) threads per row (256 / G rows per CTA), L = B / G logical threads per
// thread. Element k of thread p is column j = p + G·k; it belongs to logical thread p + G·(k mod L), whose
// elements come in ascending order as k ascends, so acc[k mod L] += pre(j) over ascending k is the written order.
#include "common.cuh"

#include <cmath>
#include <mutex>

namespace up {
namespace rr {

constexpr int kThreads = 256;
constexpr int kCache = 32;  // elements per thread held in registers across the stages
constexpr int kFormSoftmax = 1, kFormRmsNorm = 2, kFormCentred = 3;

// NaN-keeping f64 max across the row group (all G threads get it): NaN if any is NaN, else the largest.
__device__ __forceinline__ double nan_max(double a, double b) { return (a != a || b != b) ? (a != a ? a : b) : fmax(a, b); }

__device__ double group_max(double v, int G, int p, int grp, double* wred, double* slot) {
  const int width = G < 32 ? G : 32;
  for (int o = width >> 1; o >= 1; o >>= 1) v = nan_max(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (G > 32) {
    if (lane == 0) wred[w] = v;
    __syncthreads();
    if (p == 0) {
      double m = wred[w];
      for (int k = 1; k < G / 32; ++k) m = nan_max(m, wred[w + k]);
      slot[grp] = m;
    }
  } else if (p == 0) {
    slot[grp] = v;
  }
  __syncthreads();
  const double r = slot[grp];
  __syncthreads();  // the slot is read before it is reused
  return r;
}

// The written tree over the group's B logical threads (acc[q] = logical thread p + G·q); the total, in every
// thread of the group. Levels s >= G pair partials of one thread, G > s >= 32 pair warps (shared memory, one
// barrier per level), s < 32 pair lanes (shuffles).
template <int L>
__device__ double group_tree(double (&acc)[L], int G, int p, int grp, double* region, double* slot) {
#pragma unroll
  for (int h = L / 2; h >= 1; h >>= 1)
#pragma unroll
    for (int q = 0; q < h; ++q) acc[q] = acc[q] + acc[q + h];
  double v = acc[0];
  int d = G >> 1, off = 0;
  double* reg = region + grp * G;
  for (; d >= 32; d >>= 1) {
    if (p >= d && p < 2 * d) reg[off + p - d] = v;
    __syncthreads();
    if (p < d) v = v + reg[off + p];
    off += d;
  }
  for (; d >= 1; d >>= 1) v = v + __shfl_down_sync(0xffffffffu, v, d);
  if (p == 0) slot[grp] = v;
  __syncthreads();
  const double r = slot[grp];
  __syncthreads();
  return r;
}

template <int FORM, int L, bool CACHED>
__global__ void __launch_bounds__(kThreads) row_reduce_f32_kernel(const float* __restrict__ x, int64_t rows,
                                                                   int64_t cols, int64_t stride, int B, double eps,
                                                                   float* __restrict__ out, int64_t ostride) {
  __shared__ double region[kThreads];  // the cross-warp tree levels of every row group
  __shared__ double wred[kThreads / 32];
  __shared__ double slot[kThreads];
  const int G = B / L;
  const int rpc = kThreads / G;
  const int grp = threadIdx.x / G, p = threadIdx.x - grp * G;
  const int64_t K = (cols + G - 1 - p) / G;  // this thread's elements
  for (int64_t r0 = (int64_t)blockIdx.x * rpc; r0 < rows; r0 += (int64_t)gridDim.x * rpc) {
    const int64_t r = r0 + grp;
    const bool live = r < rows;
    const float* row = x + (live ? r : 0) * stride;
    float xv[CACHED ? kCache : 1];
    if constexpr (CACHED) {
#pragma unroll
      for (int k = 0; k < kCache; ++k) xv[k] = (live && k < K) ? __ldg(row + p + (int64_t)G * k) : 0.0f;
    }
    auto xat = [&](int64_t k) -> float { return __ldg(row + p + (int64_t)G * k); };  // the streaming form
    const int64_t kn = live ? (CACHED ? (K < kCache ? K : kCache) : K) : 0;

    // stage 0
    float r0f;
    if (FORM == kFormSoftmax) {
      double m = -INFINITY;
      if constexpr (CACHED) {
#pragma unroll
        for (int k = 0; k < kCache; ++k)
          if (k < kn) m = nan_max(m, (double)xv[k]);
      } else {
        for (int64_t k = 0; k < kn; ++k) m = nan_max(m, (double)xat(k));
      }
      r0f = (float)group_max(m, G, p, grp, wred, slot);
    } else {
      double acc[L];
#pragma unroll
      for (int q = 0; q < L; ++q) acc[q] = 0.0;
      if constexpr (CACHED) {
#pragma unroll
        for (int k = 0; k < kCache; ++k)
          if (k < kn) {
            const double v = (double)xv[k];
            acc[k % L] += FORM == kFormRmsNorm ? v * v : v;
          }
      } else {
        for (int64_t k = 0; k < kn; ++k) {
          const double v = (double)xat(k);
#pragma unroll
          for (int q = 0; q < L; ++q)
            if ((int)(k % L) == q) acc[q] += FORM == kFormRmsNorm ? v * v : v;
        }
      }
      r0f = (float)(group_tree<L>(acc, G, p, grp, region, slot) / (double)cols);
    }

    // stage 1 and the epilogue
    float* orow = out + (live ? r : 0) * ostride;
    if (FORM == kFormSoftmax) {
      double acc[L];
#pragma unroll
      for (int q = 0; q < L; ++q) acc[q] = 0.0;
      double ev[CACHED ? kCache : 1];
      if constexpr (CACHED) {
#pragma unroll
        for (int k = 0; k < kCache; ++k)
          if (k < kn) {
            ev[k] = exp((double)xv[k] - (double)r0f);
            acc[k % L] += ev[k];
          }
      } else {
        for (int64_t k = 0; k < kn; ++k) {
          const double e = exp((double)xat(k) - (double)r0f);
#pragma unroll
          for (int q = 0; q < L; ++q)
            if ((int)(k % L) == q) acc[q] += e;
        }
      }
      const double r1 = (double)(float)group_tree<L>(acc, G, p, grp, region, slot);
      if constexpr (CACHED) {
#pragma unroll
        for (int k = 0; k < kCache; ++k)
          if (k < kn) orow[p + (int64_t)G * k] = (float)(ev[k] / r1);
      } else {
        for (int64_t k = 0; k < kn; ++k) orow[p + (int64_t)G * k] = (float)(exp((double)xat(k) - (double)r0f) / r1);
      }
    } else if (FORM == kFormRmsNorm) {
      const double den = sqrt((double)r0f + eps);
      if constexpr (CACHED) {
#pragma unroll
        for (int k = 0; k < kCache; ++k)
          if (k < kn) orow[p + (int64_t)G * k] = (float)((double)xv[k] / den);
      } else {
        for (int64_t k = 0; k < kn; ++k) orow[p + (int64_t)G * k] = (float)((double)xat(k) / den);
      }
    } else {
      double m = -INFINITY;
      if constexpr (CACHED) {
#pragma unroll
        for (int k = 0; k < kCache; ++k)
          if (k < kn) m = nan_max(m, (double)xv[k] - (double)r0f);
      } else {
        for (int64_t k = 0; k < kn; ++k) m = nan_max(m, (double)xat(k) - (double)r0f);
      }
      const double r1 = (double)(float)group_max(m, G, p, grp, wred, slot);
      if constexpr (CACHED) {
#pragma unroll
        for (int k = 0; k < kCache; ++k)
          if (k < kn) orow[p + (int64_t)G * k] = (float)(((double)xv[k] - (double)r0f) / r1);
      } else {
        for (int64_t k = 0; k < kn; ++k) orow[p + (int64_t)G * k] = (float)(((double)xat(k) - (double)r0f) / r1);
      }
    }
  }
}

// ---- the register-resident form (at most 32 elements per thread) ----
// A quotient a / b is rounded to f32 as RN(a * RN(1 / b)): that product is within 2 f64 ulps of the quotient, so its
// f32 rounding is the quotient's unless the product lies within 4 ulps of an f32 rounding midpoint or outside the
// f32 normal range, which take the exact division (div_round_f32). exp is CUDA's f64 exp; a table-driven exp
// (Tang's method) and an integer f32 -> f64 widening both measured slower here.
__device__ __noinline__ float div_exact_f32(double a, double b) { return __double2float_rn(a / b); }

__device__ __forceinline__ float div_round_f32(double a, double b, double inv) {
  const double q = a * inv;
  const uint64_t u = (uint64_t)__double_as_longlong(q);
  const uint32_t e = (uint32_t)(u >> 52) & 0x7ffu;
  const uint32_t low = (uint32_t)u & 0x1fffffffu;
  if (e - 898u < 250u && low - (0x10000000u - 4u) > 8u) return __double2float_rn(q);
  return div_exact_f32(a, b);
}

__device__ __forceinline__ void cp_async4(float* smem, const float* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((unsigned)__cvta_generic_to_shared(smem)), "l"(gmem)
               : "memory");
}

// Rows are staged through shared memory by cp.async, the next rows' copies in flight while this row is computed:
// two buffers of kCache * kThreads floats (each row group's row at grp * kCache * G).
template <int FORM, int L, bool WHOLE>
__global__ void __launch_bounds__(kThreads) row_reduce_f32_held_kernel(const float* __restrict__ x, int64_t rows,
                                                                        int64_t cols, int64_t stride, int B,
                                                                        double eps, float* __restrict__ out,
                                                                        int64_t ostride) {
  __shared__ double region[kThreads];
  __shared__ double wred[kThreads / 32];
  __shared__ double slot[kThreads];
  extern __shared__ __align__(16) float stage[];  // [2][kCache * kThreads]
  const int G = B / L;
  const int rpc = kThreads / G;
  const int grp = threadIdx.x / G, p = threadIdx.x - grp * G;
  const int64_t K = (cols + G - 1 - p) / G;
  const int64_t rstep = (int64_t)gridDim.x * rpc;
  auto issue = [&](int64_t rr, int buf) {
    if (rr < rows) {
      const float* src = x + rr * stride + p;
      float* dst = &stage[buf * kCache * kThreads + grp * kCache * G + p];
#pragma unroll
      for (int k = 0; k < kCache; ++k)
        if (WHOLE || k < K) cp_async4(dst + G * k, src + (int64_t)G * k);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  issue((int64_t)blockIdx.x * rpc + grp, 0);
  int it = 0;
  for (int64_t r0 = (int64_t)blockIdx.x * rpc; r0 < rows; r0 += rstep, ++it) {
    const int64_t r = r0 + grp;
    const bool live = r < rows;
    float* orow = out + (live ? r : 0) * ostride;
    const int kn = live ? (int)(K < kCache ? K : kCache) : 0;
    issue(r + rstep, (it + 1) & 1);  // the next rows, into the buffer read two rows ago
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();  // every thread's copies of this row have landed
    float xv[kCache];
    const float* src = &stage[(it & 1) * kCache * kThreads + grp * kCache * G + p];
#pragma unroll
    for (int k = 0; k < kCache; ++k) xv[k] = WHOLE || k < kn ? src[G * k] : 0.0f;
    double acc[L];
#pragma unroll
    for (int q = 0; q < L; ++q) acc[q] = 0.0;
    if (FORM == kFormSoftmax) {
      float m = -INFINITY;
#pragma unroll
      for (int k = 0; k < kCache; ++k)
        if (WHOLE || k < kn) asm("max.NaN.f32 %0, %0, %1;" : "+f"(m) : "f"(xv[k]));
      const double r0d = (double)(float)group_max((double)m, G, p, grp, wred, slot);
      double ev[kCache];
#pragma unroll
      for (int k = 0; k < kCache; ++k) ev[k] = exp((double)xv[k] - r0d);
#pragma unroll
      for (int k = 0; k < kCache; ++k)
        if (WHOLE || k < kn) acc[k % L] += ev[k];
      const double r1 = (double)(float)group_tree<L>(acc, G, p, grp, region, slot);
      const double inv = 1.0 / r1;
#pragma unroll
      for (int k = 0; k < kCache; ++k)
        if (WHOLE ? live : k < kn) orow[p + (int64_t)G * k] = div_round_f32(ev[k], r1, inv);
    } else {
      double xd[kCache];
#pragma unroll
      for (int k = 0; k < kCache; ++k) xd[k] = (double)xv[k];
#pragma unroll
      for (int k = 0; k < kCache; ++k)
        if (WHOLE || k < kn) acc[k % L] += FORM == kFormRmsNorm ? xd[k] * xd[k] : xd[k];
      const double r0d = (double)(float)(group_tree<L>(acc, G, p, grp, region, slot) / (double)cols);
      if (FORM == kFormRmsNorm) {
        const double den = sqrt(r0d + eps);
        const double inv = 1.0 / den;
#pragma unroll
        for (int k = 0; k < kCache; ++k)
          if (WHOLE ? live : k < kn) orow[p + (int64_t)G * k] = div_round_f32(xd[k], den, inv);
      } else {
        double m = -INFINITY;
#pragma unroll
        for (int k = 0; k < kCache; ++k)
          if (WHOLE || k < kn) m = nan_max(m, xd[k] - r0d);
        const double r1 = (double)(float)group_max(m, G, p, grp, wred, slot);
        const double inv = 1.0 / r1;
#pragma unroll
        for (int k = 0; k < kCache; ++k)
          if (WHOLE ? live : k < kn) orow[p + (int64_t)G * k] = div_round_f32(xd[k] - r0d, r1, inv);
      }
    }
  }
}

// The held path's launch: the staged-row buffers need 64 KB of dynamic shared memory, an attribute set once per
// device and instantiation; the grid is the CTAs that fit on every SM at once (two or three, by registers).
template <int FORM, int L, bool WHOLE>
int launch_held(const float* x, int64_t rows, int64_t cols, int64_t stride, int B, double eps, float* out,
                int64_t ostride, int64_t g, cudaStream_t s) {
  constexpr size_t smem = 2 * sizeof(float) * kCache * kThreads;
  static std::mutex mu;
  static int per_sm[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  int fit = 0;
  e = ensure_smem_attr((const void*)row_reduce_f32_held_kernel<FORM, L, WHOLE>, (int)smem);
  if (e != cudaSuccess) return cuda_status(e);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64) fit = per_sm[dev];
    if (fit == 0) {
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&fit, row_reduce_f32_held_kernel<FORM, L, WHOLE>, kThreads,
                                                        smem);
      if (e != cudaSuccess) return cuda_status(e);
      if (fit < 1) fit = 1;
      if (dev >= 0 && dev < 64) per_sm[dev] = fit;
    }
  }
  const int64_t held_cap = (int64_t)sm_count() * fit;
  row_reduce_f32_held_kernel<FORM, L, WHOLE><<<(int)(g < held_cap ? g : held_cap), kThreads, smem, s>>>(
      x, rows, cols, stride, B, eps, out, ostride);
  return UP_OK;
}

template <int FORM, int L>
int launch_form(const float* x, int64_t rows, int64_t cols, int64_t stride, int B, double eps, float* out,
                int64_t ostride, cudaStream_t s) {
  const int G = B / L;
  const int rpc = kThreads / G;
  int64_t g = (rows + rpc - 1) / rpc;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (g > cap) g = cap;
  if (cols <= (int64_t)kCache * G) {
    // A row that fills each thread's kCache slots exactly needs no per-slot bound.
    const int rc = cols == (int64_t)kCache * G
                       ? launch_held<FORM, L, true>(x, rows, cols, stride, B, eps, out, ostride, g, s)
                       : launch_held<FORM, L, false>(x, rows, cols, stride, B, eps, out, ostride, g, s);
    if (rc != UP_OK) return rc;
  } else
    row_reduce_f32_kernel<FORM, L, false><<<(int)g, kThreads, 0, s>>>(x, rows, cols, stride, B, eps, out, ostride);
  note_launch();
  return check_launch();
}

template <int FORM>
int launch(const float* x, int64_t rows, int64_t cols, int64_t stride, int B, double eps, float* out, int64_t ostride,
           cudaStream_t s) {
  if (B <= kThreads) return launch_form<FORM, 1>(x, rows, cols, stride, B, eps, out, ostride, s);
  if (B == 2 * kThreads) return launch_form<FORM, 2>(x, rows, cols, stride, B, eps, out, ostride, s);
  return launch_form<FORM, 4>(x, rows, cols, stride, B, eps, out, ostride, s);
}

}  // namespace rr
}  // namespace up

using namespace up;

extern "C" int up_sm100_row_reduce_f32(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int form,
                                       int block, double eps, float* out, int64_t out_stride, void* stream) {
  UP_CHECK_ARG(rows >= 0 && cols >= 0 && row_stride >= cols && out_stride >= cols);
  if (form != rr::kFormSoftmax && form != rr::kFormRmsNorm && form != rr::kFormCentred) return UP_ERR_UNSUPPORTED;
  if (block < 1 || block > 1024 || (block & (block - 1)) != 0)
    return fail_with(UP_ERR_UNSUPPORTED, "row_reduce: the block is a power of two up to 1024");
  if (cols > 0x7fffffffLL) return UP_ERR_UNSUPPORTED;
  if (rows == 0 || cols == 0) return UP_OK;
  UP_CHECK_ARG(x != nullptr && out != nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (form) {
    case rr::kFormSoftmax: return rr::launch<rr::kFormSoftmax>(x, rows, cols, row_stride, block, eps, out, out_stride, s);
    case rr::kFormRmsNorm: return rr::launch<rr::kFormRmsNorm>(x, rows, cols, row_stride, block, eps, out, out_stride, s);
    default: return rr::launch<rr::kFormCentred>(x, rows, cols, row_stride, block, eps, out, out_stride, s);
  }
}

UP_DEFINE_REVISION(rowreduce)
