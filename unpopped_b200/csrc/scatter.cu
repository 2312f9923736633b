// scatter.cu — the launched Scatter lift: scatter / index_add with an atomic combine over axis 0 of a rank-2
// destination, and bincount.
//
// Semantics: the scatter store of the oracle (crates/unpopped/src/oracle/plan_eval.rs:430-490) with
// `WriteIndex::ScatterIndexed` (crates/unpopped/src/ir.rs:2723-2850): for every source element (i, j) of
// updates [n, cols], the target row is t = ids[i][j] (a full-shape index: torch `scatter_add`) or t = ids[i] (a 1-D
// index broadcast over the row: `index_add`), and out[t][j] = combine(out[t][j], updates[i][j]); a target outside
// [0, out_rows) is skipped (the Skip policy, no wrap of negatives). The destination holds its prior contents.
//  * Integer AtomicAdd (wrapping at the dtype's width), AtomicMax and AtomicMin are order-independent, so the
//    result is bit-exact against the serial oracle whatever order the atomics land in
//    (crates/unpopped/tests/kernel_parallel_scatter_agrees.rs:1-8).
//  * A float AtomicAdd is order-dependent: the result lies within the reassociation band the reference states for
//    its launched float scatter, |got - exact| <= gamma_(n-1) * sum|terms| with u = 2^-24 (f32) or 2^-53 (f64)
//    (kernel_parallel_float_scatter_band.rs:1-20, 102-107); it is exact on integer-valued data inside 2^24.
//  * Assign is declined, as the reference's launched lift declines it: with repeated targets its result depends on
//    the order of the stores.
// bincount (crates/unpopped/tests/kernel_bincount_agrees.rs:1-10) adds 1 to the I32 count of every in-range value.
#include "common.cuh"

#include <type_traits>

namespace up {
namespace sc {

constexpr int kThreads = 256;

template <typename T, int C>
__device__ __forceinline__ void combine_at(T* p, T v) {
  if constexpr (C == UP_COMBINE_ADD) {
    if constexpr (sizeof(T) == 8 && !std::is_floating_point<T>::value)
      atomicAdd(reinterpret_cast<unsigned long long*>(p), (unsigned long long)v);  // wraps like the i64 add
    else
      atomicAdd(p, v);
  } else if constexpr (C == UP_COMBINE_MAX) {
    if constexpr (sizeof(T) == 8)
      atomicMax(reinterpret_cast<long long*>(p), (long long)v);
    else
      atomicMax(p, v);
  } else {
    if constexpr (sizeof(T) == 8)
      atomicMin(reinterpret_cast<long long*>(p), (long long)v);
    else
      atomicMin(p, v);
  }
}

template <typename I>
__device__ __forceinline__ int64_t load_index(const I* ids, int64_t k) {
  return (int64_t)__ldg(ids + k);
}
template <>
__device__ __forceinline__ int64_t load_index<uint32_t>(const uint32_t* ids, int64_t k) {
  return (int64_t)(uint64_t)__ldg(ids + k);
}

// A warp per source row (grid-stride over rows), lanes over the columns. `ids_stride` is the index's row stride:
// cols for a full-shape index, 0 for an index_add (every lane reads the row's one index).
template <typename T, int C, typename I>
__global__ void __launch_bounds__(kThreads) scatter_kernel(const T* __restrict__ upd, int64_t n, int64_t cols,
                                                           int64_t upd_stride, const I* __restrict__ ids,
                                                           int64_t ids_stride, T* __restrict__ out, int64_t out_rows,
                                                           int64_t out_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * kThreads) >> 5;
  for (int64_t i = w0; i < n; i += nw) {
    for (int64_t j = lane; j < cols; j += 32) {
      const int64_t t = load_index(ids, ids_stride ? i * ids_stride + j : i);
      if (t < 0 || t >= out_rows) continue;  // Skip
      combine_at<T, C>(out + t * out_stride + j, __ldg(upd + i * upd_stride + j));
    }
  }
}

template <typename I>
__global__ void __launch_bounds__(kThreads) bincount_kernel(const I* __restrict__ x, int64_t n,
                                                            int32_t* __restrict__ counts, int64_t bins) {
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const int64_t v = load_index(x, i);
    if (v >= 0 && v < bins) atomicAdd(counts + v, 1);
  }
}

template <typename T, int C, typename I>
int launch(const void* upd, int64_t n, int64_t cols, int64_t upd_stride, const void* ids, int64_t ids_stride,
           void* out, int64_t out_rows, int64_t out_stride, cudaStream_t s) {
  const int64_t warps = n;
  int64_t g = (warps * 32 + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (g > cap) g = cap;
  scatter_kernel<T, C, I><<<(int)g, kThreads, 0, s>>>(static_cast<const T*>(upd), n, cols, upd_stride,
                                                      static_cast<const I*>(ids), ids_stride, static_cast<T*>(out),
                                                      out_rows, out_stride);
  note_launch();
  return check_launch();
}

template <typename T, typename I>
int launch_combine(int combine, const void* upd, int64_t n, int64_t cols, int64_t upd_stride, const void* ids,
                   int64_t ids_stride, void* out, int64_t out_rows, int64_t out_stride, cudaStream_t s) {
  if (combine == UP_COMBINE_ADD)
    return launch<T, UP_COMBINE_ADD, I>(upd, n, cols, upd_stride, ids, ids_stride, out, out_rows, out_stride, s);
  if constexpr (std::is_floating_point<T>::value) {
    return UP_ERR_UNSUPPORTED;  // float Max/Min: the reference's gate admits them for integers only
  } else {
    if (combine == UP_COMBINE_MAX)
      return launch<T, UP_COMBINE_MAX, I>(upd, n, cols, upd_stride, ids, ids_stride, out, out_rows, out_stride, s);
    return launch<T, UP_COMBINE_MIN, I>(upd, n, cols, upd_stride, ids, ids_stride, out, out_rows, out_stride, s);
  }
}

template <typename I>
int launch_dtype(int dtype, int combine, const void* upd, int64_t n, int64_t cols, int64_t upd_stride,
                 const void* ids, int64_t ids_stride, void* out, int64_t out_rows, int64_t out_stride,
                 cudaStream_t s) {
  switch (dtype) {
    case UP_EK_I32:
      return launch_combine<int32_t, I>(combine, upd, n, cols, upd_stride, ids, ids_stride, out, out_rows, out_stride, s);
    case UP_EK_U32:
      return launch_combine<uint32_t, I>(combine, upd, n, cols, upd_stride, ids, ids_stride, out, out_rows, out_stride,
                                         s);
    case UP_EK_I64:
      return launch_combine<int64_t, I>(combine, upd, n, cols, upd_stride, ids, ids_stride, out, out_rows, out_stride, s);
    case UP_EK_F32:
      return launch_combine<float, I>(combine, upd, n, cols, upd_stride, ids, ids_stride, out, out_rows, out_stride, s);
    case UP_EK_F64:
      return launch_combine<double, I>(combine, upd, n, cols, upd_stride, ids, ids_stride, out, out_rows, out_stride, s);
    default:
      return UP_ERR_UNSUPPORTED;
  }
}

}  // namespace sc
}  // namespace up

using namespace up;
using namespace up::sc;

extern "C" int up_sm100_scatter(const void* updates, int64_t n, int64_t cols, int64_t upd_stride, int dtype,
                                const void* ids, int index_dtype, int64_t ids_stride, int combine, void* out,
                                int64_t out_rows, int64_t out_stride, void* stream) {
  UP_CHECK_ARG(n >= 0 && cols >= 0 && out_rows >= 0 && upd_stride >= cols && out_stride >= cols);
  UP_CHECK_ARG(ids_stride == 0 || ids_stride >= cols);
  if (combine == UP_COMBINE_ASSIGN)
    return fail_with(UP_ERR_UNSUPPORTED, "scatter: Assign is not launched (repeated targets order the stores)");
  if (combine != UP_COMBINE_ADD && combine != UP_COMBINE_MAX && combine != UP_COMBINE_MIN) return UP_ERR_UNSUPPORTED;
  if (index_dtype != UP_EK_I32 && index_dtype != UP_EK_I64 && index_dtype != UP_EK_U32) return UP_ERR_UNSUPPORTED;
  if (n == 0 || cols == 0) return UP_OK;
  UP_CHECK_ARG(updates != nullptr && ids != nullptr && (out != nullptr || out_rows == 0));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (index_dtype == UP_EK_I32)
    return launch_dtype<int32_t>(dtype, combine, updates, n, cols, upd_stride, ids, ids_stride, out, out_rows,
                                 out_stride, s);
  if (index_dtype == UP_EK_I64)
    return launch_dtype<int64_t>(dtype, combine, updates, n, cols, upd_stride, ids, ids_stride, out, out_rows,
                                 out_stride, s);
  return launch_dtype<uint32_t>(dtype, combine, updates, n, cols, upd_stride, ids, ids_stride, out, out_rows,
                                out_stride, s);
}

extern "C" int up_sm100_bincount(const void* x, int64_t n, int index_dtype, int32_t* counts, int64_t bins,
                                 void* stream) {
  UP_CHECK_ARG(n >= 0 && bins >= 0);
  if (index_dtype != UP_EK_I32 && index_dtype != UP_EK_I64 && index_dtype != UP_EK_U32) return UP_ERR_UNSUPPORTED;
  if (n == 0 || bins == 0) return UP_OK;
  UP_CHECK_ARG(x != nullptr && counts != nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t g = (n + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (g > cap) g = cap;
  if (index_dtype == UP_EK_I32)
    bincount_kernel<int32_t><<<(int)g, kThreads, 0, s>>>(static_cast<const int32_t*>(x), n, counts, bins);
  else if (index_dtype == UP_EK_I64)
    bincount_kernel<int64_t><<<(int)g, kThreads, 0, s>>>(static_cast<const int64_t*>(x), n, counts, bins);
  else
    bincount_kernel<uint32_t><<<(int)g, kThreads, 0, s>>>(static_cast<const uint32_t*>(x), n, counts, bins);
  note_launch();
  return check_launch();
}

UP_DEFINE_REVISION(scatter)
