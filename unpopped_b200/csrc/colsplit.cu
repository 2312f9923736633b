// colsplit.cu — the split-K variant of the outer-axis Sum/Mean (crates/unpopped/ondevice/README.md:185-218,
// splitk_validate.cu:40-50): `_splitk_partial` folds each chunk of chunk_rows = ceil(rows / n_chunks) rows into a
// workspace, `_splitk_combine` adds the chunk partials in chunk order, seeded from the first partial. It is a
// different association than the serial fold (the reference's `VariantFidelity::ReassociatedDeterministic`):
// deterministic for a fixed n_chunks, no atomics, and with n_chunks = 1 the serial fold itself.
//
// Under this library's Auto policy the partials are f64 (each chunk's rows folded ascending from a 0.0 seed, as the
// serial fold is) and the combine is f64; Mean divides the total by the row count; one rounding to f32. The zero
// seed maps an all -0 column to +0, as the serial fold does (splitk_validate.cu:95-110).
#include "common.cuh"

namespace up {
namespace cs {

constexpr int kThreads = 256;

// partial[c][col] for chunk c = blockIdx.y; a thread folds 4 adjacent columns (16-byte loads) or one.
template <bool VEC>
__global__ void __launch_bounds__(kThreads) splitk_partial_kernel(const float* __restrict__ x, int64_t rows,
                                                                   int64_t cols, int64_t stride, int64_t chunk_rows,
                                                                   double* __restrict__ partial) {
  const int64_t c0 = ((int64_t)blockIdx.x * kThreads + threadIdx.x) * (VEC ? 4 : 1);
  if (c0 >= cols) return;
  const int64_t r0 = (int64_t)blockIdx.y * chunk_rows;
  const int64_t r1 = r0 + chunk_rows < rows ? r0 + chunk_rows : rows;
  double* out = partial + (int64_t)blockIdx.y * cols + c0;
  if (VEC) {
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
    int64_t r = r0;
    for (; r + 3 < r1; r += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = ld_nc_na_f4(x + (r + u) * stride + c0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a0 += (double)v[u].x;
        a1 += (double)v[u].y;
        a2 += (double)v[u].z;
        a3 += (double)v[u].w;
      }
    }
    for (; r < r1; ++r) {
      const float4 v = ld_nc_na_f4(x + r * stride + c0);
      a0 += (double)v.x;
      a1 += (double)v.y;
      a2 += (double)v.z;
      a3 += (double)v.w;
    }
    out[0] = a0;
    out[1] = a1;
    out[2] = a2;
    out[3] = a3;
  } else {
    double a = 0.0;
    int64_t r = r0;
    for (; r + 3 < r1; r += 4) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldg(x + (r + u) * stride + c0);
#pragma unroll
      for (int u = 0; u < 4; ++u) a += (double)v[u];
    }
    for (; r < r1; ++r) a += (double)__ldg(x + r * stride + c0);
    out[0] = a;
  }
}

template <bool MEAN>
__global__ void __launch_bounds__(kThreads) splitk_combine_kernel(const double* __restrict__ partial, int64_t cols,
                                                                   int64_t n_chunks, int64_t rows,
                                                                   float* __restrict__ out) {
  const int64_t c = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  double acc = partial[c];  // seeded from the first partial
  for (int64_t k = 1; k < n_chunks; ++k) acc += partial[k * cols + c];
  out[c] = __double2float_rn(MEAN ? acc / (double)rows : acc);
}

}  // namespace cs
}  // namespace up

using namespace up;

// The chunk count the kernels use for a requested one: at least 1, at most one chunk per row.
static int64_t effective_chunks(int64_t rows, int64_t n_chunks) {
  if (n_chunks > rows) n_chunks = rows;
  return n_chunks < 1 ? 1 : n_chunks;
}

extern "C" size_t up_sm100_col_sum_splitk_workspace_bytes(int64_t rows, int64_t cols, int64_t n_chunks) {
  if (rows < 0 || cols < 0 || n_chunks < 1) return 0;
  return sizeof(double) * (size_t)effective_chunks(rows, n_chunks) * (size_t)cols;
}

extern "C" int up_sm100_col_sum_f32_splitk(const float* x, int64_t rows, int64_t cols, int64_t row_stride,
                                           int64_t n_chunks, int mean, void* workspace, size_t workspace_bytes,
                                           float* out, void* stream) {
  UP_CHECK_ARG(rows >= 0 && cols >= 0 && row_stride >= cols && n_chunks >= 1);
  if (cols == 0) return UP_OK;
  UP_CHECK_ARG(out != nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {  // the empty fold: 0 (Mean: 0 / 0)
    if (!mean) return cuda_status(cudaMemsetAsync(out, 0, sizeof(float) * (size_t)cols, s));
  }
  UP_CHECK_ARG(x != nullptr || rows == 0);
  const int64_t nc = effective_chunks(rows, n_chunks);
  if (nc > 65535) return fail_with(UP_ERR_UNSUPPORTED, "col_sum_splitk: at most 65535 chunks");
  if (workspace_bytes < up_sm100_col_sum_splitk_workspace_bytes(rows, cols, n_chunks)) return UP_ERR_INVALID;
  UP_CHECK_ARG(workspace != nullptr && aligned(workspace, 8));
  double* partial = static_cast<double*>(workspace);
  if (rows > 0) {
    const int64_t chunk_rows = (rows + nc - 1) / nc;
    const bool vec = aligned(x, 16) && cols % 4 == 0 && row_stride % 4 == 0;
    const int64_t per_cta = vec ? 4 * cs::kThreads : cs::kThreads;
    const dim3 grid((unsigned)((cols + per_cta - 1) / per_cta), (unsigned)nc);
    if (vec) cs::splitk_partial_kernel<true><<<grid, cs::kThreads, 0, s>>>(x, rows, cols, row_stride, chunk_rows, partial);
    else cs::splitk_partial_kernel<false><<<grid, cs::kThreads, 0, s>>>(x, rows, cols, row_stride, chunk_rows, partial);
    note_launch();
  } else {
    const cudaError_t e = cudaMemsetAsync(partial, 0, sizeof(double) * (size_t)cols, s);  // one zero partial
    if (e != cudaSuccess) return cuda_status(e);
  }
  const unsigned g = (unsigned)((cols + cs::kThreads - 1) / cs::kThreads);
  if (mean) cs::splitk_combine_kernel<true><<<g, cs::kThreads, 0, s>>>(partial, cols, rows > 0 ? nc : 1, rows, out);
  else cs::splitk_combine_kernel<false><<<g, cs::kThreads, 0, s>>>(partial, cols, rows > 0 ? nc : 1, rows, out);
  note_launch();
  return check_launch();
}

UP_DEFINE_REVISION(colsplit)
