// gather.cu — row gather out[n, :] = table[ids[n], :] for sm_100a.
//
// Semantics: ReadIndex::Indexed on axis 0 with a 1-D index broadcast over the row
// (crates/unpopped/src/ir.rs:2620-2669, OpDef::gather/index_select/embedding :3838-3890) as the oracle
// evaluates it (crates/unpopped/src/oracle/plan_eval.rs:363-385): the index is read once; the load
// address is clamped to [0, V-1], so no out-of-range read is ever issued; an index outside [0, V) skips
// the store (Skip), writes zeros (ZeroFill) or stores the clamped row (Clamp). Rows move bit for bit.
//
// Layout: a warp owns 32 consecutive output rows at a time (a 16 KiB run of the output for bf16x256 rows): lane i
// reads index i of the run, and the warp then moves the rows UNROLL at a time, lane l carrying the 16-byte chunks
// l, l+32, ... of each row (a 512-byte row is exactly one chunk per lane), UNROLL rows' loads in flight before
// their stores. Table rows are read through L1 and L2 with the default policy (a Zipf index re-reads popular
// rows, which then hit in cache); output rows are written with evict-first stores so they do not displace table
// rows. The grid is many waves of CTAs, which evens out how long the Zipf-hot and cold runs take.
//
// Measured on the 2^24-id Zipf(1.1) configuration (8.6 GB written): this kernel 1.61-1.66 ms; a write-only pass
// over the same output bytes, 1.27 ms. Staging rows in shared memory did not help: one cp.async.bulk per 512-byte
// row with one bulk store per 16-row batch took 2.83 ms (the copy engine accepted about one row request per 48
// cycles per SM), and 16-byte cp.async loads with a bulk store per 32-row batch 1.79 ms. Eight or sixteen rows in
// flight per warp, L1 evict-last table loads and write-back output stores were all within 2 % of this kernel.
#include "common.cuh"

namespace up {

__device__ __forceinline__ int64_t read_index(const void* ids, int kind, int64_t i) {
  if (kind == UP_EK_I64) return __ldg(static_cast<const long long*>(ids) + i);
  if (kind == UP_EK_U32) return (int64_t)__ldg(static_cast<const unsigned int*>(ids) + i);
  return (int64_t)__ldg(static_cast<const int*>(ids) + i);
}

template <int UNROLL>
__global__ void __launch_bounds__(256) gather_rows_vec_kernel(const uint4* __restrict__ table, int64_t V,
                                                              int64_t row_vecs, const void* __restrict__ ids,
                                                              int kind, int64_t n, int oob,
                                                              uint4* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t tw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t hi = V > 0 ? V - 1 : 0;  // clamp bound of the load address; V itself bounds the range
  for (int64_t b0 = gw * 32; b0 < n; b0 += tw * 32) {
    const int64_t mine = (b0 + lane < n) ? read_index(ids, kind, b0 + lane) : 0;
    const int rows = (int)((n - b0) < 32 ? (n - b0) : 32);
    for (int q = 0; q < rows; q += UNROLL) {
      int64_t raw[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) raw[u] = __shfl_sync(0xffffffffu, mine, (q + u) & 31);
      for (int64_t c = lane; c < row_vecs; c += 32) {
        uint4 val[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          const int64_t g = raw[u] < 0 ? 0 : (raw[u] > hi ? hi : raw[u]);
          val[u] = (q + u < rows) ? __ldg(table + g * row_vecs + c) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          if (q + u >= rows) continue;
          const bool bad = raw[u] < 0 || raw[u] >= V;
          if (bad && oob == UP_OOB_SKIP) continue;
          st_cs_v4(out + (b0 + q + u) * row_vecs + c,
                   (bad && oob == UP_OOB_ZERO_FILL) ? make_uint4(0u, 0u, 0u, 0u) : val[u]);
        }
      }
    }
  }
}

// Any row size and alignment: one thread per output byte (or 4-byte word when both allow it).
template <typename W>
__global__ void gather_rows_any_kernel(const W* __restrict__ table, int64_t V, int64_t row_words,
                                       const void* __restrict__ ids, int kind, int64_t n, int oob,
                                       W* __restrict__ out) {
  const int64_t total = n * row_words;
  const int64_t hi = V > 0 ? V - 1 : 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / row_words, c = i - r * row_words;
    const int64_t raw = read_index(ids, kind, r);
    const int64_t g = raw < 0 ? 0 : (raw > hi ? hi : raw);
    const bool bad = raw < 0 || raw >= V;
    if (bad && oob == UP_OOB_SKIP) continue;
    out[i] = (bad && oob == UP_OOB_ZERO_FILL) ? W(0) : table[g * row_words + c];
  }
}

}  // namespace up

using namespace up;

extern "C" int up_sm100_gather_rows(const void* table, int64_t table_rows, int64_t row_bytes, const void* ids,
                                    int index_dtype, int64_t n, int oob, void* out, void* stream) {
  UP_CHECK_ARG(table_rows >= 0 && row_bytes >= 0 && n >= 0);
  if (index_dtype != UP_EK_I32 && index_dtype != UP_EK_I64 && index_dtype != UP_EK_U32) return UP_ERR_UNSUPPORTED;
  if (oob != UP_OOB_SKIP && oob != UP_OOB_CLAMP && oob != UP_OOB_ZERO_FILL) return UP_ERR_UNSUPPORTED;
  if (n == 0 || row_bytes == 0) return UP_OK;
  UP_CHECK_ARG(ids != nullptr && out != nullptr);
  // An empty table has no row to clamp to: only ZeroFill and Skip have a defined result.
  if (table_rows == 0 && oob == UP_OOB_CLAMP) return UP_ERR_OOB;
  UP_CHECK_ARG(table != nullptr || table_rows == 0);
  // With no table every index is out of range: the (clamped) load reads the output's first row instead and
  // its value is never stored.
  const void* tab = table_rows == 0 ? out : table;
  const int64_t V = table_rows;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int sms = sm_count();
  if (row_bytes % 16 == 0 && aligned(table, 16) && aligned(out, 16)) {
    const int64_t row_vecs = row_bytes / 16;
    constexpr int kUnroll = 4;
    const int64_t warps_needed = (n + 31) / 32;  // a warp per run of 32 rows
    int64_t blocks = (warps_needed + 7) / 8;
    const int64_t cap = (int64_t)sms * 64;      // many waves: the Zipf-hot and cold runs even out
    if (blocks > cap) blocks = cap;
    gather_rows_vec_kernel<kUnroll><<<(int)blocks, 256, 0, s>>>(static_cast<const uint4*>(tab), V, row_vecs, ids,
                                                               index_dtype, n, oob, static_cast<uint4*>(out));
  } else {
    const bool words = row_bytes % 4 == 0 && aligned(table, 4) && aligned(out, 4);
    const int64_t rw = words ? row_bytes / 4 : row_bytes;
    int64_t blocks = (n * rw + 255) / 256;
    const int64_t cap = (int64_t)sms * 16;
    if (blocks > cap) blocks = cap;
    if (words)
      gather_rows_any_kernel<uint32_t><<<(int)blocks, 256, 0, s>>>(static_cast<const uint32_t*>(tab), V, rw, ids,
                                                                   index_dtype, n, oob, static_cast<uint32_t*>(out));
    else
      gather_rows_any_kernel<uint8_t><<<(int)blocks, 256, 0, s>>>(static_cast<const uint8_t*>(tab), V, rw, ids,
                                                                  index_dtype, n, oob, static_cast<uint8_t*>(out));
  }
  note_launch();
  return check_launch();
}

UP_DEFINE_REVISION(gather)
