// reduce.cu — row reductions for sm_100a: f32 row sum (two accumulation policies), bf16 row max + argmax,
// and the whole-array int32 fold used as the first pass of a scan sharded over GPUs.
//
// Semantics follow the reference oracle (crates/unpopped/src/oracle/plan_eval.rs:501-651 and
// oracle/plan_contract.rs:146-245). All kernels are HBM-streaming: 128-bit loads through the read-only
// path with no L1 allocation, fixed-order warp/block combines, one CTA per row.
#include "common.cuh"
#include "spec.cuh"

#include <algorithm>

#include <cuda_bf16.h>

namespace up {

// ===================================================================================================
// Row sum, UP_ACCUM_F32: f32 accumulation in a fixed tree order.
//
// Order (deterministic, independent of the grid): thread t of 256 reads float4 number t + 256*j. Each
// group of 8 float4 a thread reads is summed as a balanced tree (the four lanes of a float4 pairwise,
// then the eight float4 pairwise); successive groups add sequentially. The 32 lanes of a warp combine
// by an xor butterfly and the 8 warps by a balanced tree. For cols <= 8192 the depth is 13 roundings, so
// |got - exact| <= gamma_13 * sum|x| < 2^-20 * sum|x| with u = 2^-24.
// ===================================================================================================
constexpr int kRowThreads = 256;

__device__ __forceinline__ float warp_sum_butterfly(float a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = a + __shfl_xor_sync(0xffffffffu, a, o);
  return a;
}

template <bool VEC>
__global__ void __launch_bounds__(kRowThreads) row_sum_f32_kernel(const float* __restrict__ x, int64_t rows,
                                                                   int64_t cols, int64_t stride,
                                                                   float* __restrict__ out) {
  __shared__ float warp_part[kRowThreads / 32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* row = x + r * stride;
    float acc = 0.0f;
    bool first = true;
    if (VEC) {
      const int64_t nv = cols >> 2;
      for (int64_t base = threadIdx.x; base < nv; base += kRowThreads * 8) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int64_t i = base + (int64_t)u * kRowThreads;
          v[u] = i < nv ? ld_nc_na_f4(row + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float s[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) s[u] = (v[u].x + v[u].y) + (v[u].z + v[u].w);
        const float g = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
        acc = first ? g : acc + g;
        first = false;
      }
    } else {
      for (int64_t base = threadIdx.x; base < cols; base += kRowThreads * 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int64_t i = base + (int64_t)u * kRowThreads;
          v[u] = i < cols ? __ldg(row + i) : 0.0f;
        }
        const float g = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
        acc = first ? g : acc + g;
        first = false;
      }
    }
    acc = warp_sum_butterfly(acc);
    if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      const float* w = warp_part;
      out[r] = ((w[0] + w[1]) + (w[2] + w[3])) + ((w[4] + w[5]) + (w[6] + w[7]));
    }
    __syncthreads();
  }
}

// ===================================================================================================
// Row sum, UP_ACCUM_AUTO: the launched lift's documented f64 order for a logical block of B threads
// (crates/unpopped/src/kernel_lift/block_reduce.rs:13-23): logical thread t folds t, t+B, t+2B, ...
// ascending into an f64; then acc[t] += acc[t+s] for s = B/2 .. 1; one rounding to f32.
//
// A physical thread holds V logical threads: with V = 4 it reads the float4 at 4p + jB, whose four
// lanes belong to logical threads 4p .. 4p+3 (B is a multiple of 4), so each logical thread still folds
// its own elements in ascending order. The tree runs literally, level by level, in shared memory.
// ===================================================================================================
template <int V>
__global__ void row_sum_auto_kernel(const float* __restrict__ x, int64_t rows, int64_t cols, int64_t stride,
                                    int B, bool mean, float* __restrict__ out) {
  extern __shared__ double sacc[];  // [rows per CTA][B]
  const int P = B / V;
  const int rpc = blockDim.x / P;
  const int lr = threadIdx.x / P;
  const int p = threadIdx.x - lr * P;
  double* s = sacc + (size_t)lr * B;
  for (int64_t r0 = (int64_t)blockIdx.x * rpc; r0 < rows; r0 += (int64_t)gridDim.x * rpc) {
    const int64_t r = r0 + lr;
    double acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0.0;
    if (lr < rpc && r < rows) {
      const float* row = x + r * stride;
      if (V == 4) {
        for (int64_t c = 4 * (int64_t)p; c < cols; c += B) {
          const float4 f = ld_nc_na_f4(row + c);
          acc[0] += (double)f.x;
          acc[V > 1 ? 1 : 0] += (double)f.y;
          acc[V > 2 ? 2 : 0] += (double)f.z;
          acc[V > 3 ? 3 : 0] += (double)f.w;
        }
      } else {
        for (int64_t c = p; c < cols; c += B) acc[0] += (double)__ldg(row + c);
      }
    }
    if (lr < rpc) {
#pragma unroll
      for (int v = 0; v < V; ++v) s[V * p + v] = acc[v];
    }
    __syncthreads();
    for (int st = B >> 1; st > 0; st >>= 1) {
      if (lr < rpc)
        for (int t = p; t < st; t += P) s[t] += s[t + st];
      __syncthreads();
    }
    // Mean divides the f64 total by the extent before the one rounding (block_reduce.rs:13-23)
    if (lr < rpc && p == 0 && r < rows) out[r] = __double2float_rn(mean ? s[0] / (double)cols : s[0]);
    __syncthreads();
  }
}

// ===================================================================================================
// Row sum, UP_ACCUM_AUTO at block 1: the serial order, which is the plan oracle's fold (plan_eval.rs:566-645),
// s = ((0 + x0) + x1) + ... in f64 with one rounding, by the chunk rule of spec.cuh. A warp takes a row, 32 chunks
// (2,048 values) at a time, lane l summarising chunk l from contiguous loads. If |s| plus the sum of the segment's
// H (both sums rounded up) is below min(lim, the smallest L of the segment), every partial sum of the fold over the
// segment (at most |s| + the H of the chunks so far) is exact, and s += the warp sum of its T (exact in any order).
// Otherwise the warp walks the segment's chunks in order, each lane's summary passed by shuffles, and folds the
// chunks that may round value by value (the warp loads the chunk, two values a lane, and adds them in order). s
// and lim are the same in every lane of the warp. A float4 lane loads its chunk in two halves, which fits three CTAs
// an SM (79 registers) and keeps more warps' loads in flight.
// ===================================================================================================
template <bool MEAN, bool VEC>
__global__ void __launch_bounds__(256, VEC ? 3 : 2) row_sum_serial_spec_kernel(const float* __restrict__ x, int64_t rows,
                                                                  int64_t cols, int64_t stride,
                                                                  float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = w0; r < rows; r += nw) {
    const float* __restrict__ row = x + r * stride;
    double s = 0.0, lim = f64_inf();
    for (int64_t c0 = 0; c0 < cols; c0 += 32 * kSpecChunk) {
      const int64_t cb = c0 + (int64_t)kSpecChunk * lane;
      double pre = 0.0, hi = 0.0;
      uint32_t mn = 0xffffffffu;
      if (VEC && cb + kSpecChunk <= cols) {
#pragma unroll 1
        for (int h0 = 0; h0 < kSpecChunk / 4; h0 += 8) {  // two halves of 8 float4
          float4 v[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) v[k] = ld_nc_na_f4(row + cb + 4 * (h0 + k));
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            spec_acc(v[k].x, pre, hi, mn);
            spec_acc(v[k].y, pre, hi, mn);
            spec_acc(v[k].z, pre, hi, mn);
            spec_acc(v[k].w, pre, hi, mn);
          }
        }
      } else {
        float v[kSpecChunk];
#pragma unroll
        for (int k = 0; k < kSpecChunk; ++k) v[k] = cb + k < cols ? __ldg(row + cb + k) : 0.f;
#pragma unroll
        for (int k = 0; k < kSpecChunk; ++k) spec_acc(v[k], pre, hi, mn);
      }
      double lc;
      float h;
      spec_finish(pre, hi, mn, lc, h);
      double hs = (double)h, ml = lc, ts = pre;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        hs = __dadd_ru(hs, __shfl_xor_sync(0xffffffffu, hs, o));
        ml = fmin(ml, __shfl_xor_sync(0xffffffffu, ml, o));
        ts += __shfl_xor_sync(0xffffffffu, ts, o);
      }
      hs = __shfl_sync(0xffffffffu, hs, 0);  // lane 0's values decide for the whole warp
      ml = __shfl_sync(0xffffffffu, ml, 0);
      ts = __shfl_sync(0xffffffffu, ts, 0);
      const double l2 = fmin(lim, ml);
      if (__dadd_ru(fabs(s), hs) < l2) {
        s += ts;
        lim = l2;
      } else {
        const int nch = (int)min((int64_t)32, (cols - c0 + kSpecChunk - 1) / kSpecChunk);
        for (int j = 0; j < nch; ++j) {
          const double tj = __shfl_sync(0xffffffffu, pre, j), lj = __shfl_sync(0xffffffffu, lc, j);
          const float hj = __shfl_sync(0xffffffffu, h, j);
          lim = fmin(lim, lj);
          if (fabs(s) + (double)hj < lim) {
            s += tj;
          } else {
            const int64_t rb = c0 + (int64_t)kSpecChunk * j;
            const float a = rb + lane < cols ? __ldg(row + rb + lane) : 0.f;
            const float b = rb + 32 + lane < cols ? __ldg(row + rb + 32 + lane) : 0.f;
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const float v = __shfl_sync(0xffffffffu, a, k);
              if (rb + k < cols) s += (double)v;
            }
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const float v = __shfl_sync(0xffffffffu, b, k);
              if (rb + 32 + k < cols) s += (double)v;
            }
            lim = spec_anchor(s);
          }
        }
      }
    }
    if (lane == 0) out[r] = __double2float_rn(MEAN ? s / (double)cols : s);
  }
}

// ===================================================================================================
// Row max + argmax over bf16 (oracle/plan_contract.rs:179-245).
//
// Key: a bf16 maps to a 16-bit unsigned key that orders like the reference's total order for ArgMax:
// every NaN is the greatest value (key 0xffff), -0 equals +0, and otherwise the numeric order. The
// argmax is the first index of the greatest key. Ties resolve to the lower index because the packed
// word (key << 16) | (0xffff - index) is combined with max, which is associative and commutative, so
// the block's combine order cannot change the answer.
// The f32 max is the bf16 at the argmax (the first of equal maxima, so the first zero's sign) when the
// row has no NaN; with a NaN it is the row's LAST NaN widened with the quiet bit set, which is what the
// Max fold (take = !have || v is NaN || v > acc) and the reference's f32->f64->f32 conversions give.
// ===================================================================================================
__device__ __forceinline__ uint32_t bf16_key(uint32_t b) {
  b &= 0xffffu;
  if ((b & 0x7fffu) > 0x7f80u) return 0xffffu;
  if (b == 0x8000u) b = 0;
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}

__device__ __forceinline__ bool bf16_isnan(uint32_t b) { return (b & 0x7fffu) > 0x7f80u; }

// Block-wide max of an unsigned 64-bit word (all threads get it).
__device__ __forceinline__ uint64_t block_max_u64(uint64_t v, uint64_t* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  uint64_t m = sm[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) m = sm[i] > m ? sm[i] : m;
  __syncthreads();
  return m;
}

__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, uint32_t* sm) {
  v = __reduce_max_sync(0xffffffffu, v);
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t m = sm[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) m = sm[i] > m ? sm[i] : m;
  __syncthreads();
  return m;
}

// Writes the outputs of one row from its argmax and whether it holds a NaN.
__device__ __forceinline__ void write_max_argmax(const uint16_t* row, int64_t r, int64_t arg, uint32_t max_bits,
                                                 float* max_out, int32_t* am32, int64_t* am64) {
  if (max_out) max_out[r] = __uint_as_float(max_bits);
  if (am32) am32[r] = (int32_t)arg;
  if (am64) am64[r] = arg;
}

// Fast path: rows of at most 65536 elements, cols % 8 == 0, 16-byte aligned rows. One streaming pass: for
// every 16-byte word (8 bf16) a thread takes the NaN-propagating max with packed bf16x2 instructions and
// keeps the first word whose max has the greatest key; at the end it re-reads that one word to find the
// first element with that key. The block then combines the packed (key, index) words.
__device__ __forceinline__ uint32_t word_max_bits(uint4 w) {
  const __nv_bfloat162 a = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162*>(&w.x),
                                       *reinterpret_cast<const __nv_bfloat162*>(&w.y));
  const __nv_bfloat162 b = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162*>(&w.z),
                                       *reinterpret_cast<const __nv_bfloat162*>(&w.w));
  const __nv_bfloat162 m = __hmax2_nan(a, b);
  return __bfloat16_as_ushort(__hmax_nan(__low2bfloat16(m), __high2bfloat16(m)));
}

template <int UNROLL>
__global__ void __launch_bounds__(kRowThreads) row_max_argmax_vec_kernel(const uint16_t* __restrict__ x,
                                                                         int64_t rows, int64_t cols,
                                                                         int64_t stride, float* max_out,
                                                                         int32_t* am32, int64_t* am64) {
  __shared__ uint32_t sm32[kRowThreads / 32];
  const int nvec = (int)(cols >> 3);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint16_t* row = x + r * stride;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    uint32_t best_key = 0;
    int best_word = -1;
    uint4 best_w = make_uint4(0u, 0u, 0u, 0u);  // the best word's bits, kept so the row is never re-read
    for (int i0 = threadIdx.x; i0 < nvec; i0 += kRowThreads * UNROLL) {
      uint4 w[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int i = i0 + u * kRowThreads;
        w[u] = i < nvec ? ld_nc_na_v4(rv + i) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int i = i0 + u * kRowThreads;
        if (i < nvec) {
          const uint32_t key = bf16_key(word_max_bits(w[u]));
          if (best_word < 0 || key > best_key) {
            best_key = key;
            best_word = i;
            best_w = w[u];
          }
        }
      }
    }
    uint32_t packed = 0, my_bits = 0;
    if (best_word >= 0) {
      const uint32_t q[4] = {best_w.x, best_w.y, best_w.z, best_w.w};
      int e = 0;
#pragma unroll
      for (int j = 7; j >= 0; --j)
        if (bf16_key((q[j >> 1] >> ((j & 1) * 16)) & 0xffffu) == best_key) e = j;
      const uint32_t idx = (uint32_t)(8 * best_word + e);
      packed = (best_key << 16) | (0xffffu - idx);
      my_bits = (q[e >> 1] >> ((e & 1) * 16)) & 0xffffu;
    }
    const uint32_t best = block_max_u32(packed, sm32);
    const uint32_t key = best >> 16;
    const int64_t arg = cols > 0 ? (int64_t)(0xffffu - (best & 0xffffu)) : 0;
    if (key == 0xffffu) {
      // NaN row: the max is the last NaN (rare; re-read the row).
      uint32_t last = 0;
      for (int64_t i = threadIdx.x; i < cols; i += kRowThreads)
        if (bf16_isnan(row[i])) last = (uint32_t)i + 1;
      last = block_max_u32(last, sm32);
      if (threadIdx.x == 0)
        write_max_argmax(row, r, arg, ((uint32_t)row[last - 1] << 16) | 0x00400000u, max_out, am32, am64);
    } else if (best_word >= 0 && packed == best) {
      // exactly one thread holds the winning (key, index): it writes from its own registers
      write_max_argmax(row, r, arg, my_bits << 16, max_out, am32, am64);
    }
  }
}

// General path: any cols, any alignment; 64-bit packed (key << 32) | (0xffffffff - index).
__global__ void __launch_bounds__(kRowThreads) row_max_argmax_any_kernel(const uint16_t* __restrict__ x,
                                                                         int64_t rows, int64_t cols,
                                                                         int64_t stride, float* max_out,
                                                                         int32_t* am32, int64_t* am64) {
  __shared__ uint64_t sm64[kRowThreads / 32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint16_t* row = x + r * stride;
    uint64_t best = 0, last = 0;
    for (int64_t i = threadIdx.x; i < cols; i += kRowThreads) {
      const uint32_t b = __ldg(row + i);
      const uint64_t cand = ((uint64_t)bf16_key(b) << 32) | (0xffffffffull - (uint64_t)i);
      best = cand > best ? cand : best;
      if (bf16_isnan(b)) last = (uint64_t)i + 1;
    }
    best = block_max_u64(best, sm64);
    last = block_max_u64(last, sm64);
    const int64_t arg = cols > 0 ? (int64_t)(0xffffffffull - (best & 0xffffffffull)) : 0;
    uint32_t max_bits = 0;
    if (cols > 0) max_bits = last ? (((uint32_t)row[last - 1] << 16) | 0x00400000u) : ((uint32_t)row[arg] << 16);
    if (threadIdx.x == 0) write_max_argmax(row, r, arg, max_bits, max_out, am32, am64);
  }
}

// ===================================================================================================
// Whole-array int32 fold (SUM wrapping, MAX, MIN). Integer combines are exact, associative and
// commutative, so per-CTA atomics give a deterministic value. CTAs take their chunks from the END of
// the array: a scan that follows this pass on the same shard starts at the beginning, which is then the
// most recently read data and partly still in L2.
// ===================================================================================================
__device__ __forceinline__ int32_t i32_identity(int op) {
  return op == UP_OP_SUM ? 0 : (op == UP_OP_MAX ? INT32_MIN : INT32_MAX);
}

template <int OP>
__device__ __forceinline__ int32_t comb_i32(int32_t a, int32_t b) {
  if (OP == UP_OP_SUM) return (int32_t)((uint32_t)a + (uint32_t)b);
  if (OP == UP_OP_MAX) return a > b ? a : b;
  return a < b ? a : b;
}

__global__ void reduce_i32_init_kernel(int32_t* total, int op) { *total = i32_identity(op); }

template <int OP>
__global__ void __launch_bounds__(256) reduce_i32_kernel(const int32_t* __restrict__ x, int64_t n,
                                                         int32_t* total, bool vec) {
  __shared__ int32_t part[8];
  int32_t acc = i32_identity(OP);
  const int64_t chunk = 256 * 4 * 8;  // elements per CTA step
  const int64_t nchunks = (n + chunk - 1) / chunk;
  for (int64_t cb = blockIdx.x; cb < nchunks; cb += gridDim.x) {
    const int64_t c = nchunks - 1 - cb;
    const int64_t lo = c * chunk;
    if (vec && lo + chunk <= n) {
      const int4* p = reinterpret_cast<const int4*>(x + lo);
      int4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        uint4 t = ld_nc_na_v4(p + u * 256 + threadIdx.x);
        v[u] = make_int4((int)t.x, (int)t.y, (int)t.z, (int)t.w);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        acc = comb_i32<OP>(acc, comb_i32<OP>(comb_i32<OP>(v[u].x, v[u].y), comb_i32<OP>(v[u].z, v[u].w)));
    } else {
      for (int64_t i = lo + threadIdx.x; i < lo + chunk && i < n; i += 256) acc = comb_i32<OP>(acc, x[i]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = comb_i32<OP>(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t a = part[0];
    for (int i = 1; i < 8; ++i) a = comb_i32<OP>(a, part[i]);
    if (OP == UP_OP_SUM) atomicAdd(total, a);
    else if (OP == UP_OP_MAX) atomicMax(total, a);
    else atomicMin(total, a);
  }
}

}  // namespace up

using namespace up;

// The Auto row sum (documented f64 order of a logical block of B threads); with `mean` it divides by cols before
// the one rounding.
static int launch_row_sum_auto(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int block, bool mean,
                               float* out, cudaStream_t s) {
  if (block < 1 || block > 1024 || (block & (block - 1)) != 0) return UP_ERR_UNSUPPORTED;
  const bool vec = aligned(x, 16) && (cols % 4 == 0) && (row_stride % 4 == 0);
  if (block == 1) {  // the serial order: a warp per row
    const int64_t g = std::min<int64_t>((rows + 7) / 8, (int64_t)sm_count() * 16);
    if (vec)
      mean ? row_sum_serial_spec_kernel<true, true><<<(int)g, 256, 0, s>>>(x, rows, cols, row_stride, out)
           : row_sum_serial_spec_kernel<false, true><<<(int)g, 256, 0, s>>>(x, rows, cols, row_stride, out);
    else
      mean ? row_sum_serial_spec_kernel<true, false><<<(int)g, 256, 0, s>>>(x, rows, cols, row_stride, out)
           : row_sum_serial_spec_kernel<false, false><<<(int)g, 256, 0, s>>>(x, rows, cols, row_stride, out);
  } else if (vec && block >= 4) {
    const int P = block / 4, threads = 256, rpc = threads / P;
    const int64_t g = (rows + rpc - 1) / rpc;
    const size_t smem = (size_t)rpc * block * sizeof(double);
    row_sum_auto_kernel<4><<<(int)(g < (1 << 30) ? g : (1 << 30)), threads, smem, s>>>(x, rows, cols, row_stride,
                                                                                       block, mean, out);
  } else {
    const int threads = block > 256 ? block : 256, rpc = threads / block;
    const int64_t g = (rows + rpc - 1) / rpc;
    const size_t smem = (size_t)rpc * block * sizeof(double);
    row_sum_auto_kernel<1><<<(int)(g < (1 << 30) ? g : (1 << 30)), threads, smem, s>>>(x, rows, cols, row_stride,
                                                                                       block, mean, out);
  }
  return UP_OK;
}

namespace up {
int row_mean_f32_auto(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int block, float* out,
                      void* stream) {
  if (rows == 0) return UP_OK;
  const int st = launch_row_sum_auto(x, rows, cols, row_stride, block, true, out, static_cast<cudaStream_t>(stream));
  if (st != UP_OK) return st;
  note_launch();
  return check_launch();
}
}  // namespace up

extern "C" int up_sm100_row_sum_f32(const float* x, int64_t rows, int64_t cols, int64_t row_stride, float* out,
                                    int accum, int block, void* stream) {
  UP_CHECK_ARG(rows >= 0 && cols >= 0 && row_stride >= cols);
  if (rows == 0) return UP_OK;
  UP_CHECK_ARG(x != nullptr || cols == 0);
  UP_CHECK_ARG(out != nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = (int)(rows < (1 << 30) ? rows : (1 << 30));
  const bool vec = aligned(x, 16) && (cols % 4 == 0) && (row_stride % 4 == 0);
  if (accum == UP_ACCUM_F32) {
    if (vec) row_sum_f32_kernel<true><<<grid, kRowThreads, 0, s>>>(x, rows, cols, row_stride, out);
    else row_sum_f32_kernel<false><<<grid, kRowThreads, 0, s>>>(x, rows, cols, row_stride, out);
  } else if (accum == UP_ACCUM_AUTO) {
    const int st = launch_row_sum_auto(x, rows, cols, row_stride, block, false, out, s);
    if (st != UP_OK) return st;
  } else {
    return UP_ERR_UNSUPPORTED;
  }
  note_launch();
  return check_launch();
}

extern "C" int up_sm100_row_max_argmax_bf16(const uint16_t* x, int64_t rows, int64_t cols, int64_t row_stride,
                                            float* max_out, int32_t* argmax_i32, int64_t* argmax_i64,
                                            void* stream) {
  UP_CHECK_ARG(rows >= 0 && cols >= 0 && row_stride >= cols);
  if (rows == 0) return UP_OK;
  UP_CHECK_ARG(x != nullptr || cols == 0);
  UP_CHECK_ARG(max_out || argmax_i32 || argmax_i64);
  if (argmax_i32 && cols > (int64_t)INT32_MAX) return UP_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = (int)(rows < (1 << 30) ? rows : (1 << 30));
  const bool vec = cols > 0 && aligned(x, 16) && (cols % 8 == 0) && (row_stride % 8 == 0) && cols <= 65536;
  if (vec)
    row_max_argmax_vec_kernel<4><<<grid, kRowThreads, 0, s>>>(x, rows, cols, row_stride, max_out, argmax_i32,
                                                              argmax_i64);
  else
    row_max_argmax_any_kernel<<<grid, kRowThreads, 0, s>>>(x, rows, cols, row_stride, max_out, argmax_i32,
                                                          argmax_i64);
  note_launch();
  return check_launch();
}

extern "C" int up_sm100_reduce_i32(const int32_t* x, int64_t n, int op, int32_t* total, void* stream) {
  UP_CHECK_ARG(n >= 0 && total != nullptr && (x != nullptr || n == 0));
  if (op != UP_OP_SUM && op != UP_OP_MAX && op != UP_OP_MIN) return UP_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  reduce_i32_init_kernel<<<1, 1, 0, s>>>(total, op);
  note_launch();
  if (n > 0) {
    const bool vec = aligned(x, 16);
    const int64_t chunks = (n + 8191) / 8192;
    const int64_t cap = (int64_t)sm_count() * 8;
    const int grid = (int)(chunks < cap ? chunks : cap);
    if (op == UP_OP_SUM) reduce_i32_kernel<UP_OP_SUM><<<grid, 256, 0, s>>>(x, n, total, vec);
    else if (op == UP_OP_MAX) reduce_i32_kernel<UP_OP_MAX><<<grid, 256, 0, s>>>(x, n, total, vec);
    else reduce_i32_kernel<UP_OP_MIN><<<grid, 256, 0, s>>>(x, n, total, vec);
    note_launch();
  }
  return check_launch();
}

UP_DEFINE_REVISION(reduce)
