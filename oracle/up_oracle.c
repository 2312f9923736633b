/*
 * up_oracle.c — CPU restatement of the reference oracle for the lifted kernel families.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker the GPU kernels are compared against (and, timed on
 * the host cores, the reported CPU baseline). Nothing in the product library links, loads or calls it.
 *
 * Each function states the reference code it restates (paths relative to the Unpopped repository).
 * The reference oracle is Rust and cannot be built in this environment, so parity is pinned by running
 * these functions on the reference tests' own corpora and comparing with the expectations those tests
 * compute independently of the oracle (tests/golden/, made by tests/golden/make_golden.py).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp, the strict-FP flags of the reference's C
 * test support, crates/unpopped-cpu-c/tests/support/cc.rs:122-175).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_OP_SUM 0
#define ORC_OP_MAX 2
#define ORC_OP_MIN 3
#define ORC_OOB_SKIP 0
#define ORC_OOB_CLAMP 1
#define ORC_OOB_ZERO_FILL 2
#define ORC_EK_I32 9
#define ORC_EK_I64 10
#define ORC_EK_U32 23

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint64_t f64_bits(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }

/* ---- codecs: crates/unpopped/src/oracle/float_codec.rs, expr_eval.rs ---------------------------- */

/* bf16_to_f64 (float_codec.rs:200-203): bf16 is the top half of an f32. */
double orc_bf16_to_f64(uint16_t b) { return (double)bits_f32((uint32_t)b << 16); }

/* f32_to_bf16_bits (float_codec.rs:260-268): RNE; a NaN keeps its top half and is made quiet. */
uint16_t orc_f32_to_bf16(float x) {
  uint32_t bits = f32_bits(x);
  if (x != x) return (uint16_t)((bits >> 16) | 0x0040);
  uint32_t bias = 0x7fff + ((bits >> 16) & 1);
  return (uint16_t)((bits + bias) >> 16);
}

/* f32_to_f16_bits (float_codec.rs:205-258): RNE with subnormals, overflow to inf, quiet NaN. */
uint16_t orc_f32_to_f16(float x) {
  uint32_t bits = f32_bits(x);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
  int32_t exp = (int32_t)((bits >> 23) & 0xff);
  uint32_t mant = bits & 0x007fffff;
  if (exp == 0xff) return mant ? (uint16_t)(sign | 0x7e00) : (uint16_t)(sign | 0x7c00);
  int32_t e = exp - 127 + 15;
  if (e >= 0x1f) return (uint16_t)(sign | 0x7c00);
  if (e <= 0) {
    if (e < -10) return sign;
    uint32_t m = mant | 0x00800000;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t half = 1u << (shift - 1), mask = (1u << shift) - 1;
    uint32_t rem = m & mask, r = m >> shift;
    if (rem > half || (rem == half && (r & 1))) r += 1;
    return (uint16_t)(sign | r);
  }
  uint32_t half = 1u << 12, mask = (1u << 13) - 1;
  uint32_t rem = mant & mask, m10 = mant >> 13;
  int32_t ee = e;
  if (rem > half || (rem == half && (m10 & 1))) {
    m10 += 1;
    if (m10 == 0x400) {
      m10 = 0;
      ee += 1;
      if (ee >= 0x1f) return (uint16_t)(sign | 0x7c00);
    }
  }
  return (uint16_t)(sign | ((uint32_t)ee << 10) | m10);
}

/* IEEE binary16 decode (the inverse of the encoder above; exact in f64), by bit assembly. */
double orc_f16_to_f64(uint16_t h) {
  uint64_t s = (uint64_t)(h >> 15) << 63;
  uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff;
  uint64_t bits;
  if (e == 0) {
    double v = (double)m * (1.0 / 16777216.0); /* m * 2^-24, exact */
    return s ? -v : v;
  }
  if (e == 0x1f) bits = s | 0x7ff0000000000000ull | ((uint64_t)m << 42) | (m ? 0x0008000000000000ull : 0);
  else bits = s | ((uint64_t)(e - 15 + 1023) << 52) | ((uint64_t)m << 42);
  double d;
  memcpy(&d, &bits, 8);
  return d;
}

/* f64_to_f32_odd (expr_eval.rs:498-512): round to odd, so a later 16-bit rounding is single. */
float orc_f64_to_f32_odd(double f) {
  float r = (float)f;
  if (!isfinite(f) || f == 0.0 || (double)r == f) return r;
  uint32_t b = f32_bits(r);
  float t = (fabs((double)r) > fabs(f)) ? bits_f32(b - 1) : r;
  return bits_f32(f32_bits(t) | 1u);
}

/* encode_float(f, Bf16) (expr_eval.rs:520-530): odd-rounded f32, then RNE to bf16. */
uint16_t orc_f64_to_bf16(double f) { return orc_f32_to_bf16(orc_f64_to_f32_odd(f)); }

/* ---- reductions: oracle/plan_eval.rs:501-651, plan_contract.rs:146-245 ---------------------------- */

/* Float Sum over the last axis: f64 accumulator from 0, ascending index (fold_step,
 * plan_contract.rs:146-156), one rounding to f32 at the store (store_val / encode_float, F32 arm). */
void orc_row_sum_f32(const float* x, int64_t rows, int64_t cols, int64_t row_stride, float* out,
                     int threads) {
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
  for (int64_t r = 0; r < rows; ++r) {
    double acc = 0.0;
    const float* row = x + r * row_stride;
    for (int64_t c = 0; c < cols; ++c) acc += (double)row[c];
    out[r] = (float)acc;
  }
}

/* The launched lift's documented order (kernel_lift/block_reduce.rs:13-23; restated in the reference
 * test crates/unpopped/tests/kernel_parallel_reduction_float_sum_bound.rs:147-170, `documented`):
 * logical thread t < B folds t, t+B, ... ascending into an f64; then acc[t] += acc[t+s] for
 * s = B/2 .. 1; one rounding to f32. B is a power of two. */
void orc_row_sum_f32_documented(const float* x, int64_t rows, int64_t cols, int64_t row_stride,
                                int64_t block, float* out, int threads) {
#pragma omp parallel num_threads(threads) if (threads > 1)
  {
    double* acc = (double*)malloc(sizeof(double) * (size_t)block);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      const float* row = x + r * row_stride;
      for (int64_t t = 0; t < block; ++t) {
        double a = 0.0;
        for (int64_t c = t; c < cols; c += block) a += (double)row[c];
        acc[t] = a;
      }
      for (int64_t s = block / 2; s > 0; s /= 2)
        for (int64_t t = 0; t < s; ++t) acc[t] += acc[t + s];
      out[r] = (float)acc[0];
    }
    free(acc);
  }
}

/* Window pooling (Access::Window; the oracle's eval_window, oracle/plan_window.rs:249-475) along the middle axis of
 * a dense [outer, k_in, inner] input into [outer, k_out, inner]: output o folds the taps
 * p = o*stride - pad_lo + kk*dilation (kk ascending) inside [0, k_in). f32 (dtype 2): Sum/Mean in f64, Mean over
 * `size` or the valid taps, one rounding; Max/Min: take = !have || v is NaN || v better (the result widened and
 * narrowed back as the oracle's f32 -> f64 -> f32 does: a NaN gets the quiet bit). i32 (dtype 9): Sum wraps, Max and
 * Min from the first tap. op: 0 Sum, 1 Mean, 2 Max, 3 Min. */
void orc_window(const void* x, int dtype, int64_t outer, int64_t k_in, int64_t inner, int op, int64_t size,
                int64_t stride, int64_t dilation, int64_t pad_lo, int include_pad, void* out, int64_t k_out) {
  for (int64_t b = 0; b < outer; ++b)
    for (int64_t o = 0; o < k_out; ++o)
      for (int64_t i = 0; i < inner; ++i) {
        double acc = 0.0, best = 0.0;
        uint32_t acc_i = 0;
        int32_t best_i = 0;
        int64_t cnt = 0;
        int have = 0;
        for (int64_t kk = 0; kk < size; ++kk) {
          const int64_t p = o * stride - pad_lo + kk * dilation;
          if (p < 0 || p >= k_in) continue;
          const int64_t at = (b * k_in + p) * inner + i;
          if (dtype == 2) {
            const double v = (double)((const float*)x)[at];
            if (op <= 1) {
              acc += v;
              ++cnt;
            } else {
              if (!have || v != v || (op == 2 ? v > best : v < best)) best = v;
              have = 1;
            }
          } else {
            const int32_t v = ((const int32_t*)x)[at];
            if (op == 0) {
              acc_i += (uint32_t)v;
            } else {
              if (!have || (op == 2 ? v > best_i : v < best_i)) best_i = v;
              have = 1;
            }
          }
        }
        const int64_t dst = (b * k_out + o) * inner + i;
        if (dtype == 2) {
          float r;
          if (op == 0) r = (float)acc;
          else if (op == 1) r = (float)(acc / (double)(include_pad ? size : cnt));
          else r = best != best ? bits_f32(f32_bits((float)best) | 0x00400000u) : (float)best;
          ((float*)out)[dst] = r;
        } else {
          ((int32_t*)out)[dst] = op == 0 ? (int32_t)acc_i : best_i;
        }
      }
}

/* Im2Col (the oracle's eval_im2col, oracle/plan_window.rs:483-535): a dense NCHW input of `esz`-byte elements into
 * [N, C*kh*kw, oH*oW]; a raw-bit copy, zero bytes outside the input. */
void orc_im2col(const uint8_t* x, int64_t esz, int64_t n, int64_t c, int64_t h, int64_t w, int64_t kh, int64_t kw,
                int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw, uint8_t* out) {
  const int64_t oh_n = (h + 2 * ph - dh * (kh - 1) - 1) / sh + 1, ow_n = (w + 2 * pw - dw * (kw - 1) - 1) / sw + 1;
  const int64_t total = n * c * kh * kw * oh_n * ow_n;
  for (int64_t t = 0; t < total; ++t) {
    const int64_t col = t % (oh_n * ow_n), row = t / (oh_n * ow_n);
    const int64_t oh = col / ow_n, ow = col - oh * ow_n;
    const int64_t patch = row % (c * kh * kw), nn = row / (c * kh * kw);
    const int64_t cc = patch / (kh * kw), kij = patch - cc * (kh * kw);
    const int64_t ki = kij / kw, kj = kij - ki * kw;
    const int64_t ih = oh * sh - ph + ki * dh, iw = ow * sw - pw + kj * dw;
    if (ih >= 0 && ih < h && iw >= 0 && iw < w)
      memcpy(out + t * esz, x + (((nn * c + cc) * h + ih) * w + iw) * esz, (size_t)esz);
    else
      memset(out + t * esz, 0, (size_t)esz);
  }
}

/* The split-K variant of the outer-axis Sum/Mean (ondevice/README.md:185-218, splitk_validate.cu:40-50): f64
 * partials over chunks of ceil(rows / n_chunks) rows, each folded ascending from 0.0, added in chunk order from
 * the first; Mean divides by rows; one rounding. n_chunks clamped to [1, rows]. */
void orc_col_sum_f32_splitk(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int64_t n_chunks,
                            int mean, float* out, int threads) {
  if (n_chunks > rows) n_chunks = rows;
  if (n_chunks < 1) n_chunks = 1;
  const int64_t chunk_rows = rows > 0 ? (rows + n_chunks - 1) / n_chunks : 0;
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
  for (int64_t c = 0; c < cols; ++c) {
    double total = 0.0;
    for (int64_t k = 0; k < n_chunks; ++k) {
      double a = 0.0;
      const int64_t r0 = k * chunk_rows, r1 = r0 + chunk_rows < rows ? r0 + chunk_rows : rows;
      for (int64_t r = r0; r < r1; ++r) a += (double)x[r * row_stride + c];
      total = k == 0 ? a : total + a;
    }
    out[c] = (float)(mean ? total / (double)rows : total);
  }
}

/* RowReduce forms (Access::RowReduce; kernel_lift/row_reduce_launched.rs:1-24, the oracle's eval_row_reduce,
 * oracle/plan_contract.rs:265-360), in the launched lift's written order for a logical block of B threads:
 * form 1 softmax (Max(x); Sum(exp(x - r0)); exp(x - r0) / r1), 2 RMS norm (Mean(x * x); x / sqrt(r0 + eps)),
 * 3 centred quotient (Mean(x); Max(x - r0); (x - r0) / r1) — the forms of
 * crates/unpopped/tests/kernel_parallel_row_reduce_agrees.rs:99-131. Every expression is evaluated in f64 from the
 * f32 inputs and the f32 stage values; a Sum/Mean stage folds in the documented order (Mean divides the f64 total);
 * a Max stage folds as the oracle does (take = !have || v is NaN || v > acc); each stage value is rounded once to
 * f32, and the epilogue once on the store. */
static double orc_doc_total(const double* pre, int64_t n, int64_t block, double* acc) {
  for (int64_t t = 0; t < block; ++t) {
    double a = 0.0;
    for (int64_t c = t; c < n; c += block) a += pre[c];
    acc[t] = a;
  }
  for (int64_t s = block / 2; s > 0; s /= 2)
    for (int64_t t = 0; t < s; ++t) acc[t] += acc[t + s];
  return acc[0];
}

static double orc_max_stage(const double* pre, int64_t n) {
  double acc = 0.0;
  int have = 0;
  for (int64_t c = 0; c < n; ++c) {
    const double v = pre[c];
    if (!have || v != v || v > acc) acc = v;
    have = 1;
  }
  return acc;
}

void orc_row_reduce_f32(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int form, int64_t block,
                        double eps, float* out, int64_t out_stride, int threads) {
#pragma omp parallel num_threads(threads) if (threads > 1)
  {
    double* pre = (double*)malloc(sizeof(double) * (size_t)(cols > 0 ? cols : 1));
    double* acc = (double*)malloc(sizeof(double) * (size_t)block);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      const float* row = x + r * row_stride;
      float* o = out + r * out_stride;
      if (form == 1) {
        for (int64_t c = 0; c < cols; ++c) pre[c] = (double)row[c];
        const float r0 = (float)orc_max_stage(pre, cols);
        for (int64_t c = 0; c < cols; ++c) pre[c] = exp((double)row[c] - (double)r0);
        const float r1 = (float)orc_doc_total(pre, cols, block, acc);
        for (int64_t c = 0; c < cols; ++c) o[c] = (float)(pre[c] / (double)r1);
      } else if (form == 2) {
        for (int64_t c = 0; c < cols; ++c) pre[c] = (double)row[c] * (double)row[c];
        const float r0 = (float)(orc_doc_total(pre, cols, block, acc) / (double)cols);
        const double den = sqrt((double)r0 + eps);
        for (int64_t c = 0; c < cols; ++c) o[c] = (float)((double)row[c] / den);
      } else {
        for (int64_t c = 0; c < cols; ++c) pre[c] = (double)row[c];
        const float r0 = (float)(orc_doc_total(pre, cols, block, acc) / (double)cols);
        for (int64_t c = 0; c < cols; ++c) pre[c] = (double)row[c] - (double)r0;
        const float r1 = (float)orc_max_stage(pre, cols);
        for (int64_t c = 0; c < cols; ++c) o[c] = (float)(pre[c] / (double)r1);
      }
    }
    free(pre);
    free(acc);
  }
}

/* Max (extremum_fold, plan_contract.rs:179-210: take = !have || v is NaN || v > acc) and ArgMax
 * (arg_fold, plan_contract.rs:213-245: take = !have || (!acc.is_nan() && (v.is_nan() || v > acc)))
 * over a bf16 row, folded in f64. The max is stored as f32 (exact: bf16 is a subset). A NaN max is the
 * last NaN of the row, widened as the reference's f32->f64->f32 conversions widen it (quiet bit set). */
void orc_row_max_argmax_bf16(const uint16_t* x, int64_t rows, int64_t cols, int64_t row_stride,
                             float* max_out, int64_t* argmax_out, int threads) {
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* row = x + r * row_stride;
    double acc_m = 0.0, acc_a = 0.0;
    uint32_t acc_m_bits = 0;
    int have_m = 0, have_a = 0;
    int64_t best = 0;
    for (int64_t c = 0; c < cols; ++c) {
      double v = orc_bf16_to_f64(row[c]);
      int vnan = (v != v);
      if (!have_m || vnan || v > acc_m) {
        acc_m = v;
        acc_m_bits = vnan ? (((uint32_t)row[c] << 16) | 0x00400000u) : f32_bits((float)v);
      }
      have_m = 1;
      int take = !have_a || (!(acc_a != acc_a) && (vnan || v > acc_a));
      if (take) { acc_a = v; best = c; }
      have_a = 1;
    }
    if (max_out) max_out[r] = cols > 0 ? bits_f32(acc_m_bits) : 0.0f;
    if (argmax_out) argmax_out[r] = best;
  }
}

/* eval_reduction (oracle/plan_eval.rs:501-651) for a rank-2 f32 [rows, cols] input reduced over one axis (axis 1:
 * out[rows]; axis 0: out[cols]) in the serial order: fold_step / extremum_fold (plan_contract.rs:146-210) with an
 * f64 accumulator from 0, Mean divided by the reduced extent (an empty Mean is 0/0), one rounding to f32 at the
 * store. op: 0 Sum, 1 Mean, 2 Max, 3 Min. Max/Min: take = !have || v is NaN || v better than acc; a NaN result is
 * the fold's last NaN, widened as the f32->f64->f32 conversions widen it (quiet bit set). */
void orc_reduce2d_f32(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int axis, int op, float* out,
                      int threads) {
  const int64_t nk = axis == 1 ? rows : cols, nr = axis == 1 ? cols : rows;
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
  for (int64_t k = 0; k < nk; ++k) {
    double acc = 0.0;
    uint32_t acc_bits = 0;
    int have = 0;
    for (int64_t i = 0; i < nr; ++i) {
      const float f = axis == 1 ? x[k * row_stride + i] : x[i * row_stride + k];
      const double v = (double)f;
      if (op == 0 || op == 1) {
        acc += v;
      } else {
        const int vnan = v != v;
        const int better = op == 2 ? v > acc : v < acc;
        if (!have || vnan || better) {
          acc = v;
          acc_bits = vnan ? (f32_bits(f) | 0x00400000u) : f32_bits(f);
        }
        have = 1;
      }
    }
    if (op == 0) out[k] = (float)acc;
    else if (op == 1) out[k] = (float)(acc / (double)nr);
    else out[k] = have ? bits_f32(acc_bits) : 0.0f;
  }
}

/* Mean over the last axis in the launched lift's documented order (kernel_lift/block_reduce.rs:13-23): the
 * documented f64 sum of orc_row_sum_f32_documented, divided by the extent, one rounding. */
void orc_row_mean_f32_documented(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int64_t block,
                                 float* out, int threads) {
#pragma omp parallel num_threads(threads) if (threads > 1)
  {
    double* acc = (double*)malloc(sizeof(double) * (size_t)block);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      const float* row = x + r * row_stride;
      for (int64_t t = 0; t < block; ++t) {
        double a = 0.0;
        for (int64_t c = t; c < cols; c += block) a += (double)row[c];
        acc[t] = a;
      }
      for (int64_t s = block / 2; s > 0; s /= 2)
        for (int64_t t = 0; t < s; ++t) acc[t] += acc[t + s];
      out[r] = (float)(acc[0] / (double)cols);
    }
    free(acc);
  }
}

/* Sum (or Mean) over the outer axis of a rank-2 f32 input in the launched lift's documented order
 * (kernel_lift/block_reduce.rs:13-30: with the outer axis reduced, logical thread t folds rows t, t+B, ... of each
 * column into an f64; then acc[t] += acc[t+s] for s = B/2 .. 1; Mean divides by the row count; one rounding). */
void orc_col_sum_f32_documented(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int64_t block,
                                int mean, float* out, int threads) {
#pragma omp parallel num_threads(threads) if (threads > 1)
  {
    double* acc = (double*)malloc(sizeof(double) * (size_t)block);
#pragma omp for schedule(static)
    for (int64_t c = 0; c < cols; ++c) {
      for (int64_t t = 0; t < block; ++t) {
        double a = 0.0;
        for (int64_t r = t; r < rows; r += block) a += (double)x[r * row_stride + c];
        acc[t] = a;
      }
      for (int64_t s = block / 2; s > 0; s /= 2)
        for (int64_t t = 0; t < s; ++t) acc[t] += acc[t + s];
      out[c] = mean ? (float)(acc[0] / (double)rows) : (float)acc[0];
    }
    free(acc);
  }
}

/* eval_reduction for a rank-2 i32 input over one axis: the oracle folds in an i128 wrapped at 64 bits and the store
 * truncates to 32 (plan_eval.rs:530-545), which for Sum and Prod is wrapping 32-bit arithmetic; Max/Min take the
 * first element and then a strictly better one; And/Or/Xor are seeded by the first element (bit_fold); an empty fold
 * stores 0, or 1 for Prod. op: 0 Sum, 2 Max, 3 Min, 4 Prod, 5 And, 6 Or, 7 Xor. */
void orc_reduce2d_i32(const int32_t* x, int64_t rows, int64_t cols, int64_t row_stride, int axis, int op,
                      int32_t* out, int threads) {
  const int64_t nk = axis == 1 ? rows : cols, nr = axis == 1 ? cols : rows;
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
  for (int64_t k = 0; k < nk; ++k) {
    uint32_t acc = op == 4 ? 1u : 0u;
    int have = 0;
    for (int64_t i = 0; i < nr; ++i) {
      const int32_t v = axis == 1 ? x[k * row_stride + i] : x[i * row_stride + k];
      switch (op) {
        case 0: acc += (uint32_t)v; break;
        case 4: acc *= (uint32_t)v; break;
        case 2: if (!have || v > (int32_t)acc) acc = (uint32_t)v; break;
        case 3: if (!have || v < (int32_t)acc) acc = (uint32_t)v; break;
        case 5: acc = have ? (acc & (uint32_t)v) : (uint32_t)v; break;
        case 6: acc = have ? (acc | (uint32_t)v) : (uint32_t)v; break;
        case 7: acc = have ? (acc ^ (uint32_t)v) : (uint32_t)v; break;
      }
      have = 1;
    }
    out[k] = (int32_t)acc;
  }
}

/* ---- scatter: oracle/plan_eval.rs:430-490 (the scatter store), ir.rs:2723-2850 ---------------------- */

static int64_t orc_index_at(const void* ids, int kind, int64_t k) {
  if (kind == ORC_EK_I64) return ((const int64_t*)ids)[k];
  if (kind == ORC_EK_U32) return (int64_t)((const uint32_t*)ids)[k];
  return (int64_t)((const int32_t*)ids)[k];
}

/* Serial in the source order (row-major over updates [n, cols]): the target row is t = ids[i*ids_stride + j] (a
 * full-shape index) or ids[i] (ids_stride 0: index_add); a target outside [0, out_rows) is skipped; then
 * out[t][j] = combine(out[t][j], upd[i][j]). Element kinds: 9 I32, 23 U32, 10 I64 (Add wraps at the width, Max/Min
 * compare at the type's signedness); 2 F32, 4 F64 (Add in f64, stored at the dtype: one rounding per step).
 * combine: 1 Add, 2 Max, 3 Min. */
void orc_scatter(const void* upd, int64_t n, int64_t cols, int dtype, const void* ids, int index_dtype,
                 int64_t ids_stride, int combine, void* out, int64_t out_rows) {
  for (int64_t i = 0; i < n; ++i)
    for (int64_t j = 0; j < cols; ++j) {
      const int64_t t = orc_index_at(ids, index_dtype, ids_stride ? i * ids_stride + j : i);
      if (t < 0 || t >= out_rows) continue;
      const int64_t o = t * cols + j, u = i * cols + j;
      if (dtype == 2) {
        float* d = (float*)out;
        d[o] = (float)((double)d[o] + (double)((const float*)upd)[u]);
      } else if (dtype == 4) {
        double* d = (double*)out;
        d[o] = d[o] + ((const double*)upd)[u];
      } else if (dtype == ORC_EK_I64) {
        int64_t* d = (int64_t*)out;
        const int64_t v = ((const int64_t*)upd)[u];
        if (combine == 1) d[o] = (int64_t)((uint64_t)d[o] + (uint64_t)v);
        else if (combine == 2) d[o] = v > d[o] ? v : d[o];
        else d[o] = v < d[o] ? v : d[o];
      } else if (dtype == ORC_EK_U32) {
        uint32_t* d = (uint32_t*)out;
        const uint32_t v = ((const uint32_t*)upd)[u];
        if (combine == 1) d[o] = d[o] + v;
        else if (combine == 2) d[o] = v > d[o] ? v : d[o];
        else d[o] = v < d[o] ? v : d[o];
      } else {
        int32_t* d = (int32_t*)out;
        const int32_t v = ((const int32_t*)upd)[u];
        if (combine == 1) d[o] = (int32_t)((uint32_t)d[o] + (uint32_t)v);
        else if (combine == 2) d[o] = v > d[o] ? v : d[o];
        else d[o] = v < d[o] ? v : d[o];
      }
    }
}

/* bincount (crates/unpopped/tests/kernel_bincount_agrees.rs:1-10): counts[x[i]] += 1 for 0 <= x[i] < bins. */
void orc_bincount(const void* x, int64_t n, int index_dtype, int32_t* counts, int64_t bins) {
  for (int64_t i = 0; i < n; ++i) {
    const int64_t v = orc_index_at(x, index_dtype, i);
    if (v >= 0 && v < bins) counts[v] += 1;
  }
}

/* ---- scans: oracle/plan_window.rs:10-238 ---------------------------------------------------------- */

static inline int32_t orc_combine_i32(int op, int32_t a, int32_t b) {
  if (op == ORC_OP_SUM) return (int32_t)((uint32_t)a + (uint32_t)b); /* wrap_bits(.., 32) */
  if (op == ORC_OP_MAX) return a > b ? a : b;
  return a < b ? a : b;
}

/* scan_identity (plan_window.rs:221-238): Sum 0, Max the type minimum, Min the type maximum. */
int32_t orc_scan_identity_i32(int op) {
  if (op == ORC_OP_SUM) return 0;
  if (op == ORC_OP_MAX) return INT32_MIN;
  return INT32_MAX;
}

/* eval_scan for an I32 row-major [rows, k] scan along the last axis: inclusive writes after the combine;
 * exclusive writes before it, so element 0 gets the identity (Sum: acc starts at 0; Max/Min:
 * `have ? cur : ident`, plan_window.rs:165-172). Reverse walks j = k-1 .. 0. Integer Sum wraps at 32
 * bits (plan_window.rs:100-106). `carry` is combined in front of each row (a sharded scan's prefix). */
void orc_scan_i32(const int32_t* x, int32_t* y, int64_t rows, int64_t k, int op, int exclusive,
                  int reverse, int32_t carry, int threads) {
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1 && rows > 1)
  for (int64_t r = 0; r < rows; ++r) {
    const int32_t* xr = x + r * k;
    int32_t* yr = y + r * k;
    int32_t acc = carry;
    for (int64_t jj = 0; jj < k; ++jj) {
      int64_t j = reverse ? k - 1 - jj : jj;
      if (exclusive) {
        yr[j] = acc;
        acc = orc_combine_i32(op, acc, xr[j]);
      } else {
        acc = orc_combine_i32(op, acc, xr[j]);
        yr[j] = acc;
      }
    }
  }
}

/* The same scan over one long row on several threads: chunk totals, an exclusive scan of the totals,
 * then each chunk scanned from its carry (integer combines are associative, so the bytes equal the
 * serial walk's). Forward only; the CPU baseline of the reference arm. */
void orc_scan_i32_chunked(const int32_t* x, int32_t* y, int64_t n, int op, int exclusive, int threads) {
  if (threads < 1) threads = 1;
  int32_t* tot = (int32_t*)malloc(sizeof(int32_t) * (size_t)threads);
  int64_t chunk = (n + threads - 1) / threads;
#pragma omp parallel num_threads(threads)
  {
    int t = 0;
#ifdef _OPENMP
    t = omp_get_thread_num();
#endif
    int64_t lo = (int64_t)t * chunk, hi = lo + chunk < n ? lo + chunk : n;
    int32_t a = orc_scan_identity_i32(op);
    for (int64_t i = lo; i < hi; ++i) a = orc_combine_i32(op, a, x[i]);
    tot[t] = a;
#pragma omp barrier
    int32_t carry = orc_scan_identity_i32(op);
    for (int u = 0; u < t; ++u) carry = orc_combine_i32(op, carry, tot[u]);
    int32_t acc = carry;
    for (int64_t i = lo; i < hi; ++i) {
      if (exclusive) { y[i] = acc; acc = orc_combine_i32(op, acc, x[i]); }
      else { acc = orc_combine_i32(op, acc, x[i]); y[i] = acc; }
    }
  }
  free(tot);
}

/* Fold of a whole array (the per-shard total of a sharded scan). */
int32_t orc_reduce_i32(const int32_t* x, int64_t n, int op) {
  int32_t a = orc_scan_identity_i32(op);
  for (int64_t i = 0; i < n; ++i) a = orc_combine_i32(op, a, x[i]);
  return a;
}

/* ---- gather: oracle/plan_eval.rs:284-430 (gather arm 363-385) --------------------------------------- */

/* out[n, :] = table[ids[n], :] for a 1-D index broadcast over the row (OpDef::embedding /
 * index_select / gather on axis 0, ir.rs:3838-3890). The index is read once (as i64); the load address
 * is clamped to [0, V-1]; an index outside [0, V) skips the store (Skip: the output keeps its bytes),
 * writes zeros (ZeroFill: Val::Float(0.0) / Val::Int(0), all-zero bits) or stores the clamped row
 * (Clamp). The row moves verbatim (store_val's Raw arm, expr_eval.rs:480-484). */
void orc_gather_rows(const uint8_t* table, int64_t table_rows, int64_t row_bytes, const void* ids,
                     int index_dtype, int64_t n, int oob, uint8_t* out, int threads) {
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
  for (int64_t i = 0; i < n; ++i) {
    int64_t raw;
    if (index_dtype == ORC_EK_I64) raw = ((const int64_t*)ids)[i];
    else if (index_dtype == ORC_EK_U32) raw = (int64_t)((const uint32_t*)ids)[i];
    else raw = (int64_t)((const int32_t*)ids)[i];
    int64_t hi = table_rows - 1 > 0 ? table_rows - 1 : 0;
    int64_t g = raw < 0 ? 0 : (raw > hi ? hi : raw);
    uint8_t* dst = out + i * row_bytes;
    if (raw < 0 || raw >= table_rows) {
      if (oob == ORC_OOB_SKIP) continue;
      if (oob == ORC_OOB_ZERO_FILL) { memset(dst, 0, (size_t)row_bytes); continue; }
    }
    if (table_rows > 0) memcpy(dst, table + g * row_bytes, (size_t)row_bytes);
  }
}

/* ---- int4 dequant and the dequant GEMM ---------------------------------------------------------------- */

/* i4 read (tests/sub_byte_packing.rs:24-40, cfamily.rs:446-470): two per byte, low nibble = even index,
 * sign-extended. */
static inline int orc_i4_at(const uint8_t* w, int64_t idx) {
  uint8_t b = w[idx >> 1];
  int v = (idx & 1) ? (b >> 4) : (b & 0x0f);
  return v >= 8 ? v - 16 : v;
}

int orc_i4_value(const uint8_t* w, int64_t idx) { return orc_i4_at(w, idx); }

/* The reference's dequant GEMM KAT form (crates/unpopped/tests/support/dequant.rs:1-5,163-178):
 * out[r][c] = sum_k (w[r][k] - zero[r][k/G]) * scale[r][k/G] * x[k][c] with I32 zero points, scales,
 * activations and result; `w` is I4 (signed) or U4 (unsigned) [R, K]. Shares the nibble reader with
 * the W4A16 oracle below, so the KAT pins its packing and group indexing. */
void orc_dequant_gemm_kat(const uint8_t* w, int is_signed, const int32_t* zero, const int32_t* scale,
                          const int32_t* x, int64_t R, int64_t K, int64_t C, int64_t group, int32_t* out) {
  int64_t g = K / group;
  for (int64_t r = 0; r < R; ++r)
    for (int64_t c = 0; c < C; ++c) {
      int64_t acc = 0;
      for (int64_t k = 0; k < K; ++k) {
        int v = orc_i4_at(w, r * K + k);
        if (!is_signed && v < 0) v += 16;
        acc += (int64_t)(v - zero[r * g + k / group]) * scale[r * g + k / group] * x[k * C + c];
      }
      out[r * C + c] = (int32_t)acc;
    }
}

/* out[n][k] = bf16(w[n][k] * scale[n][k/group]): the product is exact in f64 and rounds once
 * (encode_float's Bf16 arm). `w` is [N, K] i4 row-major, `scale` f16 [N, K/group]. */
void orc_dequant_i4_bf16(const uint8_t* w, const uint16_t* scale, int64_t n, int64_t k, int64_t group,
                         uint16_t* out, int threads) {
  int64_t g = k / group;
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
  for (int64_t r = 0; r < n; ++r)
    for (int64_t c = 0; c < k; ++c) {
      double s = orc_f16_to_f64(scale[r * g + c / group]);
      out[r * k + c] = orc_f64_to_bf16((double)orc_i4_at(w, r * k + c) * s);
    }
}

/* The dequant GEMM (crates/unpopped/tests/support/dequant.rs:1-5,163-178, generalized to a f16 group scale,
 * bf16 activations and no zero point): out[m][n] = sum_k w[n][k] * scale[n][k/group] * x[m][k], every
 * product exact in f64, summed in ascending k in f64 (the WideFloat model, docs/accum-policies.md:8-20),
 * one rounding to bf16. `abs_sum` (optional) receives sum_k |w * scale * x| per output, the scale of the
 * tolerance a device f32 accumulation is held to. */
void orc_w4a16(const uint8_t* w, const uint16_t* scale, const uint16_t* x, int64_t m, int64_t n,
               int64_t k, int64_t group, uint16_t* out, double* exact, double* abs_sum, int threads) {
  int64_t g = k / group;
  double* xf = (double*)malloc(sizeof(double) * (size_t)(m * k));
  for (int64_t i = 0; i < m * k; ++i) xf[i] = orc_bf16_to_f64(x[i]);
#pragma omp parallel num_threads(threads) if (threads > 1)
  {
    double* ws = (double*)malloc(sizeof(double) * (size_t)k); /* w * scale of one row, exact */
#pragma omp for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
      for (int64_t c = 0; c < k; ++c)
        ws[c] = (double)orc_i4_at(w, r * k + c) * orc_f16_to_f64(scale[r * g + c / group]);
      for (int64_t i = 0; i < m; ++i) {
        const double* xi = xf + i * k;
        double acc = 0.0, sa = 0.0;
        for (int64_t c = 0; c < k; ++c) {
          double p = ws[c] * xi[c];
          acc += p;
          sa += fabs(p);
        }
        out[i * n + r] = orc_f64_to_bf16(acc);
        if (exact) exact[i * n + r] = acc;
        if (abs_sum) abs_sum[i * n + r] = sa;
      }
    }
    free(ws);
  }
  free(xf);
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
