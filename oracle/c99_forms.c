/*
 * c99_forms.c — restatements of the serial C that the reference's C99 emitter (crates/unpopped-cpu-c) writes for
 * the lifted kernels of the five benchmark configurations.
 *
 * TEST INFRASTRUCTURE ONLY: these are timed on the host cores as the "C99" CPU baseline beside the oracle, and
 * checked against the oracle by the CPU tests. Nothing in the product library links, loads or calls them.
 *
 * The emitter spells a launched kernel as the "serialized thread loop" (crates/unpopped-cpu-c/src/launch.rs:1-45):
 * every local is an array with one element per thread of a block, the blocks run one after another, and each run
 * of barrier-free statements is a loop over the threads (a Barrier ends one thread loop and starts the next). A
 * statement that holds a Barrier (the row loop of a block-strided kernel, a tree round) is spelled once, around
 * the thread loops of its body. A kernel with no launch shape (a serial lift) is a plain nest of loops. Buffers
 * use the emitter's argument ABI (crates/unpopped-cpu-c/src/base.rs:75-95): a pointer, its shape and stride
 * arrays (elements) and a base offset, so every access is `b[base + sum(i_d * stride_d)]`; the function returns
 * an int status, 0 on success.
 *
 * Forms, each citing the lift whose KernelFn it serializes:
 *  - row sum: the serial lift (kernel_lift.rs:447-490, f64 accumulator, one rounding) and the launched
 *    block-tree lift (kernel_lift/block_reduce.rs:1-100: thread t folds t, t+B, ...; the tree s = B/2 .. 1);
 *  - scan: the serial lift (kernel_lift.rs:504-520) and the launched three-phase lift
 *    (kernel_lift/scan_launched.rs:1-30: chunk totals, Kogge-Stone over the B totals with the round's old
 *    values, rewrite), for a rank-1 row that block 0 does;
 *  - gather: the per-cell loop nest of the gather lift (kernel_lift/gather.rs:35-60, 184-232: the index is read
 *    once per cell, the load address clamped, the store guarded by the OOB policy);
 *  - max + argmax: the kernel-layer loop (crates/unpopped/tests/support/arg_loop.rs:1-15);
 *  - W4A16: the dequant GEMM KernelFn (crates/unpopped/tests/support/dequant.rs:1-60), one thread per output cell,
 *    `acc += widen(w) * scale * x` ascending in k, here with bf16 activations, f16 group scales and an f32
 *    accumulator rounded once to bf16.
 *
 * Build: with up_oracle.c into liborc.so (oracle/Makefile), gcc -O2 -ffp-contract=off.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef long long ll;

/* codecs from up_oracle.c */
uint16_t orc_f32_to_bf16(float x);
double orc_f16_to_f64(uint16_t h);

static inline float bf16_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

#define AT2(base, st, i, j) ((base) + (ll)(i) * (st)[0] + (ll)(j) * (st)[1])

/* ---- row sum ------------------------------------------------------------------------------------------------ */

/* The serial reduction lift over the last axis of [rows, cols]: out[r] = (float)(sum in f64, ascending). */
int c99_row_sum_serial(const float* b0, const ll* b0_shape, const ll* b0_stride, ll b0_base, float* b1,
                       const ll* b1_shape, const ll* b1_stride, ll b1_base) {
  (void)b1_shape;
  for (ll r = 0; r < b0_shape[0]; ++r) {
    double acc = 0.0;
    for (ll c = 0; c < b0_shape[1]; ++c) acc += (double)b0[AT2(b0_base, b0_stride, r, c)];
    b1[b1_base + r * b1_stride[0]] = (float)acc;
  }
  return 0;
}

/* The launched block-tree lift on `grid` blocks of `block` threads, serialized. */
int c99_row_sum_launched(const float* b0, const ll* b0_shape, const ll* b0_stride, ll b0_base, float* b1,
                         const ll* b1_shape, const ll* b1_stride, ll b1_base, unsigned block, unsigned grid) {
  (void)b1_shape;
  if (block == 0 || block > 1024 || (block & (block - 1)) || grid == 0) return 2;
  double acc[1024];     /* local acc, one per thread */
  double partial[1024]; /* the Shared array */
  const ll rows = b0_shape[0], cols = b0_shape[1];
  for (unsigned bx = 0; bx < grid; ++bx) {
    for (ll r = bx; r < rows; r += grid) {  /* block-level: the row loop holds barriers */
      for (unsigned t = 0; t < block; ++t) { /* thread loop: fold the slice, publish */
        acc[t] = 0.0;
        for (ll c = t; c < cols; c += block) acc[t] += (double)b0[AT2(b0_base, b0_stride, r, c)];
        partial[t] = acc[t];
      }
      for (unsigned s = block / 2; s >= 1; s /= 2) { /* each round ends at a barrier */
        for (unsigned t = 0; t < block; ++t)
          if (t < s) partial[t] = partial[t] + partial[t + s];
      }
      for (unsigned t = 0; t < block; ++t)
        if (t == 0) b1[b1_base + r * b1_stride[0]] = (float)partial[0];
    }
  }
  return 0;
}

/* ---- scan (rank 1, i32; op 0 Sum wrapping, 2 Max) ------------------------------------------------------------ */

static inline int32_t comb(int op, int32_t a, int32_t b) {
  if (op == 0) return (int32_t)((uint32_t)a + (uint32_t)b);
  return op == 2 ? (a > b ? a : b) : (a < b ? a : b);
}
static inline int32_t ident(int op) { return op == 0 ? 0 : (op == 2 ? INT32_MIN : INT32_MAX); }

int c99_scan_serial(const int32_t* b0, const ll* b0_shape, const ll* b0_stride, ll b0_base, int32_t* b1,
                    const ll* b1_shape, const ll* b1_stride, ll b1_base, int op, int exclusive) {
  (void)b1_shape;
  int32_t acc = ident(op);
  for (ll i = 0; i < b0_shape[0]; ++i) {
    const int32_t v = b0[b0_base + i * b0_stride[0]];
    if (exclusive) {
      b1[b1_base + i * b1_stride[0]] = acc;
      acc = comb(op, acc, v);
    } else {
      acc = comb(op, acc, v);
      b1[b1_base + i * b1_stride[0]] = acc;
    }
  }
  return 0;
}

int c99_scan_launched(const int32_t* b0, const ll* b0_shape, const ll* b0_stride, ll b0_base, int32_t* b1,
                      const ll* b1_shape, const ll* b1_stride, ll b1_base, int op, int exclusive, unsigned block) {
  (void)b1_shape;
  if (block == 0 || block > 1024 || (block & (block - 1))) return 2;
  int32_t acc[1024], red[1024], partial[1024];
  ll lo[1024], hi[1024];
  const ll n = b0_shape[0];
  const ll chunk = (n + block - 1) / block;
  /* 1. totals */
  for (unsigned t = 0; t < block; ++t) {
    lo[t] = (ll)t * chunk < n ? (ll)t * chunk : n;
    hi[t] = lo[t] + chunk < n ? lo[t] + chunk : n;
    acc[t] = ident(op);
    for (ll i = lo[t]; i < hi[t]; ++i) acc[t] = comb(op, acc[t], b0[b0_base + i * b0_stride[0]]);
    partial[t] = acc[t];
  }
  /* 2. Kogge-Stone over the totals: each round reads the old values into a local, then writes them back */
  for (unsigned d = 1; d < block; d *= 2) {
    for (unsigned t = 0; t < block; ++t) red[t] = t >= d ? comb(op, partial[t], partial[t - d]) : partial[t];
    for (unsigned t = 0; t < block; ++t) partial[t] = red[t];
  }
  /* 3. writes, from each thread's offset */
  for (unsigned t = 0; t < block; ++t) {
    acc[t] = t > 0 ? partial[t - 1] : ident(op);
    for (ll i = lo[t]; i < hi[t]; ++i) {
      const int32_t v = b0[b0_base + i * b0_stride[0]];
      if (exclusive) {
        b1[b1_base + i * b1_stride[0]] = acc[t];
        acc[t] = comb(op, acc[t], v);
      } else {
        acc[t] = comb(op, acc[t], v);
        b1[b1_base + i * b1_stride[0]] = acc[t];
      }
    }
  }
  return 0;
}

/* ---- gather: out[n, d] = table[ids[n], d], per cell (bf16 or any 2-byte element), i32 ids --------------------- */

int c99_gather_rows_u16(const uint16_t* b0, const ll* b0_shape, const ll* b0_stride, ll b0_base, const int32_t* b1,
                        const ll* b1_shape, const ll* b1_stride, ll b1_base, uint16_t* b2, const ll* b2_shape,
                        const ll* b2_stride, ll b2_base, int oob) {
  (void)b1_shape;
  const ll extent = b0_shape[0];
  for (ll n = 0; n < b2_shape[0]; ++n)
    for (ll d = 0; d < b2_shape[1]; ++d) {
      const ll raw = (ll)b1[b1_base + n * b1_stride[0]]; /* the index, once per cell */
      const int in_range = raw >= 0 && raw < extent;
      const ll clamped = extent == 0 ? 0 : (raw < 0 ? 0 : (raw >= extent ? extent - 1 : raw));
      if (!in_range && oob == 0) continue; /* Skip: the destination keeps its bytes */
      uint16_t v = 0;
      if (in_range || oob == 1) v = b0[AT2(b0_base, b0_stride, clamped, d)];
      b2[AT2(b2_base, b2_stride, n, d)] = v;
    }
  return 0;
}

/* ---- max + argmax over bf16 rows (the kernel-layer loop) --------------------------------------------------- */

int c99_row_max_argmax_bf16(const uint16_t* b0, const ll* b0_shape, const ll* b0_stride, ll b0_base, float* b1,
                            ll b1_base, int64_t* b2, ll b2_base) {
  for (ll r = 0; r < b0_shape[0]; ++r) {
    float best = bf16_f32(b0[AT2(b0_base, b0_stride, r, 0)]);
    int64_t bi = 0;
    for (ll j = 1; j < b0_shape[1]; ++j) {
      const float x = bf16_f32(b0[AT2(b0_base, b0_stride, r, j)]);
      if (best == best && (x != x || x > best)) {
        best = x;
        bi = j;
      }
    }
    b1[b1_base + r] = best;
    b2[b2_base + r] = bi;
  }
  return 0;
}

/* ---- W4A16: one thread per output cell (m, n), serialized ------------------------------------------------- */

int c99_w4a16(const uint8_t* w, const uint16_t* scale, const uint16_t* x, ll m, ll n, ll k, ll group,
              uint16_t* out) {
  if (group <= 0 || k % group) return 2;
  const ll groups = k / group;
  for (ll r = 0; r < n; ++r)      /* threads: x fastest over the M columns of the output, as the KernelFn */
    for (ll c = 0; c < m; ++c) {
      float acc = 0.0f;
      for (ll g = 0; g < groups; ++g) {
        const float s = (float)orc_f16_to_f64(scale[r * groups + g]);
        for (ll kk = 0; kk < group; ++kk) {
          const ll kx = g * group + kk;
          const ll idx = r * k + kx;
          int v = (w[idx >> 1] >> ((idx & 1) * 4)) & 0xF;
          if (v >= 8) v -= 16;
          acc += (float)v * s * bf16_f32(x[c * k + kx]);
        }
      }
      out[c * n + r] = orc_f32_to_bf16(acc);
    }
  return 0;
}
