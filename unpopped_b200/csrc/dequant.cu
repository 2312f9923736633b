// dequant.cu — group-wise int4 -> bf16 dequant for sm_100a: out[n][k] = bf16(w[n][k] * scale[n][k/group]).
//
// Semantics: the i4 reader of the reference (two per byte, low nibble = even index, sign-extended;
// crates/unpopped/tests/sub_byte_packing.rs:24-40, crates/unpopped/src/cfamily.rs:446-470) and the
// dequant product of crates/unpopped/tests/support/dequant.rs:163-178 with a f16 group scale and no zero
// point. w * scale needs at most 4 + 11 significant bits, so the f32 product is exact and the bf16
// conversion is the single round-to-nearest-even the oracle's f64 path performs (encode_float's Bf16 arm,
// crates/unpopped/src/oracle/expr_eval.rs:520-530).
//
// Each thread turns one 32-bit word of w (8 nibbles) into one 16-byte chunk of output: the int4 bytes are
// read 4 per lane and the bf16 bytes written 16 per lane, both as contiguous warp accesses.
#include "common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace up {

// 8 signed nibbles of `q` (low first) times `s`, as four packed bf16x2 words.
__device__ __forceinline__ uint4 dequant8(uint32_t q, float s) {
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    // 2^23 + (nibble ^ 8) as an f32, minus 2^23 + 8: the signed nibble, exactly.
    const uint32_t a = ((q >> (8 * j)) & 0xfu) ^ 0x8u;
    const uint32_t b = ((q >> (8 * j + 4)) & 0xfu) ^ 0x8u;
    const float fa = (__uint_as_float(0x4b000000u | a) - 8388616.0f) * s;
    const float fb = (__uint_as_float(0x4b000000u | b) - 8388616.0f) * s;
    uint32_t packed;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(fb), "f"(fa));
    o[j] = packed;
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// k % 8 == 0 and group % 8 == 0: a word of w never straddles a row or a group. CTAs take whole rows; a row's
// words are split over the threads with 32-bit index arithmetic only.
//
// Rows of at most 1024 words (k <= 8192) are software-pipelined: a CTA issues the loads of its next row (words
// and scales) before it converts and stores the current one, so the read latency hides behind the stores. The
// launch gives each CTA only a few rows (a grid of 32 CTAs per SM), which measured fastest: 90 % of the copy
// bandwidth against 79 % for one row at a time with 8 CTAs per SM. Longer rows take the plain loop.
__global__ void __launch_bounds__(256) dequant_i4_rows_kernel(const uint32_t* __restrict__ w,
                                                              const __half* __restrict__ scale, int64_t n, int wpr,
                                                              int gpr, int wpg, uint4* __restrict__ out) {
  if (wpr <= 4 * 256) {
    uint32_t q[4];
    __half sh[4];
    auto load = [&](int64_t r) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = threadIdx.x + u * 256;
        if (r < n && i < wpr) {
          q[u] = __ldg(w + r * wpr + i);
          sh[u] = scale[r * gpr + (unsigned)i / (unsigned)wpg];
        }
      }
    };
    int64_t r = blockIdx.x;
    load(r);
    for (; r < n; r += gridDim.x) {
      uint32_t cq[4];
      float sc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        cq[u] = q[u];
        sc[u] = __half2float(sh[u]);
      }
      load(r + gridDim.x);
      uint4* orow = out + r * wpr;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = threadIdx.x + u * 256;
        if (i < wpr) st_cs_v4(orow + i, dequant8(cq[u], sc[u]));
      }
    }
    return;
  }
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const uint32_t* wr = w + r * wpr;
    const __half* sr = scale + r * gpr;
    uint4* orow = out + r * wpr;
    for (int i0 = threadIdx.x; i0 < wpr; i0 += 256 * 4) {
      uint32_t q[4];
      float sc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * 256;
        if (i < wpr) {
          q[u] = __ldg(wr + i);
          sc[u] = __half2float(sr[(unsigned)i / (unsigned)wpg]);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * 256;
        if (i < wpr) st_cs_v4(orow + i, dequant8(q[u], sc[u]));
      }
    }
  }
}

// Any k and group (k % group == 0): one output element per thread.
__global__ void dequant_i4_any_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ scale, int64_t n,
                                      int64_t k, int64_t group, uint16_t* __restrict__ out) {
  const int64_t total = n * k, gpr = k / group;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / k, c = i - r * k;
    const uint8_t b = w[i >> 1];
    int v = (i & 1) ? (b >> 4) : (b & 0xf);
    v = v >= 8 ? v - 16 : v;
    const float f = (float)v * __half2float(scale[r * gpr + c / group]);
    out[i] = __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
}

}  // namespace up

using namespace up;

extern "C" int up_sm100_dequant_i4_bf16(const uint8_t* w, const uint16_t* scale, int64_t n, int64_t k, int64_t group,
                                        uint16_t* out, void* stream) {
  UP_CHECK_ARG(n >= 0 && k >= 0 && group > 0);
  if (k % group != 0) return UP_ERR_UNSUPPORTED;
  if (n == 0 || k == 0) return UP_OK;
  UP_CHECK_ARG(w != nullptr && scale != nullptr && out != nullptr);
  if ((n * k) % 2 != 0) return UP_ERR_UNSUPPORTED;  // the last byte would be half a row
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int sms = sm_count();
  const auto* sc = reinterpret_cast<const __half*>(scale);
  if (k % 8 == 0 && group % 8 == 0 && aligned(w, 4) && aligned(out, 16) && k / 8 <= 0x7fffffff) {
    int64_t blocks = n;
    const int64_t cap = (int64_t)sms * (k / 8 <= 4 * 256 ? 32 : 8);
    if (blocks > cap) blocks = cap;
    dequant_i4_rows_kernel<<<(int)blocks, 256, 0, s>>>(reinterpret_cast<const uint32_t*>(w), sc, n, (int)(k / 8),
                                                       (int)(k / group), (int)(group / 8), reinterpret_cast<uint4*>(out));
  } else {
    int64_t blocks = (n * k + 255) / 256;
    const int64_t cap = (int64_t)sms * 16;
    if (blocks > cap) blocks = cap;
    dequant_i4_any_kernel<<<(int)blocks, 256, 0, s>>>(w, sc, n, k, group, out);
  }
  note_launch();
  return check_launch();
}

UP_DEFINE_REVISION(dequant)
