// w4a16.cu — int4 group-wise dequant fused into a W4A16 GEMM on the sm_100a tensor cores (tcgen05).
//
//   out[m][n] = bf16( sum_k x[m][k] * w[n][k] * scale[n][k / group] )
//
// Semantics: the dequant GEMM of crates/unpopped/tests/support/dequant.rs:1-5,163-178 generalized to f16
// group scales, bf16 activations and no zero point (i4: two per byte, low nibble = even k, sign-extended;
// tests/sub_byte_packing.rs:24-40), with f32 accumulation. The oracle sums exactly and rounds once
// (docs/accum-policies.md:8-20); this kernel is held to |got - exact_bf16| <= 1/2 ulp_bf16 + gamma * sum|x w s|.
//
// Design (swap-AB: the weight rows are the MMA's M, the <= 16 activation rows its N):
//  * A unit of work is one k-block (128 k) of one 128-row tile of W. The N/128 x K/128 units are split
//    evenly over one persistent CTA per SM (stream-K), so every SM streams the same share of W.
//  * warp 0 (one lane): TMA producer. Per unit it loads the int4 tile (128 rows x 64 bytes, 64-byte
//    swizzle) and the bf16 activation k-block (16 rows x 128 k, 128-byte swizzle) into a ring of smem
//    stages. No multicast.
//  * warps 2..9: dequant. Each thread owns one W row (its TMEM lane) and half of the k-block; it turns
//    the nibbles into exact bf16 with one prmt + one lop3 + one bf16x2 subtract per pair and stores them
//    straight into tensor memory (tcgen05.st), where they are the MMA's A operand. Dequantized weights
//    never touch shared memory, which keeps smem bandwidth for the TMA stream.
//  * warp 1 (one lane): issues 8 tcgen05.mma (M=128, N=16, K=16, A from TMEM, B from smem) per unit into
//    one of four TMEM accumulator slots, and commits to mbarriers.
//  * the same dequant warps, two units behind, read the unit's f32 accumulator (tcgen05.ld), scale it by
//    scale[n][k-block] in f32 and add it to registers. A tile finished inside one CTA is written as bf16;
//    a tile split between CTAs writes f32 partials, and whichever CTA finishes it last (an atomic count)
//    sums the partials in CTA order and writes bf16 — no CTA ever waits on another.
// Every mbarrier wait is bounded; a wait that runs out sets the workspace error word and the CTA unwinds.
#include "common.cuh"
#include "tc.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace up {
namespace w4 {

constexpr int kTileN = 128;                    // W rows per tile = MMA M
constexpr int kMmaN = 16;                      // activation rows = MMA N
constexpr int kKB = 128;                       // k per unit
constexpr int kStages = 10;                    // smem ring depth
constexpr int kWBytes = kTileN * kKB / 2;      // 8 KiB of int4
constexpr int kXBytes = kMmaN * kKB * 2;       // 4 KiB of bf16
constexpr int kSBytes = kTileN * 8 * 2;        // 2 KiB: an 8-wide column block of f16 scales per row
constexpr int kStageBytes = kWBytes + kXBytes + kSBytes;  // 14 KiB (1024-aligned parts)
constexpr int kAStages = 4;                    // TMEM A stages, 64 columns each
constexpr int kDSlots = 4;                     // TMEM accumulator slots, 16 columns each
constexpr int kTmemCols = 512;
constexpr int kACol0 = 0;
constexpr int kDCol0 = kAStages * 64;          // 256
constexpr int kLag = 2;                        // epilogue trails the dequant by this many units
constexpr int kThreads = 320;                  // warp 0 TMA, warp 1 MMA, warps 2..9 dequant/epilogue
constexpr int kDqThreads = 256;
constexpr int kBarBytes = 1024;
constexpr size_t kSmemBytes = 1024 /*alignment slack*/ + (size_t)kStages * kStageBytes + kBarBytes;

struct WsHeader {
  uint32_t ticket, done, epoch, error;  // same layout as the scan workspace: `error` at byte 12
  uint32_t pad[12];
};

__device__ __forceinline__ int64_t cta_of_unit(int64_t u, int64_t U, int64_t P) {
  int64_t c = (u * P) / U;
  while (c + 1 < P && ((c + 1) * U) / P <= u) ++c;
  while (c > 0 && (c * U) / P > u) --c;
  return c;
}

__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) ^ c
  return d;
}

// Two signed nibbles (low = even k) -> exact bf16x2.
__device__ __forceinline__ uint32_t nib2_to_bf16x2(uint32_t q, uint32_t q4, int p) {
  const uint32_t sel = (uint32_t)(p | (p << 4) | ((4 + p) << 8) | ((4 + p) << 12));
  // bf16 0x4300|(n^8) == 128 + (n ^ 8); minus 136 gives the signed nibble.
  const uint32_t t = lop3_and_xor(__byte_perm(q, q4, sel), 0x000f000fu, 0x43084308u);
  __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&t);
  const uint32_t c136 = 0x43084308u;
  v = __hsub2(v, *reinterpret_cast<const __nv_bfloat162*>(&c136));
  return *reinterpret_cast<const uint32_t*>(&v);
}

// kScaleTma: the unit's group scales arrive in the stage by TMA (needs K/group % 8 == 0, so a row of scales
// is a whole number of 16-byte chunks); otherwise each thread reads its scale from global memory.
template <bool kScaleTma>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                 const __grid_constant__ CUtensorMap tmS, const __half* __restrict__ scale, uint16_t* __restrict__ out, int M, int64_t N, int64_t K,
                 int64_t group, int64_t U, int64_t G, int64_t S_max, WsHeader* hdr, uint32_t* counters,
                 float* partials, uint64_t wait_ns) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* a_full = empty + kStages;
  uint64_t* a_empty = a_full + kAStages;
  uint64_t* d_full = a_empty + kAStages;
  uint64_t* d_empty = d_full + kDSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d_empty + kDSlots);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t P = gridDim.x;
  const int64_t lo = ((int64_t)blockIdx.x * U) / P, hi = (((int64_t)blockIdx.x + 1) * U) / P;
  const int64_t n_units = hi - lo;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], kDqThreads + 1);
    }
    for (int a = 0; a < kAStages; ++a) {
      tc::mbar_init(&a_full[a], kDqThreads);
      tc::mbar_init(&a_empty[a], 1);
    }
    for (int d = 0; d < kDSlots; ++d) {
      tc::mbar_init(&d_full[d], 1);
      tc::mbar_init(&d_empty[d], kDqThreads);
    }
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  auto give_up = [&]() {
    *abort_flag = 1;
    atomicOr(&hdr->error, 1u);
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tc::tma_prefetch_desc(&tmW);
      tc::tma_prefetch_desc(&tmX);
      if (kScaleTma) tc::tma_prefetch_desc(&tmS);
      int64_t issued = 0;
      for (int64_t i = 0; i < n_units; ++i) {
        const int s = (int)(i % kStages);
        const uint32_t ph = (uint32_t)((i / kStages) & 1);
        if (!tc::mbar_wait(&empty[s], ph ^ 1u, wait_ns, abort_flag)) {
          give_up();
          break;
        }
        const int64_t u = lo + i;
        const int32_t t = (int32_t)(u / G), kb = (int32_t)(u % G);
        uint8_t* st = smem + (size_t)s * kStageBytes;
        tc::mbar_arrive_expect_tx(&full[s], kScaleTma ? kStageBytes : kWBytes + kXBytes);
        tc::tma_load_2d(st, &tmW, &full[s], kb * (kKB / 2), t * kTileN);
        tc::tma_load_2d(st + kWBytes, &tmX, &full[s], kb * kKB, 0);
        tc::tma_load_2d(st + kWBytes + 2048, &tmX, &full[s], kb * kKB + 64, 0);
        if (kScaleTma)
          tc::tma_load_2d(st + kWBytes + kXBytes, &tmS, &full[s], (int32_t)(((int64_t)kb * kKB / group) & ~int64_t(7)),
                          t * kTileN);
        issued = i + 1;
      }
      // Unwinding after an abort: let the copies already issued land before smem is released.
      if (*abort_flag) {
        for (int64_t i = (issued > kStages ? issued - kStages : 0); i < issued; ++i)
          tc::mbar_wait(&full[i % kStages], (uint32_t)((i / kStages) & 1), wait_ns, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(kTileN, kMmaN);
      int64_t issued = 0;
      for (int64_t i = 0; i < n_units; ++i) {
        const int s = (int)(i % kStages), a = (int)(i % kAStages), d = (int)(i % kDSlots);
        const uint32_t ph = (uint32_t)((i / kStages) & 1), aph = (uint32_t)((i / kAStages) & 1),
                       dph = (uint32_t)((i / kDSlots) & 1);
        if (!tc::mbar_wait(&full[s], ph, wait_ns, abort_flag) || !tc::mbar_wait(&a_full[a], aph, wait_ns, abort_flag) ||
            !tc::mbar_wait(&d_empty[d], dph ^ 1u, wait_ns, abort_flag)) {
          give_up();
          break;
        }
        tc::fence_after_sync();
        const uint32_t xaddr = tc::smem_u32(smem + (size_t)s * kStageBytes + kWBytes);
#pragma unroll
        for (int j = 0; j < kKB / 16; ++j) {
          const uint64_t bdesc = tc::sdesc_kmajor_sw128(xaddr + (uint32_t)((j >> 2) * 2048 + (j & 3) * 32));
          tc::mma_ts_bf16(tmem + kDCol0 + d * 16, tmem + kACol0 + a * 64 + j * 8, bdesc, idesc, j > 0 ? 1u : 0u);
        }
        tc::commit(&d_full[d]);
        tc::commit(&a_empty[a]);
        tc::commit(&empty[s]);
        issued = i + 1;
      }
      // Unwinding after an abort: the MMAs already issued must finish before TMEM is released.
      if (*abort_flag && issued > 0) {
        const int64_t i = issued - 1;
        tc::mbar_wait(&d_full[i % kDSlots], (uint32_t)((i / kDSlots) & 1), wait_ns, nullptr);
      }
    }
  } else {
    // ---------------- dequant + epilogue ----------------
    const int dw = warp - 2;
    const int q = warp & 3;         // TMEM lane quarter this warp may access
    const int h = dw >> 2;          // k half (dequant) and m half (epilogue)
    const int r = q * 32 + lane;    // row of the tile = TMEM lane
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const int sw = (r >> 1) & 3;    // 64-byte swizzle of this row
    const int64_t gpr = K / group;  // scales per row
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    float p0 = 0.f, p1 = 0.f, p2 = 0.f;  // scale pipeline: units i, i-1, i-2
    int64_t seg_kb0 = 0;
    for (int64_t i = 0; i < n_units + kLag; ++i) {
      p2 = p1;
      p1 = p0;
      if (i < n_units) {
        const int s = (int)(i % kStages), a = (int)(i % kAStages);
        const uint32_t ph = (uint32_t)((i / kStages) & 1), aph = (uint32_t)((i / kAStages) & 1);
        const int64_t u = lo + i;
        const int64_t t = u / G, kb = u % G;
        const int64_t n = t * kTileN + r;
        if (!kScaleTma) p0 = n < N ? __half2float(scale[n * gpr + (kb * kKB) / group]) : 0.f;
        bool ok = tc::mbar_wait(&full[s], ph, wait_ns, abort_flag) &&
                  tc::mbar_wait(&a_empty[a], aph ^ 1u, wait_ns, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {  // warp-uniform: the tcgen05 ops below are .sync.aligned
          give_up();
          break;
        }
        if (kScaleTma) {  // rows past N arrive as zeros
          const __half* sst = reinterpret_cast<const __half*>(smem + (size_t)s * kStageBytes + kWBytes + kXBytes);
          p0 = __half2float(sst[r * 8 + (int)(((kb * kKB) / group) & 7)]);
        }
        const uint8_t* wrow = smem + (size_t)s * kStageBytes + r * 64;
        uint32_t regs[32];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * h + cc;
          const uint4 v = *reinterpret_cast<const uint4*>(wrow + ((c ^ sw) << 4));
          const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint32_t q4 = wd[w] >> 4;
#pragma unroll
            for (int pp = 0; pp < 4; ++pp) regs[cc * 16 + w * 4 + pp] = nib2_to_bf16x2(wd[w], q4, pp);
          }
        }
        tc::mbar_arrive(&empty[s]);
        tc::st_32x32b_x32(tmem + lane_addr + kACol0 + a * 64 + 32 * h, regs);
        tc::wait_st();
        tc::fence_before_sync();
        tc::mbar_arrive(&a_full[a]);
      }
      if (i >= kLag) {
        const int64_t e = i - kLag;
        const int d = (int)(e % kDSlots);
        const uint32_t dph = (uint32_t)((e / kDSlots) & 1);
        const bool ok = tc::mbar_wait(&d_full[d], dph, wait_ns, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          give_up();
          break;
        }
        tc::fence_after_sync();
        uint32_t dv[8];
        tc::ld_32x32b_x8(tmem + lane_addr + kDCol0 + d * 16 + 8 * h, dv);
        tc::wait_ld();
        tc::fence_before_sync();
        tc::mbar_arrive(&d_empty[d]);
        const int64_t u = lo + e;
        const int64_t t = u / G, kb = u % G;
        if (e == 0 || kb == 0) {
          seg_kb0 = kb;
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = fmaf(p2, __uint_as_float(dv[j]), acc[j]);
        if (u + 1 == hi || kb == G - 1) {
          // ---- the segment [seg_kb0, kb] of tile t ends here ----
          const int64_t n = t * kTileN + r;
          if (seg_kb0 == 0 && kb == G - 1) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int m = 8 * h + j;
              if (m < M && n < N) out[(int64_t)m * N + n] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[j]));
            }
          } else {
            // Split tile: this warp publishes its 32 rows x 8 columns of f32 partials; the warp that
            // completes the tile's count (8 warps per contributing CTA) sums the partials in CTA order.
            const int64_t c0 = cta_of_unit(t * G, U, P), c1 = cta_of_unit(t * G + G - 1, U, P);
            const int64_t nseg = c1 - c0 + 1, sidx = (int64_t)blockIdx.x - c0;
            float* slot = partials + ((t * S_max + sidx) * kMmaN) * kTileN;
#pragma unroll
            for (int j = 0; j < 8; ++j) __stcg(slot + (8 * h + j) * kTileN + r, acc[j]);
            __threadfence();
            __syncwarp();
            uint32_t last = 0;
            if (lane == 0) last = (atomicAdd(&counters[t], 1u) == (uint32_t)(nseg * 8 - 1)) ? 1u : 0u;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
              __threadfence();
              for (int rr = 0; rr < kTileN / 32; ++rr) {
                const int row = rr * 32 + lane;
                const int64_t nn = t * kTileN + row;
                for (int m = 0; m < kMmaN; ++m) {
                  float v = 0.f;
                  for (int64_t sg = 0; sg < nseg; ++sg) {
                    float* pp = partials + ((t * S_max + sg) * kMmaN + m) * kTileN + row;
                    const float pv = __ldcg(pp);
                    __stcg(pp, 0.f);  // leave the workspace all-zero: any later shape may reuse these bytes
                    v = (sg == 0) ? pv : v + pv;
                  }
                  if (m < M && nn < N) out[(int64_t)m * N + nn] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
                }
              }
              if (lane == 0) counters[t] = 0u;  // re-armed for the next launch
            }
          }
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}

// ---- host side ----
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

static int64_t host_cta_of_unit(int64_t u, int64_t U, int64_t P) {
  int64_t c = (u * P) / U;
  while (c + 1 < P && ((c + 1) * U) / P <= u) ++c;
  while (c > 0 && (c * U) / P > u) --c;
  return c;
}

struct Plan {
  int64_t tiles, G, U, P, S_max;
  size_t counters_off, partials_off, bytes;
};

static Plan make_plan(int64_t n, int64_t k) {
  Plan p{};
  p.tiles = (n + kTileN - 1) / kTileN;
  p.G = k / kKB;
  p.U = p.tiles * p.G;
  p.P = p.U < sm_count() ? p.U : sm_count();
  if (p.P < 1) p.P = 1;
  p.S_max = 1;
  for (int64_t t = 0; t < p.tiles && p.U > 0; ++t) {
    const int64_t ns = host_cta_of_unit(t * p.G + p.G - 1, p.U, p.P) - host_cta_of_unit(t * p.G, p.U, p.P) + 1;
    if (ns > p.S_max) p.S_max = ns;
  }
  p.counters_off = sizeof(WsHeader);
  p.partials_off = (p.counters_off + (size_t)p.tiles * 4 + 255) & ~size_t(255);
  p.bytes = p.partials_off + (size_t)p.tiles * p.S_max * kMmaN * kTileN * sizeof(float);
  return p;
}


// The two tensor maps of a call. Encoding is a host-side driver call of a few microseconds; the last few
// (pointer, shape) combinations are cached so a steady stream of calls on the same buffers skips it.
static int tensor_maps(const uint8_t* w, const uint16_t* x, const uint16_t* scale, int64_t m, int64_t n, int64_t k,
                       int64_t group, CUtensorMap* tmW, CUtensorMap* tmX, CUtensorMap* tmS) {
  struct Entry {
    const void* w;
    const void* x;
    const void* sc;
    int64_t m, n, k, g;
    CUtensorMap tw, tx, ts;
  };
  static std::mutex mu;
  static Entry cache[8];
  static int next = 0, used = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < used; ++i) {
      const Entry& e = cache[i];
      if (e.w == w && e.x == x && e.sc == scale && e.m == m && e.n == n && e.k == k && e.g == group) {
        *tmW = e.tw;
        *tmX = e.tx;
        *tmS = e.ts;
        return UP_OK;
      }
    }
  }
  auto enc = encode_fn();
  if (!enc) return UP_ERR_CUDA;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)(k / 2), (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)(k / 2)};
    const cuuint32_t box[2] = {kKB / 2, kTileN};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return UP_ERR_CUDA;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
    const cuuint64_t strides[1] = {(cuuint64_t)(k * 2)};
    const cuuint32_t box[2] = {64, kMmaN};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return UP_ERR_CUDA;
  }
  *tmS = *tmX;  // unused unless the scales qualify for TMA
  if ((k / group) % 8 == 0 && reinterpret_cast<uintptr_t>(scale) % 16 == 0) {
    const cuuint64_t dims[2] = {(cuuint64_t)(k / group), (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)(k / group * 2)};
    const cuuint32_t box[2] = {8, kTileN};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(tmS, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(scale), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return UP_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[next] = Entry{w, x, scale, m, n, k, group, *tmW, *tmX, *tmS};
  next = (next + 1) % 8;
  if (used < 8) ++used;
  return UP_OK;
}

}  // namespace w4
}  // namespace up

using namespace up;
using namespace up::w4;

extern "C" size_t up_sm100_w4a16_workspace_bytes(int64_t m, int64_t n, int64_t k, int64_t group) {
  (void)m;
  (void)group;
  if (n <= 0 || k <= 0) return sizeof(WsHeader);
  return make_plan(n, k).bytes;
}

extern "C" int up_sm100_w4a16_gemm(const uint8_t* w, const uint16_t* scale, const uint16_t* x, int64_t m, int64_t n,
                                   int64_t k, int64_t group, uint16_t* out, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  UP_CHECK_ARG(m >= 0 && n >= 0 && k >= 0 && group > 0);
  if (m == 0 || n == 0) return UP_OK;
  if (m > kMmaN) return UP_ERR_UNSUPPORTED;
  if (k == 0 || k % kKB != 0 || group % kKB != 0 || k % group != 0) return UP_ERR_UNSUPPORTED;
  if (k / 2 > 0x7fffffff || n > 0x7fffffff) return UP_ERR_UNSUPPORTED;
  UP_CHECK_ARG(w && scale && x && out && workspace);
  if (!aligned(w, 16) || !aligned(x, 16) || !aligned(workspace, 256)) return UP_ERR_INVALID;
  const Plan p = make_plan(n, k);
  if (workspace_bytes < p.bytes) return UP_ERR_INVALID;
  CUtensorMap tmW, tmX, tmS;
  {
    const int st = tensor_maps(w, x, scale, m, n, k, group, &tmW, &tmX, &tmS);
    if (st != UP_OK) return st;
  }
  const bool scale_tma = (k / group) % 8 == 0 && aligned(scale, 16);
  {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e);
    static std::mutex mu;
    static bool attr_set[64] = {false};
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      e = cudaFuncSetAttribute(w4a16_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(w4a16_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
      if (e != cudaSuccess) return cuda_status(e);
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
  }
  auto* base = static_cast<char*>(workspace);
  auto* hdr = reinterpret_cast<WsHeader*>(base);
  auto* counters = reinterpret_cast<uint32_t*>(base + p.counters_off);
  auto* partials = reinterpret_cast<float*>(base + p.partials_off);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto kern = scale_tma ? w4a16_kernel<true> : w4a16_kernel<false>;
  kern<<<(unsigned)p.P, kThreads, kSmemBytes, s>>>(tmW, tmX, tmS, reinterpret_cast<const __half*>(scale), out,
                                                  (int)m, n, k, group, p.U, p.G, p.S_max, hdr, counters, partials,
                                                  wait_limit_ns());
  note_launch();
  return check_launch();
}
