// w4a16.cu — int4 group-wise dequant fused into a W4A16 GEMM on the sm_100a tensor cores (tcgen05).
//
//   out[m][n] = bf16( sum_k x[m][k] * w[n][k] * scale[n][k / group] )
//
// Semantics: the dequant GEMM of crates/unpopped/tests/support/dequant.rs:1-5,163-178 generalized to f16
// group scales, bf16 activations and no zero point (i4: two per byte, low nibble = even k, sign-extended;
// tests/sub_byte_packing.rs:24-40), with f32 accumulation. The oracle sums exactly and rounds once
// (docs/accum-policies.md:8-20); this kernel is held to |got - exact_bf16| <= 1/2 ulp_bf16 + gamma * sum|x w s|.
//
// Design (swap-AB: the weight rows are the MMA's M = 128, the <= 16 activation rows its N = 16):
//  * A unit of work is one k-block (128 k) of one 128-row tile of W. The N/128 x K/128 units are split
//    evenly over one persistent CTA per SM (stream-K), so every SM streams the same share of W.
//  * Data movement: every dequant thread keeps its own copy pipeline, kPrefetch units deep, of plain
//    asynchronous 16-byte copies (cp.async): the 32 bytes of its W row for the unit, one 16-byte piece of
//    the unit's activation tile (written straight into the 128-byte-swizzled layout the MMA reads), and the
//    16-byte chunk holding its row's group scale. The tensor-memory-access (TMA) unit is not used: its
//    fixed cost of a few hundred cycles per copy would cap this kernel far below the HBM bound for tiles
//    this narrow.
//  * warps 4..11 (dequant): each thread owns one W row (its TMEM lane) and half of the k-block. It turns
//    the nibbles into exact bf16 (one prmt, one lop3 and one bf16x2 subtract per pair) and stores them into
//    tensor memory (tcgen05.st), where they are the MMA's A operand; dequantized weights never touch shared
//    memory.
//  * warps 0..3 (MMA issuers): a single thread issues only about one tcgen05.mma per ~100 cycles, much
//    slower than an M=128, N=16, K=16 MMA executes, so four warps issue in parallel: warp g runs k-steps
//    2g and 2g+1 of every unit into its own TMEM accumulator.
//  * the dequant warps, two units behind, read the unit's four accumulators (tcgen05.ld), add them, scale
//    by scale[n][k-block] in f32 and accumulate in registers. A tile finished inside one CTA is written as
//    bf16; a tile split between CTAs writes f32 partials, and whichever CTA finishes it last (an atomic
//    count) sums them in CTA order, writes bf16 and clears the partials — no CTA ever waits on another.
// Every mbarrier wait is bounded; a wait that runs out sets the workspace error word and the CTA unwinds.
#include "common.cuh"
#include "tc.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

namespace up {
namespace w4 {

constexpr int kTileN = 128;                    // W rows per tile = MMA M
constexpr int kMmaN = 16;                      // activation rows = MMA N
constexpr int kKB = 128;                       // k per unit
constexpr int kDqThreads = 256;                // 8 dequant warps: 128 rows x 2 k-halves
constexpr int kWBytes = kTileN * kKB / 2;      // 8 KiB of int4 per unit: [2 chunks][256 threads][16 B]
constexpr int kXBytes = kMmaN * kKB * 2;       // 4 KiB of bf16 per unit, 128-byte swizzled (2 atoms per 64 k)
constexpr int kSBytes = kDqThreads * 16;       // 4 KiB: each thread's 16-byte chunk of scales
constexpr int kStageBytes = kXBytes + kWBytes + kSBytes;  // 16 KiB; x first (1024-aligned)
constexpr int kPrefetch = 4;                   // units a thread's copies run ahead
constexpr int kStages = kPrefetch + 3;         // a stage is refilled 3 units after its MMAs were issued
constexpr int kRing = 4;                       // units in flight between dequant, MMA and epilogue
constexpr int kIssuers = 4;                    // MMA-issuing warps
constexpr int kTmemCols = 512;
constexpr int kACol0 = 0;                      // A (dequantized W) stages: kRing x 64 columns
constexpr int kDCol0 = kRing * 64;             // accumulators: kRing units x kIssuers x 16 columns
constexpr int kLag = 2;                        // epilogue trails the dequant by this many units
constexpr int kDq0 = kIssuers;                 // first dequant warp
constexpr int kThreads = 32 * kIssuers + kDqThreads;  // 384
constexpr int kBarBytes = 512;
constexpr size_t kSmemBytes = 1024 /*alignment slack*/ + (size_t)kStages * kStageBytes + kBarBytes;
static_assert(kStages * kStageBytes + kBarBytes + 1024 <= 227 * 1024, "shared memory");
static_assert(kStages - kPrefetch >= 3 && kRing >= kLag + 2, "pipeline distances");

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

// Position of a unit (tile t, k-block kb, scale-group index gi = kb*128/group) advanced one unit at a time
// with additions only: 64-bit division and modulo are emulated in software and would dominate the loop.
struct UnitCursor {
  int t, kb, sub, gi;  // sub = kb % (group / 128)
  __device__ __forceinline__ void init(int64_t u, int64_t G, int kpg) {
    t = (int)(u / G);
    kb = (int)(u - (int64_t)t * G);
    gi = kb / kpg;
    sub = kb - gi * kpg;
  }
  __device__ __forceinline__ void next(int G, int kpg) {
    if (++kb == G) {
      kb = 0;
      sub = 0;
      gi = 0;
      ++t;
    } else if (++sub == kpg) {
      sub = 0;
      ++gi;
    }
  }
};

// 16-byte asynchronous copy global -> shared; `valid` == false fills zeros without reading the source.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(tc::smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// kScaleChunk: K/group % 8 == 0 and the scales are 16-byte aligned, so each row's scales are whole 16-byte
// chunks and every thread copies the chunk holding its scale; otherwise each thread reads its scale with a
// plain load.
template <bool kScaleChunk>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ scale, const uint16_t* __restrict__ x,
                 uint16_t* __restrict__ out, int M, int64_t N, int64_t K, int64_t group, int64_t U, int64_t G,
                 int64_t S_max, WsHeader* hdr, uint32_t* counters, float* partials, uint64_t wait_ns) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* x_ready = reinterpret_cast<uint64_t*>(smem + (size_t)kStages * kStageBytes);  // [kStages]: 256
  uint64_t* a_full = x_ready + kStages;        // [kRing][2]: the A half h of a unit is in TMEM (128 threads)
  uint64_t* mma_done = a_full + 2 * kRing;     // [kRing]: every issuer's MMAs of the unit completed
  uint64_t* d_empty = mma_done + kRing;        // [kRing]: the epilogue has read the unit's accumulators
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d_empty + kRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t P = gridDim.x;
  const int64_t lo = ((int64_t)blockIdx.x * U) / P, hi = (((int64_t)blockIdx.x + 1) * U) / P;
  const int64_t n_units = hi - lo;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) tc::mbar_init(&x_ready[s], kDqThreads);
    for (int a = 0; a < kRing; ++a) {
      tc::mbar_init(&a_full[2 * a], kDqThreads / 2);
      tc::mbar_init(&a_full[2 * a + 1], kDqThreads / 2);
      tc::mbar_init(&mma_done[a], kIssuers);
      tc::mbar_init(&d_empty[a], kDqThreads);
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

  if (warp < kIssuers) {
    // ---------------- MMA issuers: warp g issues k-steps 2g, 2g+1 of every unit ----------------
    const int g = warp;
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(kTileN, kMmaN);
      int64_t issued = 0;
      for (int64_t i = 0; i < n_units; ++i) {
        const int s = (int)(i % kStages), a = (int)(i % kRing);
        const uint32_t ph = (uint32_t)((i / kStages) & 1), rph = (uint32_t)((i / kRing) & 1);
        if (!tc::mbar_wait(&x_ready[s], ph, wait_ns, abort_flag) ||
            !tc::mbar_wait(&a_full[2 * a + (g >> 1)], rph, wait_ns, abort_flag) ||
            !tc::mbar_wait(&d_empty[a], rph ^ 1u, wait_ns, abort_flag)) {
          give_up();
          break;
        }
        tc::fence_after_sync();
        const uint32_t xaddr = tc::smem_u32(smem + (size_t)s * kStageBytes);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = 2 * g + jj;
          const uint64_t bdesc = tc::sdesc_kmajor_sw128(xaddr + (uint32_t)((j >> 2) * 2048 + (j & 3) * 32));
          tc::mma_ts_bf16(tmem + kDCol0 + a * (16 * kIssuers) + g * 16, tmem + kACol0 + a * 64 + j * 8, bdesc, idesc,
                          jj > 0 ? 1u : 0u);
        }
        tc::commit(&mma_done[a]);
        issued = i + 1;
      }
      // Unwinding after an abort: the MMAs already issued must finish before TMEM is released.
      if (*abort_flag && issued > 0) {
        const int64_t i = issued - 1;
        tc::mbar_wait(&mma_done[i % kRing], (uint32_t)((i / kRing) & 1), wait_ns, nullptr);
      }
    }
  } else {
    // ---------------- dequant + epilogue ----------------
    const int dw = warp - kDq0;
    const int q = warp & 3;         // TMEM lane quarter this warp may access
    const int h = dw >> 2;          // k half (dequant) and m half (epilogue)
    const int r = q * 32 + lane;    // row of the tile = TMEM lane
    const int slot = dw * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const int64_t gpr = K / group;  // scales per row
    // this thread's piece of every activation tile: row xm, 16-byte chunk xc of the 256-byte row
    const int xm = slot >> 4, xc = slot & 15, xkh = xc >> 3, xcc = xc & 7;
    const uint32_t x_dst = (uint32_t)(xkh * 2048 + xm * 128 + ((xcc ^ (xm & 7)) << 4));

    const int Gi = (int)G, kpg = (int)(group / kKB);
    const int64_t wrow = K / 2;
    // issue the copies of unit j (at cursor c) into its stage
    auto issue = [&](int64_t j, const UnitCursor& c) {
      uint8_t* st = smem + (size_t)(j % kStages) * kStageBytes;
      const int64_t n = (int64_t)c.t * kTileN + r;
      const bool nv = n < N;
      const uint8_t* wsrc = w + (nv ? n : 0) * wrow + c.kb * (kKB / 2) + h * 32;
      cp_async16(st + kXBytes + slot * 16, wsrc, nv);
      cp_async16(st + kXBytes + 4096 + slot * 16, wsrc + 16, nv);
      const bool mv = xm < M;
      cp_async16(st + x_dst, x + (mv ? xm : 0) * K + c.kb * kKB + xkh * 64 + xcc * 8, mv);
      if (kScaleChunk) cp_async16(st + kXBytes + kWBytes + slot * 16, scale + (nv ? n : 0) * gpr + (c.gi & ~7), nv);
    };

    UnitCursor cn, cu, ce;  // the unit being prefetched, dequantized, and finished by the epilogue
    cn.init(lo, G, kpg);
    cu = cn;
    ce = cn;
    for (int64_t j = 0; j < kPrefetch; ++j) {
      if (j < n_units) {
        issue(j, cn);
        cn.next(Gi, kpg);
      }
      cp_async_commit();
    }

    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    float p0 = 0.f, p1 = 0.f, p2 = 0.f;  // scale pipeline: units i, i-1, i-2
    int64_t seg_kb0 = 0;
    for (int64_t i = 0; i < n_units + kLag; ++i) {
      p2 = p1;
      p1 = p0;
      if (i < n_units) {
        const int s = (int)(i % kStages), a = (int)(i % kRing);
        const uint32_t aph = (uint32_t)((i / kRing) & 1);
        // refill the stage of unit i + kPrefetch once the MMAs that read its previous contents are done
        const int64_t jn = i + kPrefetch;
        bool ok = true;
        if (jn < n_units && jn >= kStages) {
          const int64_t old = jn - kStages;  // <= i - 3
          ok = tc::mbar_wait(&mma_done[old % kRing], (uint32_t)((old / kRing) & 1), wait_ns, abort_flag);
        }
        // the A stage is free once the unit kRing earlier has been multiplied
        ok = ok && tc::mbar_wait(&mma_done[a], aph ^ 1u, wait_ns, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {  // warp-uniform: the tcgen05 ops below are .sync.aligned
          give_up();
          break;
        }
        if (jn < n_units) {
          issue(jn, cn);
          cn.next(Gi, kpg);
        }
        cp_async_commit();
        cp_async_wait<kPrefetch>();  // this thread's copies of unit i have landed
        tc::fence_proxy_async_smem();  // ... and are visible to the tensor core's reads of the activations
        tc::mbar_arrive(&x_ready[s]);
        const uint8_t* st = smem + (size_t)s * kStageBytes;
        if (kScaleChunk) {
          p0 = __half2float(reinterpret_cast<const __half*>(st + kXBytes + kWBytes + slot * 16)[cu.gi & 7]);
        } else {
          const int64_t n = (int64_t)cu.t * kTileN + r;
          p0 = n < N ? __half2float(scale[n * gpr + cu.gi]) : 0.f;
        }
        cu.next(Gi, kpg);
        uint32_t regs[32];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const uint4 v = *reinterpret_cast<const uint4*>(st + kXBytes + cc * 4096 + slot * 16);
          const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint32_t q4 = wd[wi] >> 4;
#pragma unroll
            for (int pp = 0; pp < 4; ++pp) regs[cc * 16 + wi * 4 + pp] = nib2_to_bf16x2(wd[wi], q4, pp);
          }
        }
        tc::st_32x32b_x32(tmem + lane_addr + kACol0 + a * 64 + 32 * h, regs);
        tc::wait_st();
        tc::fence_before_sync();
        tc::mbar_arrive(&a_full[2 * a + h]);
      }
      if (i >= kLag) {
        const int64_t e = i - kLag;
        const int d = (int)(e % kRing);
        const uint32_t dph = (uint32_t)((e / kRing) & 1);
        const bool ok = tc::mbar_wait(&mma_done[d], dph, wait_ns, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          give_up();
          break;
        }
        tc::fence_after_sync();
        uint32_t dv[kIssuers][8];
#pragma unroll
        for (int gg = 0; gg < kIssuers; ++gg)
          tc::ld_32x32b_x8(tmem + lane_addr + kDCol0 + d * (16 * kIssuers) + gg * 16 + 8 * h, dv[gg]);
        tc::wait_ld();
        tc::fence_before_sync();
        tc::mbar_arrive(&d_empty[d]);
        const int64_t u = lo + e;
        const int64_t t = ce.t, kb = ce.kb;
        ce.next(Gi, kpg);
        if (e == 0 || kb == 0) {
          seg_kb0 = kb;
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float sum = (__uint_as_float(dv[0][j]) + __uint_as_float(dv[1][j])) +
                            (__uint_as_float(dv[2][j]) + __uint_as_float(dv[3][j]));
          acc[j] = fmaf(p2, sum, acc[j]);
        }
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
            float* pslot = partials + ((t * S_max + sidx) * kMmaN) * kTileN;
#pragma unroll
            for (int j = 0; j < 8; ++j) __stcg(pslot + (8 * h + j) * kTileN + r, acc[j]);
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
    cp_async_wait<0>();  // no copy may still target this CTA's shared memory when it exits
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}

// ---- host side ----
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
  // 16-byte copies: W rows (K/2 bytes, a multiple of 64) and activation rows (2K bytes) start 16-byte aligned
  if (!aligned(w, 16) || !aligned(x, 16) || !aligned(workspace, 256)) return UP_ERR_INVALID;
  const Plan p = make_plan(n, k);
  if (workspace_bytes < p.bytes) return UP_ERR_INVALID;
  const bool scale_chunk = (k / group) % 8 == 0 && aligned(scale, 16);
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
  auto kern = scale_chunk ? w4a16_kernel<true> : w4a16_kernel<false>;
  kern<<<(unsigned)p.P, kThreads, kSmemBytes, s>>>(w, reinterpret_cast<const __half*>(scale), x, out, (int)m, n, k,
                                                  group, p.U, p.G, p.S_max, hdr, counters, partials, wait_limit_ns());
  note_launch();
  return check_launch();
}
