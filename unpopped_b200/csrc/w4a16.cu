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
//  * A unit of work is UK k-blocks (UK x 128 k; UK = 2 when K allows, else 1) of one 128-row tile of W. The
//    units are split evenly over one persistent CTA per SM (stream-K), so every SM streams the same share of
//    W. Each k-block keeps its own accumulator (its own group scale), but a unit's hand-offs between the roles
//    are paid once for UK k-blocks: measured, these hand-offs, not the data or the math, set the unit's time.
//  * warp 18 (W loader): one thread brings each unit's W, 128 rows x 64 UK bytes, into a ring of shared-memory
//    stages with one TMA box (128-byte swizzled when a box row is 128 bytes; rows past N read as 0). The ring holds
//    128 KiB, far ahead of use, and the load path of the SM stays free for everything else: the plain 16-byte loads
//    this replaced put 32 rows' worth of sector requests behind every warp instruction.
//  * warps 0..7 (dequant): warp w owns TMEM lane quarter w % 4 and k-quarters 2 (w / 4) and 2 (w / 4) + 1, so
//    thread (w, lane) owns row 32 (w % 4) + lane of the tile and 64 UK k of every unit: 32 UK bytes of W, read from
//    the W stage (conflict free under the swizzle). Each k-quarter is released to its issuer as soon as it is in
//    tensor memory. (Sixteen warps, one k-quarter each, measured 1 % slower and left fewer registers per thread.) It turns the nibbles into exact bf16 (a shift, one lop3 and one bf16x2 subtract per
//    pair, pairing k with k + 4) and stores them into tensor memory (tcgen05.st) as the MMA's A operand, whose k
//    order inside each group of 8 is therefore 0,4,1,5,2,6,3,7.
//  * warps 8..11 (MMA issuers): a single thread issues only about one tcgen05.mma per ~100 cycles, so four
//    threads share a unit's 8 UK k-steps as pipelines: issuer g runs the 2 UK k-steps of k-quarter g into
//    its k-block's accumulator after the issuer before it in that k-block has issued its own (an mbarrier
//    hand-off between tcgen05.fence::before_thread_sync and ::after_thread_sync orders them), so each
//    k-block ends in one accumulator while several units are in issue at once. (Four separate accumulators per unit were measured
//    slower: the epilogue's reads of four times the tensor-memory data cost more than the hand-offs.)
//  * warp 16 (activation loader): one thread brings each unit's [16 x 128 UK] activation tile into a ring of
//    shared-memory stages with 2 UK TMA boxes, 128-byte swizzled as the MMA reads it; rows past M read as 0.
//  * warp 19 (activation permuter): rewrites each landed 16-byte chunk (8 k) in place to the k order 0,4,1,5,2,6,
//    3,7 of the A operand (the swizzle moves whole chunks, so it is unaffected), then releases the stage to the MMA.
//  * warp 17 (scale loader): one thread brings each unit's scales, f16 groups [g0, g0 + 16) of its 128 rows with
//    g0 = the unit's first group rounded down to a multiple of 8, into a ring of shared-memory slots with one TMA
//    box. (A scale row stride that is not a multiple of 16 bytes cannot be a TMA tensor; then the warp's lanes load
//    and store the same slot layout.) Loading them in the epilogue put a global-load latency on every unit.
//  * warps 12..15 (epilogue): read the unit's accumulators (tcgen05.ld), scale each by scale[n][k-block] in
//    f32 and accumulate in registers, k-block by k-block. A tile finished inside one CTA is written as bf16;
//    a tile split between CTAs writes f32 partials, and whichever CTA finishes it last (an atomic count)
//    sums them in CTA order, writes bf16 and clears the partials — no CTA ever waits on another.
// Every mbarrier wait is bounded; a wait that runs out sets the workspace error word and the CTA unwinds.
#include "common.cuh"
#include "tc.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstring>
#include <mutex>

namespace up {
namespace w4 {

constexpr int kTileN = 128;                      // W rows per tile = MMA M
constexpr int kMmaN = 16;                        // activation rows = MMA N
constexpr int kKB = 128;                         // k per unit
constexpr int kDqWarps = 8;                      // warps 0..7
constexpr int kIssuers = 4;                      // warps 8..11
constexpr int kEpiWarps = 4;                     // warps 12..15
constexpr int kIss0 = kDqWarps, kEpi0 = kIss0 + kIssuers, kXWarp = kEpi0 + kEpiWarps, kScWarp = kXWarp + 1;
constexpr int kWWarp = kScWarp + 1, kXpWarp = kWWarp + 1;
constexpr int kThreads = 32 * (kXpWarp + 1);     // 640
constexpr int kScRing = 8;                       // units of scales staged in shared memory
constexpr int kScCols = 16;                      // f16 scales per row in a slot: groups [g0, g0 + 16), g0 % 8 == 0
constexpr uint32_t kSleepNs = 64;                // pause between polls of a waiting dequant/epilogue/loader warp
constexpr int kXBytes = kMmaN * kKB * 2;         // 4 KiB of bf16 per k-block: two 128-byte-swizzled boxes of 64 k
constexpr int kTmemCols = 512;

// The layout for units of UK k-blocks.
template <int UK>
struct Cfg {
  static constexpr int kACols = 64 * UK;               // A (dequantized W) columns per unit
  static constexpr int kDCols = kMmaN * UK;            // accumulator columns per unit: one 16-column block per k-block
  static constexpr int kRing = UK == 1 ? 6 : 3;        // units in flight between dequant, MMA and epilogue
  static constexpr int kACol0 = 0;
  static constexpr int kDCol0 = kRing * kACols;
  static constexpr int kXUnit = kXBytes * UK;          // activation bytes per unit
  static constexpr int kXStages = 8 / UK;              // 32 KiB of activation stages either way
  static constexpr int kChain = kIssuers / UK;         // issuers chained into one k-block's accumulator
  static constexpr int kWRow = 64 * UK;                // bytes of one W row in a unit
  static constexpr int kWUnit = kTileN * kWRow;        // W bytes per unit (one TMA box of 128 rows)
  static constexpr int kWStages = 16 / UK;             // 128 KiB of W in flight either way
  // mbarriers: x_full, x_empty [kXStages]; a_full [kRing][4]; mma_done, d_empty [kRing]; hand [kIssuers][kRing];
  // seg_in, seg_out; then the TMEM address word, the abort word and the fix-up verdict
  static constexpr int kNumBars =
      3 * kXStages + 4 * kRing + 2 * kRing + kIssuers * kRing + 2 * kScRing + 2 * kWStages + 2;
  static_assert(kDCol0 + kRing * kDCols <= kTmemCols, "tensor memory");
};
constexpr int kBarBytes = 2048;
constexpr size_t kWBytes = (size_t)16 * kTileN * 64;  // the W ring: Cfg<UK>::kWStages * kWUnit for either UK
static_assert(Cfg<1>::kNumBars * 8 + 12 <= kBarBytes && Cfg<2>::kNumBars * 8 + 12 <= kBarBytes, "barrier region");
constexpr size_t kScSlot = (size_t)kTileN * kScCols * 2;  // one TMA box of 128 rows x 16 f16
constexpr size_t kScBytes = kScRing * kScSlot;
constexpr size_t kSmemBytes = 1024 /*alignment slack*/ + (size_t)8 * kXBytes + kWBytes + kScBytes + kBarBytes;
static_assert(kEpi0 % 4 == 0, "epilogue warp e reads TMEM lane quarter e % 4");

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

// The eight signed nibbles of one word (low nibble = even k) -> four exact bf16x2 in the k order 0,4,1,5,2,6,3,7:
// nibbles k and k + 4 sit at the same position of the word's two 16-bit halves, so one mask of the word shifted
// by 4j takes the pair (j, j + 4) with no byte permute. Each becomes the mantissa of 128 + (n ^ 8) and one bf16x2
// subtract of 136 gives n, exactly. The activations are permuted the same way (see the activation permuter), so
// the MMA's products are the same set. Seven integer ops per word instead of nine.
__device__ __forceinline__ void nib8_to_bf16x2_k4(uint32_t w, uint32_t* out) {
  const uint32_t c136 = 0x43084308u;
  const __nv_bfloat162 b136 = *reinterpret_cast<const __nv_bfloat162*>(&c136);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t t = lop3_and_xor(w >> (4 * j), 0x000f000fu, 0x43084308u);
    __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&t);
    v = __hsub2(v, b136);
    out[j] = *reinterpret_cast<const uint32_t*>(&v);
  }
}

// Position of a unit of UK k-blocks (tile t, first k-block kb, scale-group index gi = kb*128/group) advanced
// one unit at a time with additions only: 64-bit division and modulo are emulated in software and would
// dominate the loops. G (k-blocks per tile) is a multiple of UK.
template <int UK>
struct UnitCursor {
  int t, kb, sub, gi;  // sub = kb % (group / 128)
  __device__ __forceinline__ void init(int64_t u, int64_t G, int kpg) {
    const int64_t GU = G / UK;
    t = (int)(u / GU);
    kb = (int)(u - (int64_t)t * GU) * UK;
    gi = kb / kpg;
    sub = kb - gi * kpg;
  }
  __device__ __forceinline__ void next(int G, int kpg) {
    kb += UK;
    if (kb == G) {
      kb = 0;
      sub = 0;
      gi = 0;
      ++t;
      return;
    }
#pragma unroll
    for (int h = 0; h < UK; ++h)
      if (++sub == kpg) {
        sub = 0;
        ++gi;
      }
  }
  // scale-group index of k-block kb + h of the unit
  __device__ __forceinline__ int gi_at(int h, int kpg) const { return gi + (sub + h) / kpg; }
};

// The order in which a CTA takes its units [lo, hi): first the units of its last tile when that tile is split with
// the next CTA ([rot, hi), rot the tile's first unit), then [lo, rot). Both parts of every split tile are then done
// early in both CTAs, so the split-tile fix-up (a chain of dependent global round trips) happens while other work
// runs, and each CTA ends on whole tiles. Every role that needs a unit's position walks this same order.
template <int UK>
struct RotCursor {
  UnitCursor<UK> c;
  int64_t lo, rot, n_first, e;
  __device__ __forceinline__ void init(int64_t lo_, int64_t hi_, int64_t rot_, int64_t G, int kpg) {
    lo = lo_;
    rot = rot_;
    n_first = hi_ - rot_;
    e = 0;
    c.init(rot_, G, kpg);
  }
  __device__ __forceinline__ void next(int64_t G, int kpg) {
    if (++e == n_first) c.init(lo, G, kpg);
    else c.next((int)G, kpg);
  }
  __device__ __forceinline__ int64_t unit() const { return e < n_first ? rot + e : lo + (e - n_first); }
};

// The end of a tile segment in the epilogue (all kEpiWarps epilogue warps reach it together):
// a whole tile is written as bf16. For a tile split between CTAs, each epilogue thread publishes its row's
// 16 f32 partials; the epilogue warps meet on an mbarrier (seg_in, one arrival per warp), one thread counts
// this CTA in and announces whether it completed the count (seg_out); in the CTA that did, every epilogue
// thread sums its own row over the contributing CTAs in CTA order (a segment's loads issued together),
// writes bf16 and clears the partials. `nfix` counts this warp's split-tile ends (the barriers' phase).
// Both waits are bounded; false means the CTA is giving up.
__device__ __forceinline__ bool finish_segment(const float (&acc)[kMmaN], int64_t t, bool whole, int r, int lane,
                                               int M, int64_t N, int64_t U, int64_t GU, int64_t P, int64_t S_max,
                                               uint16_t* out, uint32_t* counters, float* partials, uint64_t* seg_in,
                                               uint64_t* seg_out, volatile uint32_t* s_last, uint32_t& nfix,
                                               uint64_t wait_ns, volatile int* abort_flag) {
  const int64_t n = t * kTileN + r;
  if (whole) {
#pragma unroll
    for (int m = 0; m < kMmaN; ++m)
      if (m < M && n < N) out[(int64_t)m * N + n] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[m]));
    return true;
  }
  const int64_t c0 = cta_of_unit(t * GU, U, P), c1 = cta_of_unit(t * GU + GU - 1, U, P);
  const int64_t nseg = c1 - c0 + 1, sidx = (int64_t)blockIdx.x - c0;
  float* tile_parts = partials + t * S_max * kMmaN * kTileN;
#pragma unroll
  for (int m = 0; m < kMmaN; ++m) __stcg(tile_parts + (sidx * kMmaN + m) * kTileN + r, acc[m]);
  __threadfence();
  __syncwarp();
  const uint32_t ph = nfix & 1u;
  ++nfix;
  if (lane == 0) tc::mbar_arrive(seg_in);
  if (!__all_sync(0xffffffffu, tc::mbar_wait(seg_in, ph, wait_ns, abort_flag))) return false;
  if (r == 0) {
    *s_last = (atomicAdd(&counters[t], 1u) == (uint32_t)(nseg - 1)) ? 1u : 0u;
    tc::mbar_arrive(seg_out);
  }
  if (!__all_sync(0xffffffffu, tc::mbar_wait(seg_out, ph, wait_ns, abort_flag))) return false;
  if (!*s_last) return true;
  __threadfence();
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // 8 activation rows at a time (register budget)
    float v[8];
    for (int64_t sg = 0; sg < nseg; ++sg) {
      float pv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) pv[j] = __ldcg(tile_parts + (sg * kMmaN + 8 * half + j) * kTileN + r);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = (sg == 0) ? pv[j] : v[j] + pv[j];
        __stcg(tile_parts + (sg * kMmaN + 8 * half + j) * kTileN + r, 0.f);  // all-zero again for any later shape
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = 8 * half + j;
      if (m < M && n < N) out[(int64_t)m * N + n] = __bfloat16_as_ushort(__float2bfloat16_rn(v[j]));
    }
  }
  if (r == 0) counters[t] = 0u;  // re-armed for the next launch
  return true;
}

template <int UK>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                 const __grid_constant__ CUtensorMap smap, int scale_tma,
                 const __half* __restrict__ scale, uint16_t* __restrict__ out, int M, int64_t N, int64_t K,
                 int64_t group, int64_t U, int64_t G, int64_t S_max, WsHeader* hdr, uint32_t* counters,
                 float* partials, uint64_t wait_ns) {
  using C = Cfg<UK>;
  constexpr int kRing = C::kRing, kXStages = C::kXStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* xs = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wst = xs + (size_t)kXStages * C::kXUnit;  // [kWStages] W boxes (1024-byte aligned: 32 KiB after xs)
  __half* scs = reinterpret_cast<__half*>(wst + kWBytes);  // [kScRing][128][kScCols] f16 scales
  uint64_t* x_full = reinterpret_cast<uint64_t*>(wst + kWBytes + kScBytes);  // [kXStages]: TMA landed
  uint64_t* x_empty = x_full + kXStages;        // [kXStages]: the stage's MMAs completed (chain ends' commits)
  uint64_t* a_full = x_empty + kXStages;        // [kRing][4]: k-quarter q of the unit's A is in TMEM (4 warps)
  uint64_t* mma_done = a_full + 4 * kRing;      // [kRing]: all of the unit's MMAs completed
  uint64_t* d_empty = mma_done + kRing;         // [kRing]: the epilogue has read the unit's accumulators
  uint64_t* hand = d_empty + kRing;             // [kIssuers][kRing]: issuer g has issued the unit's k-quarter g
  uint64_t* sc_full = hand + kIssuers * kRing;  // [kScRing]: the scale warp has written the unit's scales
  uint64_t* sc_empty = sc_full + kScRing;       // [kScRing]: every epilogue warp has read them
  uint64_t* w_full = sc_empty + kScRing;        // [kWStages]: the unit's W box has landed
  uint64_t* w_empty = w_full + C::kWStages;     // [kWStages]: every dequant warp has read it
  uint64_t* x_raw = w_empty + C::kWStages;      // [kXStages]: the activation TMA has landed (not yet permuted)
  uint64_t* seg_in = x_raw + kXStages;          // split-tile end: every epilogue warp has published
  uint64_t* seg_out = seg_in + 1;               // split-tile end: the count verdict is in s_last
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(seg_out + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile uint32_t* s_last = reinterpret_cast<volatile uint32_t*>(tmem_slot + 2);  // split-tile fix-up verdict

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t P = gridDim.x;
  const int64_t lo = ((int64_t)blockIdx.x * U) / P, hi = (((int64_t)blockIdx.x + 1) * U) / P;
  const int64_t n_units = hi - lo;
  // the first unit of this CTA's last tile when that tile starts inside the range and is cut by its end
  const int64_t GUk = G / UK, t1s = (hi / GUk) * GUk;
  const int64_t rot = (t1s > lo && t1s < hi) ? t1s : lo;
  const int Gi = (int)G, kpg = (int)(group / kKB);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kXStages; ++s) {
      tc::mbar_init(&x_full[s], 1);
      tc::mbar_init(&x_empty[s], UK);
    }
    for (int a = 0; a < kRing; ++a) {
      for (int q = 0; q < 4; ++q) tc::mbar_init(&a_full[4 * a + q], 4);
      tc::mbar_init(&mma_done[a], UK);
      tc::mbar_init(&d_empty[a], kEpiWarps);
      for (int g = 0; g < kIssuers; ++g) tc::mbar_init(&hand[g * kRing + a], 1);
    }
    for (int q = 0; q < kScRing; ++q) {
      tc::mbar_init(&sc_full[q], 1);
      tc::mbar_init(&sc_empty[q], kEpiWarps);
    }
    for (int q = 0; q < C::kWStages; ++q) {
      tc::mbar_init(&w_full[q], 1);
      tc::mbar_init(&w_empty[q], kDqWarps);
    }
    for (int q = 0; q < kXStages; ++q) tc::mbar_init(&x_raw[q], 1);
    tc::mbar_init(seg_in, kEpiWarps);
    tc::mbar_init(seg_out, 1);
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

  if (warp < kDqWarps) {
    // ---------------- dequant: row 32 (warp % 4) + lane, k-quarters 2 (warp / 4) and 2 (warp / 4) + 1 ----------------
    const int lq = warp & 3, kh = warp >> 2;  // k-half kh: k-quarters 2 kh and 2 kh + 1
    const int r = lq * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(lq * 32) << 16;
    // this thread's 16-byte chunks of its row in a W stage: chunk UK kq + h, 128-byte swizzled when UK = 2
    const uint8_t* wrow = wst + (size_t)r * C::kWRow;
    bool ok = true;
    for (int64_t i = 0; ok && i < n_units; ++i) {
      {
        const int sw = (int)(i % C::kWStages);
        if (!__all_sync(0xffffffffu, tc::mbar_wait(&w_full[sw], (uint32_t)((i / C::kWStages) & 1), wait_ns,
                                                   abort_flag))) {
          give_up();
          break;
        }
      }
      uint4 cur[2][UK];
#pragma unroll
      for (int qq = 0; qq < 2; ++qq)
#pragma unroll
        for (int h = 0; h < UK; ++h) {
          const int c = UK * (2 * kh + qq) + h;
          const int cs = UK == 2 ? (c ^ (r & 7)) : c;
          cur[qq][h] = *reinterpret_cast<const uint4*>(wrow + (size_t)(i % C::kWStages) * C::kWUnit + (cs << 4));
        }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&w_empty[i % C::kWStages]);
      {
        const int a = (int)(i % kRing);
        const uint32_t aph = (uint32_t)((i / kRing) & 1);
        // the A stage is free once the unit kRing earlier has been multiplied
        const bool good = tc::mbar_wait_sleepy(&mma_done[a], aph ^ 1u, wait_ns, abort_flag, kSleepNs);
        if (!__all_sync(0xffffffffu, good)) {  // warp-uniform: the tcgen05 ops below are .sync.aligned
          give_up();
          ok = false;
          break;
        }
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
          const int kq = 2 * kh + qq;
#pragma unroll
          for (int h = 0; h < UK; ++h) {
            uint32_t regs[16];
            const uint32_t wd[4] = {cur[qq][h].x, cur[qq][h].y, cur[qq][h].z, cur[qq][h].w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) nib8_to_bf16x2_k4(wd[wi], regs + 4 * wi);
            tc::st_32x32b_x16(tmem + lane_addr + C::kACol0 + a * C::kACols + 16 * (UK * kq + h), regs);
          }
          tc::wait_st();
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&a_full[4 * a + kq]);
        }
      }
    }
  } else if (warp < kEpi0) {
    // ------- MMA issuers: issuer g runs the 2 UK k-steps of k-quarter g, in its k-block's chain -------
    const int g = warp - kIss0;
    const int hk = (UK * g) / 4;          // the k-block (accumulator) of this issuer's k-steps
    const int pos = g % C::kChain;        // place in that k-block's chain
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(kTileN, kMmaN);
      int64_t issued = 0;
      for (int64_t i = 0; i < n_units; ++i) {
        const int a = (int)(i % kRing), s = (int)(i % kXStages);
        const uint32_t rph = (uint32_t)((i / kRing) & 1), xph = (uint32_t)((i / kXStages) & 1);
        // the first issuer of a chain starts the accumulator once the epilogue has read the slot's previous
        // unit; the others add to it after the issuer before them
        const bool ready = tc::mbar_wait(&a_full[4 * a + g], rph, wait_ns, abort_flag) &&
                           tc::mbar_wait(&x_full[s], xph, wait_ns, abort_flag) &&
                           (pos == 0 ? tc::mbar_wait(&d_empty[a], rph ^ 1u, wait_ns, abort_flag)
                                     : tc::mbar_wait(&hand[(g - 1) * kRing + a], rph, wait_ns, abort_flag));
        if (!ready) {
          give_up();
          break;
        }
        tc::fence_after_sync();
        const uint32_t xaddr = tc::smem_u32(xs + (size_t)s * C::kXUnit);
#pragma unroll
        for (int jj = 0; jj < 2 * UK; ++jj) {
          const int j = 2 * UK * g + jj;  // k-step: 16 k = 32 bytes of a 128-byte swizzle atom row
          const uint64_t bdesc = tc::sdesc_kmajor_sw128(xaddr + (uint32_t)((j >> 2) * 2048 + (j & 3) * 32));
          tc::mma_ts_bf16(tmem + C::kDCol0 + a * C::kDCols + hk * kMmaN, tmem + C::kACol0 + a * C::kACols + j * 8,
                          bdesc, idesc, (pos > 0 || jj > 0) ? 1u : 0u);
        }
        if (pos + 1 < C::kChain) {
          tc::fence_before_sync();
          tc::mbar_arrive(&hand[g * kRing + a]);
        } else {
          // a chain's MMAs run in issue order, so its last issuer's completing covers all of them
          tc::commit(&mma_done[a]);
          tc::commit(&x_empty[s]);
        }
        issued = i + 1;
      }
      // Unwinding after an abort: the MMAs already issued must finish before TMEM is released.
      if (*abort_flag && issued > 0) {
        const int64_t i = issued - 1;
        tc::mbar_wait(&mma_done[i % kRing], (uint32_t)((i / kRing) & 1), wait_ns, nullptr);
      }
    }
  } else if (warp < kXWarp) {
    // ---------------- epilogue: row 32 (warp % 4) + lane, all 16 activation rows ----------------
    const int lq = warp & 3;
    const int r = lq * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(lq * 32) << 16;
    const int64_t GU = G / UK;      // units per tile
    RotCursor<UK> ce;               // the unit being finished
    ce.init(lo, hi, rot, G, kpg);
    float acc[kMmaN];
#pragma unroll
    for (int j = 0; j < kMmaN; ++j) acc[j] = 0.f;
    int64_t seg_kb0 = 0;
    uint32_t nfix = 0;
    for (int64_t e = 0; e < n_units; ++e) {
      const int d = (int)(e % kRing);
      const uint32_t dph = (uint32_t)((e / kRing) & 1);
      // this row's scales of the unit, staged by the scale warp; the slot is released once they are read
      const int q = (int)(e % kScRing);
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&sc_full[q], (uint32_t)((e / kScRing) & 1), wait_ns, abort_flag))) {
        give_up();
        break;
      }
      float sc[UK];
#pragma unroll
      for (int h = 0; h < UK; ++h)
        sc[h] = __half2float(scs[((size_t)q * kTileN + r) * kScCols + (ce.c.gi_at(h, kpg) - (ce.c.gi & ~7))]);
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&sc_empty[q]);
      const bool good = tc::mbar_wait_sleepy(&mma_done[d], dph, wait_ns, abort_flag, kSleepNs);
      if (!__all_sync(0xffffffffu, good)) {
        give_up();
        break;
      }
      tc::fence_after_sync();
      const int64_t t = ce.c.t, kb = ce.c.kb;
      if (e == 0 || e == hi - rot || kb == 0) {  // a segment starts: the range's start, the wrap, a tile
        seg_kb0 = kb;
#pragma unroll
        for (int j = 0; j < kMmaN; ++j) acc[j] = 0.f;
      }
#pragma unroll
      for (int h = 0; h < UK; ++h) {  // k-block by k-block, in k order
        uint32_t dv[kMmaN];
        tc::ld_32x32b_x16(tmem + lane_addr + C::kDCol0 + d * C::kDCols + h * kMmaN, dv);
        tc::wait_ld();
#pragma unroll
        for (int j = 0; j < kMmaN; ++j) acc[j] = fmaf(sc[h], __uint_as_float(dv[j]), acc[j]);
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&d_empty[d]);
      const int64_t u = ce.unit();
      ce.next(Gi, kpg);
      if (u + 1 == hi || kb + UK == G)  // the segment [seg_kb0, kb + UK) of tile t ends here
        if (!finish_segment(acc, t, seg_kb0 == 0 && kb + UK == G, r, lane, M, N, U, GU, P, S_max, out, counters,
                            partials, seg_in, seg_out, s_last, nfix, wait_ns, abort_flag)) {
          give_up();
          break;
        }
    }
  } else if (warp == kScWarp) {
    // ------- scale warp: stages each unit's scales, f16 groups [g0, g0 + 16) of its 128 rows, g0 = gi & ~7 -------
    // With a scale row stride of a multiple of 16 bytes one thread brings them in with one TMA box per unit;
    // otherwise the lanes load and store them (rows l, l + 32, l + 64, l + 96).
    RotCursor<UK> rs;
    rs.init(lo, hi, rot, G, kpg);
    const UnitCursor<UK>& cs = rs.c;
    if (scale_tma) {
      if (lane == 0) {
        tc::tma_prefetch_desc(&smap);
        int64_t issued = 0;
        for (int64_t i = 0; i < n_units; ++i) {
          const int q = (int)(i % kScRing);
          if (!tc::mbar_wait_sleepy(&sc_empty[q], (uint32_t)(((i / kScRing) & 1) ^ 1), wait_ns, abort_flag,
                                    kSleepNs)) {
            give_up();
            break;
          }
          tc::mbar_arrive_expect_tx(&sc_full[q], (uint32_t)kScSlot);
          tc::tma_load_2d(scs + (size_t)q * kTileN * kScCols, &smap, &sc_full[q], cs.gi & ~7,
                          cs.t * kTileN);
          rs.next(Gi, kpg);
          issued = i + 1;
        }
        for (int64_t j = issued > kScRing ? issued - kScRing : 0; j < issued; ++j)
          tc::mbar_wait(&sc_full[j % kScRing], (uint32_t)((j / kScRing) & 1), wait_ns, nullptr);
      }
    } else {
      const int64_t gpr = K / group;  // scales per row
      for (int64_t i = 0; i < n_units; ++i) {
        const int q = (int)(i % kScRing);
        if (!__all_sync(0xffffffffu, tc::mbar_wait_sleepy(&sc_empty[q], (uint32_t)(((i / kScRing) & 1) ^ 1), wait_ns,
                                                          abort_flag, kSleepNs))) {
          give_up();
          break;
        }
        __half* slot = scs + (size_t)q * kTileN * kScCols;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int row = lane + 32 * j;
          const int64_t n = (int64_t)cs.t * kTileN + row;
#pragma unroll
          for (int h = 0; h < UK; ++h) {
            const int gi = cs.gi_at(h, kpg);
            slot[row * kScCols + (gi - (cs.gi & ~7))] = n < N ? scale[n * gpr + gi] : __ushort_as_half(0);
          }
        }
        rs.next(Gi, kpg);
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&sc_full[q]);
      }
    }
  } else if (warp == kWWarp) {
    // ---------------- W loader: one TMA box of 128 rows x 64 UK bytes per unit ----------------
    if (lane == 0) {
      tc::tma_prefetch_desc(&wmap);
      RotCursor<UK> rw;
      rw.init(lo, hi, rot, G, kpg);
      const UnitCursor<UK>& cw = rw.c;
      int64_t issued = 0;
      for (int64_t i = 0; i < n_units; ++i) {
        const int sw = (int)(i % C::kWStages);
        if (!tc::mbar_wait_sleepy(&w_empty[sw], (uint32_t)(((i / C::kWStages) & 1) ^ 1), wait_ns, abort_flag,
                                  kSleepNs)) {
          give_up();
          break;
        }
        tc::mbar_arrive_expect_tx(&w_full[sw], C::kWUnit);
        tc::tma_load_2d(wst + (size_t)sw * C::kWUnit, &wmap, &w_full[sw], cw.kb * (kKB / 2), cw.t * kTileN);
        rw.next(Gi, kpg);
        issued = i + 1;
      }
      // every issued load must land before this CTA's shared memory is released
      for (int64_t j = issued > C::kWStages ? issued - C::kWStages : 0; j < issued; ++j)
        tc::mbar_wait(&w_full[j % C::kWStages], (uint32_t)((j / C::kWStages) & 1), wait_ns, nullptr);
    }
  } else if (warp == kXpWarp) {
    // ------- activation permuter: each 16-byte chunk (8 k) of a landed stage to the k order 0,4,1,5,2,6,3,7 -------
    // in place (the swizzle moves whole chunks, so it is unaffected), matching the dequant's nibble pairing
    for (int64_t i = 0; i < n_units; ++i) {
      const int s = (int)(i % kXStages);
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&x_raw[s], (uint32_t)((i / kXStages) & 1), wait_ns, abort_flag))) {
        give_up();
        break;
      }
      uint4* chunk = reinterpret_cast<uint4*>(xs + (size_t)s * C::kXUnit);
#pragma unroll 4
      for (int c = lane; c < C::kXUnit / 16; c += 32) {
        const uint4 v = chunk[c];  // bf16 pairs (k0,k1) (k2,k3) (k4,k5) (k6,k7)
        uint4 o;
        o.x = __byte_perm(v.x, v.z, 0x5410);  // (k0, k4)
        o.y = __byte_perm(v.x, v.z, 0x7632);  // (k1, k5)
        o.z = __byte_perm(v.y, v.w, 0x5410);  // (k2, k6)
        o.w = __byte_perm(v.y, v.w, 0x7632);  // (k3, k7)
        chunk[c] = o;
      }
      tc::fence_proxy_async_smem();  // the MMA reads the stage through the async proxy
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&x_full[s]);
    }
  } else {
    // ---------------- activation loader: 2 UK TMA boxes per unit ----------------
    if (lane == 0) {
      tc::tma_prefetch_desc(&xmap);
      RotCursor<UK> rx;
      rx.init(lo, hi, rot, G, kpg);
      const UnitCursor<UK>& cx = rx.c;
      int64_t issued = 0;
      for (int64_t i = 0; i < n_units; ++i) {
        const int s = (int)(i % kXStages);
        if (!tc::mbar_wait_sleepy(&x_empty[s], (uint32_t)(((i / kXStages) & 1) ^ 1), wait_ns, abort_flag, kSleepNs)) {
          give_up();
          break;
        }
        uint8_t* dst = xs + (size_t)s * C::kXUnit;
        tc::mbar_arrive_expect_tx(&x_raw[s], C::kXUnit);
#pragma unroll
        for (int bx = 0; bx < 2 * UK; ++bx)
          tc::tma_load_2d(dst + bx * (kXBytes / 2), &xmap, &x_raw[s], cx.kb * kKB + bx * (kKB / 2), 0);
        rx.next(Gi, kpg);
        issued = i + 1;
      }
      // every issued load must land before this CTA's shared memory is released
      for (int64_t j = issued > kXStages ? issued - kXStages : 0; j < issued; ++j)
        tc::mbar_wait(&x_raw[j % kXStages], (uint32_t)((j / kXStages) & 1), wait_ns, nullptr);
    }
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
  int64_t tiles, G, UK, GU, U, P, S_max;  // G k-blocks per tile, UK k-blocks per unit, GU units per tile
  size_t counters_off, partials_off, bytes;
};

static Plan make_plan(int64_t n, int64_t k) {
  Plan p{};
  p.tiles = (n + kTileN - 1) / kTileN;
  p.G = k / kKB;
  p.UK = (p.G % 2 == 0) ? 2 : 1;
  p.GU = p.G / p.UK;
  p.U = p.tiles * p.GU;
  p.P = p.U < sm_count() ? p.U : sm_count();
  if (p.P < 1) p.P = 1;
  p.S_max = 1;
  for (int64_t t = 0; t < p.tiles && p.U > 0; ++t) {
    const int64_t ns =
        host_cta_of_unit(t * p.GU + p.GU - 1, p.U, p.P) - host_cta_of_unit(t * p.GU, p.U, p.P) + 1;
    if (ns > p.S_max) p.S_max = ns;
  }
  p.counters_off = sizeof(WsHeader);
  p.partials_off = (p.counters_off + (size_t)p.tiles * 4 + 255) & ~size_t(255);
  p.bytes = p.partials_off + (size_t)p.tiles * p.S_max * kMmaN * kTileN * sizeof(float);
  return p;
}

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
  // TMA boxes of W rows (K/2 bytes, a multiple of 64) and of activation rows (2K bytes)
  if (!aligned(w, 16) || !aligned(x, 16) || !aligned(workspace, 256)) return UP_ERR_INVALID;
  const Plan p = make_plan(n, k);
  if (workspace_bytes < p.bytes) return UP_ERR_INVALID;
  auto enc = encode_fn();
  if (enc == nullptr) return fail_with(UP_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  // activations as a [M, K] bf16 tensor; boxes of 16 rows x 64 k, 128-byte swizzled; rows >= M read as zero
  CUtensorMap xmap;
  const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
  const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  const cuuint32_t box[2] = {(cuuint32_t)(kKB / 2), (cuuint32_t)kMmaN};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult cr = enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(x), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail_with(UP_ERR_CUDA, "cuTensorMapEncodeTiled refused the activation tensor map");
  // W as a [N, K/2] byte tensor; boxes of 128 rows x 64 UK bytes (one unit), 128-byte swizzled when a box row is
  // 128 bytes; rows >= N read as zero
  CUtensorMap wmap;
  {
    const cuuint64_t wdims[2] = {(cuuint64_t)(k / 2), (cuuint64_t)n};
    const cuuint64_t wstrides[1] = {(cuuint64_t)(k / 2)};
    const cuuint32_t wbox[2] = {(cuuint32_t)(64 * p.UK), (cuuint32_t)kTileN};
    const CUresult wr = enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), wdims, wstrides, wbox,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            p.UK == 2 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (wr != CUDA_SUCCESS) return fail_with(UP_ERR_CUDA, "cuTensorMapEncodeTiled refused the weight tensor map");
  }
  // scales as a [N, K / group] f16 tensor; boxes of 128 rows x 16 groups. A TMA row stride must be a multiple of
  // 16 bytes; other shapes stage the scales with plain loads.
  CUtensorMap smap;
  std::memset(&smap, 0, sizeof(smap));
  const int64_t gpr = k / group;
  const int scale_tma = (gpr % 8 == 0 && aligned(scale, 16)) ? 1 : 0;
  if (scale_tma) {
    const cuuint64_t sdims[2] = {(cuuint64_t)gpr, (cuuint64_t)n};
    const cuuint64_t sstrides[1] = {(cuuint64_t)gpr * 2};
    const cuuint32_t sbox[2] = {(cuuint32_t)kScCols, (cuuint32_t)kTileN};
    const CUresult sr = enc(&smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(scale), sdims, sstrides,
                            sbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (sr != CUDA_SUCCESS) return fail_with(UP_ERR_CUDA, "cuTensorMapEncodeTiled refused the scale tensor map");
  }
  {
    cudaError_t e = ensure_smem_attr((const void*)w4a16_kernel<1>, (int)kSmemBytes);
    if (e == cudaSuccess) e = ensure_smem_attr((const void*)w4a16_kernel<2>, (int)kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
  }
  auto* base = static_cast<char*>(workspace);
  auto* hdr = reinterpret_cast<WsHeader*>(base);
  auto* counters = reinterpret_cast<uint32_t*>(base + p.counters_off);
  auto* partials = reinterpret_cast<float*>(base + p.partials_off);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto kern = p.UK == 2 ? w4a16_kernel<2> : w4a16_kernel<1>;
  kern<<<(unsigned)p.P, kThreads, kSmemBytes, s>>>(xmap, wmap, smap, scale_tma, reinterpret_cast<const __half*>(scale),
                                                   out, (int)m, n, k,
                                                   group, p.U, p.G, p.S_max, hdr, counters, partials,
                                                   wait_limit_ns());
  note_launch();
  return check_launch();
}

namespace up {
size_t w4a16_smem_bytes() { return w4::kSmemBytes; }  // for the kernel interface
}  // namespace up

UP_DEFINE_REVISION(w4a16)
