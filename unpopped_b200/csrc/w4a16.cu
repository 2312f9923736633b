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
//    the W stage (conflict free under the swizzle). (Sixteen warps, one k-quarter each, measured 4 % slower and left
//    fewer registers per thread.) It turns the nibbles into exact bf16 (a shift, one lop3 and one bf16x2 subtract per
//    pair, pairing k with k + 4) and stores them into tensor memory (tcgen05.st) as the MMA's A operand, whose k
//    order inside each group of 8 is therefore 0,4,1,5,2,6,3,7. The four warps of k-half h (w / 4 = h) release
//    half h of the unit's A together (one barrier per half).
//  * warps 8..11 (MMA issuers): one thread issues a tcgen05.mma of this shape about every 49 cycles alone (measured;
//    four issuing threads reach one per 12 cycles), so the issuers work in two pairs: pair p takes units p, p + 2,
//    ..., and issuer h of the pair issues the 4 UK k-steps of half h into its own accumulator (a k-block's when
//    UK = 2) and commits the unit's barriers (counts of two). No issuer waits for another: chaining issuers inside a
//    unit (an mbarrier hand-off per k-quarter) put four hand-off latencies on every unit. Every ring an issuer waits
//    on (A and D slots in tensor memory, activation stages) is at least as deep as the number of pairs, so no parity
//    wait can meet a barrier two phases behind.
//  * warp 16 (activation loader): one thread brings each unit's [16 x 128 UK] activation tile into a ring of
//    shared-memory stages with 2 UK TMA boxes, 128-byte swizzled as the MMA reads it; rows past M read as 0.
//  * warp 19 (activation permuter): rewrites each landed 16-byte chunk (8 k) in place to the k order 0,4,1,5,2,6,
//    3,7 of the A operand (the swizzle moves whole chunks, so it is unaffected), then releases the stage to the MMA.
//  * warp 17 (scale loader): one thread brings each unit's scales, f16 groups [g0, g0 + 16) of its 128 rows with
//    g0 = the unit's first group rounded down to a multiple of 8, into a ring of shared-memory slots with one TMA
//    box. (A scale row stride that is not a multiple of 16 bytes cannot be a TMA tensor; then the warp's lanes load
//    and store the same slot layout.) Loading them in the epilogue put a global-load latency on every unit. Beside
//    each unit's scales it writes the unit's header: the tile, where tile segments start and end, and the slot
//    columns of the unit's scales.
//  * warps 12..15 (epilogue): read the unit's two half accumulators (tcgen05.ld), scale each k-block by
//    scale[n][k-block] in f32 (for UK = 1, the two halves of the one k-block are summed first) and accumulate in
//    registers, unit by unit as the headers say. A tile finished inside one CTA is written as bf16;
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
constexpr int kIssuers = 4;                      // warps 8..11: two pairs
constexpr int kPairs = kIssuers / 2;             // units in issue at once
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
  // accumulator columns per unit: one 16-column block per half of the unit (64 UK k: a k-block when UK = 2)
  static constexpr int kDCols = 2 * kMmaN;
  static constexpr int kRing = UK == 1 ? 5 : 3;        // A slots: units in flight between dequant and MMA
  static constexpr int kACol0 = 0;
  static constexpr int kDCol0 = kRing * kACols;
  // D slots: the accumulators take the columns the A slots leave, so the epilogue runs one or more units behind the
  // MMAs without holding back an A slot (4 for two k-blocks a unit, 8 for one)
  static constexpr int kDRing = (kTmemCols - kDCol0) / kDCols;
  static constexpr int kXUnit = kXBytes * UK;          // activation bytes per unit
  static constexpr int kXStages = 12 / UK;             // 48 KiB of activation stages either way
  static constexpr int kWRow = 64 * UK;                // bytes of one W row in a unit
  static constexpr int kWUnit = kTileN * kWRow;        // W bytes per unit (one TMA box of 128 rows)
  static constexpr int kWStages = 16 / UK;             // 128 KiB of W in flight either way
  // mbarriers: x_full, x_empty, x_raw [kXStages]; a_full [kRing][2]; mma_done [kRing]; d_done, d_empty [kDRing];
  // drain [kIssuers]; sc_full, sc_empty [kScRing]; w_full, w_empty [kWStages]; seg_in, seg_out; then the TMEM address
  // word, the abort word and the fix-up verdict
  static constexpr int kNumBars =
      3 * kXStages + 3 * kRing + 2 * kDRing + kIssuers + 2 * kScRing + 2 * kWStages + 2;
  static_assert(kDRing >= kRing && kDCol0 + kDRing * kDCols <= kTmemCols, "tensor memory");
  // Issuer pair p takes units p, p + kPairs, ...; for unit i an issuer waits on ring slots for the phase of unit i (or
  // of i - depth), which is only sound while the slot's phase before that has completed. The issuer's previous unit,
  // i - kPairs, already saw every unit up to it through, so a ring at least kPairs deep is enough.
  static_assert(kRing >= kPairs && kDRing >= kPairs && kXStages >= kPairs, "ring shallower than the issuer pairs");
};
constexpr int kBarBytes = 2048;
constexpr size_t kWBytes = (size_t)16 * kTileN * 64;  // the W ring: Cfg<UK>::kWStages * kWUnit for either UK
static_assert(Cfg<1>::kNumBars * 8 + 12 <= kBarBytes && Cfg<2>::kNumBars * 8 + 12 <= kBarBytes, "barrier region");
constexpr size_t kScSlot = (size_t)kTileN * kScCols * 2;  // one TMA box of 128 rows x 16 f16
constexpr size_t kScBytes = kScRing * kScSlot;
// Each scale slot carries its unit's header, written by the scale warp with the scales: {tile, segment flags,
// the slot columns of the unit's UK scale groups (16 bits each), 0}. The epilogue then keeps no unit cursor.
constexpr size_t kHdrBytes = kScRing * sizeof(int4);
constexpr uint32_t kSegStart = 1u, kSegEnd = 2u, kSegWhole = 4u;  // header flags: a tile segment starts / ends here;
                                                                   // the segment is the whole tile
constexpr size_t kSmemBytes =
    1024 /*alignment slack*/ + (size_t)12 * kXBytes + kWBytes + kScBytes + kHdrBytes + kBarBytes;
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
  static_assert(UK == 1 || UK == 2, "one or two k-blocks a unit");
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
  // scale-group index of k-block kb + h of the unit (h < UK <= 2 and sub < kpg, so (sub + h) / kpg is 0 or 1)
  __device__ __forceinline__ int gi_at(int h, int kpg) const { return gi + (sub + h == kpg ? 1 : 0); }
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
  uint8_t* wst = xs + (size_t)kXStages * C::kXUnit;  // [kWStages] W boxes (1024-byte aligned: 48 KiB after xs)
  __half* scs = reinterpret_cast<__half*>(wst + kWBytes);  // [kScRing][128][kScCols] f16 scales
  int4* sc_hdr = reinterpret_cast<int4*>(wst + kWBytes + kScBytes);  // [kScRing] unit headers
  uint64_t* x_full = reinterpret_cast<uint64_t*>(wst + kWBytes + kScBytes + kHdrBytes);  // [kXStages]: TMA landed
  uint64_t* x_empty = x_full + kXStages;        // [kXStages]: the stage's MMAs completed (the issuer's commit)
  uint64_t* a_full = x_empty + kXStages;        // [kRing][2]: half h of the unit's A is in TMEM (4 dequant warps)
  uint64_t* mma_done = a_full + 2 * kRing;      // [kRing]: all of the unit's MMAs completed (its A slot is free)
  uint64_t* d_done = mma_done + kRing;          // [kDRing]: the same, by D slot (the epilogue may read it)
  uint64_t* d_empty = d_done + C::kDRing;       // [kDRing]: the epilogue has read the unit's accumulators
  uint64_t* drain = d_empty + C::kDRing;        // [kIssuers]: an unwinding issuer's MMAs completed
  uint64_t* sc_full = drain + kIssuers;         // [kScRing]: the scale warp has written the unit's scales
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
      tc::mbar_init(&x_empty[s], 2);
    }
    for (int a = 0; a < kRing; ++a) {
      for (int h = 0; h < 2; ++h) tc::mbar_init(&a_full[2 * a + h], kDqWarps / 2);
      tc::mbar_init(&mma_done[a], 2);
    }
    for (int g = 0; g < kIssuers; ++g) tc::mbar_init(&drain[g], 1);
    for (int d = 0; d < C::kDRing; ++d) {
      tc::mbar_init(&d_done[d], 2);
      tc::mbar_init(&d_empty[d], kEpiWarps);
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
    // this thread's 16-byte chunks of its row in a W stage: chunk UK kq + h, 128-byte swizzled when UK = 2. The
    // loop keeps its ring positions as 32-bit counters advanced by increments: the integer pipe is the one the
    // nibble conversion fills, so the loop's own arithmetic is kept off it.
    uint32_t coff[2][UK];  // byte offsets of the chunks inside a W stage
#pragma unroll
    for (int qq = 0; qq < 2; ++qq)
#pragma unroll
      for (int h = 0; h < UK; ++h) {
        const int c = UK * (2 * kh + qq) + h;
        coff[qq][h] = (uint32_t)(r * C::kWRow + ((UK == 2 ? (c ^ (r & 7)) : c) << 4));
      }
    const uint32_t a_base = tmem + lane_addr + C::kACol0 + 16 * (UK * 2 * kh);  // this warp's columns of A slot 0
    int sw = 0, a = 0;
    uint32_t wph = 0, aph = 0;
    const int nu = (int)n_units;
    for (int i = 0; i < nu; ++i) {
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&w_full[sw], wph, wait_ns, abort_flag))) {
        give_up();
        break;
      }
      uint4 cur[2][UK];
      const uint8_t* stage = wst + (size_t)sw * C::kWUnit;
#pragma unroll
      for (int qq = 0; qq < 2; ++qq)
#pragma unroll
        for (int h = 0; h < UK; ++h) cur[qq][h] = *reinterpret_cast<const uint4*>(stage + coff[qq][h]);
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&w_empty[sw]);
      if (++sw == C::kWStages) {
        sw = 0;
        wph ^= 1u;
      }
      // the A stage is free once the unit kRing earlier has been multiplied
      const bool good = tc::mbar_wait(&mma_done[a], aph ^ 1u, wait_ns, abort_flag);
      if (!__all_sync(0xffffffffu, good)) {  // warp-uniform: the tcgen05 ops below are .sync.aligned
        give_up();
        break;
      }
#pragma unroll
      for (int qq = 0; qq < 2; ++qq)
#pragma unroll
        for (int h = 0; h < UK; ++h) {
          uint32_t regs[16];
          const uint32_t wd[4] = {cur[qq][h].x, cur[qq][h].y, cur[qq][h].z, cur[qq][h].w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) nib8_to_bf16x2_k4(wd[wi], regs + 4 * wi);
          tc::st_32x32b_x16(a_base + a * C::kACols + 16 * (UK * qq + h), regs);
        }
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&a_full[2 * a + kh]);  // this warp's k-quarters are half kh of the unit
      if (++a == kRing) {
        a = 0;
        aph ^= 1u;
      }
    }
  } else if (warp < kEpi0) {
    // ------- MMA issuers: pair p takes units p, p + 2, ...; issuer h of the pair the 4 UK k-steps of half h -------
    const int g = warp - kIss0, p = g >> 1, hh = g & 1;
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(kTileN, kMmaN);
      bool issued = false;
      // ring positions of unit i, advanced by kPairs units a step
      int a = p, s = p, dsl = p;
      uint32_t rph = 0, xph = 0, dph = 0;
      auto step = [](int& slot, uint32_t& ph, int depth) {
        if ((slot += kPairs) >= depth) {
          slot -= depth;
          ph ^= 1u;
        }
      };
      const int nu = (int)n_units;
      for (int i = p; i < nu; i += kPairs, step(a, rph, kRing), step(s, xph, kXStages), step(dsl, dph, C::kDRing)) {
        // the half's A and the unit's activations are in place and the epilogue has read the D slot's previous unit
        const bool ready = tc::mbar_wait(&a_full[2 * a + hh], rph, wait_ns, abort_flag) &&
                           tc::mbar_wait(&x_full[s], xph, wait_ns, abort_flag) &&
                           tc::mbar_wait(&d_empty[dsl], dph ^ 1u, wait_ns, abort_flag);
        if (!ready) {
          give_up();
          break;
        }
        tc::fence_after_sync();
        const uint32_t xaddr = tc::smem_u32(xs + (size_t)s * C::kXUnit);
#pragma unroll
        for (int jj = 0; jj < 4 * UK; ++jj) {
          const int j = 4 * UK * hh + jj;  // k-step j: 16 k = 32 bytes of a 128-byte swizzle atom row
          const uint64_t bdesc = tc::sdesc_kmajor_sw128(xaddr + (uint32_t)((j >> 2) * 2048 + (j & 3) * 32));
          tc::mma_ts_bf16(tmem + C::kDCol0 + dsl * C::kDCols + hh * kMmaN, tmem + C::kACol0 + a * C::kACols + j * 8,
                          bdesc, idesc, jj > 0 ? 1u : 0u);
        }
        // the commits arrive once this thread's MMAs so far (so its half of the unit) have completed
        tc::commit(&mma_done[a]);
        tc::commit(&d_done[dsl]);
        tc::commit(&x_empty[s]);
        issued = true;
      }
      // Unwinding after an abort: this issuer's MMAs must finish before TMEM is released.
      if (*abort_flag && issued) {
        tc::commit(&drain[g]);
        tc::mbar_wait(&drain[g], 0u, wait_ns, nullptr);
      }
    }
  } else if (warp >= kEpi0 && warp < kXWarp) {
    // ---------------- epilogue: row 32 (warp % 4) + lane, all 16 activation rows ----------------
    // Per unit: the scale slot (its header says the tile, where segments start and end and which scale columns to
    // take), then the accumulators; ring positions advance by increments (no 64-bit division in the loop).
    const int lq = warp & 3;
    const int r = lq * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(lq * 32) << 16;
    const int64_t GU = G / UK;  // units per tile
    float acc[kMmaN];
#pragma unroll
    for (int j = 0; j < kMmaN; ++j) acc[j] = 0.f;
    uint32_t nfix = 0;
    int d = 0, q = 0;
    uint32_t dph = 0, qph = 0;
    const int nu = (int)n_units;
    for (int e = 0; e < nu; ++e) {
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&sc_full[q], qph, wait_ns, abort_flag))) {
        give_up();
        break;
      }
      const int4 hd = sc_hdr[q];
      float sc[UK];
#pragma unroll
      for (int h = 0; h < UK; ++h)
        sc[h] = __half2float(scs[((size_t)q * kTileN + r) * kScCols + ((hd.z >> (16 * h)) & 0xffff)]);
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&sc_empty[q]);
      if (++q == kScRing) {
        q = 0;
        qph ^= 1u;
      }
      const bool good = tc::mbar_wait(&d_done[d], dph, wait_ns, abort_flag);
      if (!__all_sync(0xffffffffu, good)) {
        give_up();
        break;
      }
      tc::fence_after_sync();
      if (hd.y & kSegStart) {  // a segment starts: the range's start, the wrap, a tile
#pragma unroll
        for (int j = 0; j < kMmaN; ++j) acc[j] = 0.f;
      }
      {
        uint32_t dv[2][kMmaN];  // the unit's two half accumulators
        tc::ld_32x32b_x16(tmem + lane_addr + C::kDCol0 + d * C::kDCols, dv[0]);
        tc::ld_32x32b_x16(tmem + lane_addr + C::kDCol0 + d * C::kDCols + kMmaN, dv[1]);
        tc::wait_ld();
        if (UK == 2) {  // the halves are the k-blocks: each its own scale, in k order
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int j = 0; j < kMmaN; ++j) acc[j] = fmaf(sc[h], __uint_as_float(dv[h][j]), acc[j]);
        } else {  // both halves of the one k-block, summed, then scaled
#pragma unroll
          for (int j = 0; j < kMmaN; ++j)
            acc[j] = fmaf(sc[0], __uint_as_float(dv[0][j]) + __uint_as_float(dv[1][j]), acc[j]);
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&d_empty[d]);
      if (++d == C::kDRing) {
        d = 0;
        dph ^= 1u;
      }
      if (hd.y & kSegEnd)  // the segment ends here: write the tile, or publish this CTA's part of it
        if (!finish_segment(acc, hd.x, (hd.y & kSegWhole) != 0, r, lane, M, N, U, GU, P, S_max, out, counters,
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
    int seg_kb0 = 0;
    // the unit's header: a segment starts at the range's start, at the wrap and at a tile's first unit, and ends at
    // the range's end and at a tile's last unit
    auto header = [&](int64_t i) {
      const int64_t u = rs.unit();
      const bool start = i == 0 || i == rs.n_first || cs.kb == 0;
      if (start) seg_kb0 = cs.kb;
      const bool end = u + 1 == hi || cs.kb + UK == Gi;
      const uint32_t flags = (start ? kSegStart : 0u) | (end ? kSegEnd : 0u) |
                             (end && seg_kb0 == 0 && cs.kb + UK == Gi ? kSegWhole : 0u);
      const int g0 = cs.gi & ~7;
      int cols = cs.gi_at(0, kpg) - g0;
      if (UK == 2) cols |= (cs.gi_at(1, kpg) - g0) << 16;
      return make_int4(cs.t, (int)flags, cols, 0);
    };
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
          sc_hdr[q] = header(i);  // published by the arrive (release) below
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
        const int4 hd = header(i);
        if (lane == 0) sc_hdr[q] = hd;
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
  } else if (warp == kXWarp) {
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
  if (p.U / p.P + 1 > 0x7fffffff) return UP_ERR_UNSUPPORTED;  // a CTA counts its units in 32 bits
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
