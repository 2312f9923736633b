// scan.cu — single-pass int32 scans (inclusive / exclusive; SUM wrapping, MAX, MIN; forward / reverse)
// by decoupled look-back, for sm_100a.
//
// Semantics: `Access::Scan` (crates/unpopped/src/ir.rs:2153-2195) as the oracle evaluates it
// (crates/unpopped/src/oracle/plan_window.rs:10-238): per row of k elements, an inclusive scan writes
// after the combine, an exclusive scan before it (so element 0 gets the monoid identity: 0, INT32_MIN,
// INT32_MAX); Sum wraps at 32 bits; a reverse scan walks from the row's end. Integer combines are exact
// and associative, so the tile decomposition below produces the serial walk's bytes.
//
// Two forms share one flag protocol:
//  * the persistent form (scan_i32_persist_kernel, below), for rows that are 16-byte aligned and whole
//    16-byte chunks long: one CTA per SM streams 8192-element tiles through a ring of shared-memory stages
//    by bulk copies, and resolves each tile's prefix from the other tiles' aggregates off the critical path;
//  * the general form (scan_i32_kernel), for any alignment: one CTA per 16384-element tile, element loads,
//    decoupled look-back with aggregate and inclusive flags.
//
// Look-back flags: one 64-bit word per tile = epoch(30) | status(2) | value(32), written and read with
// relaxed gpu-scope atomics (the value travels inside the flag word). Status: 1 = aggregate of this tile,
// 2 = inclusive prefix through this tile, 3 = aborted. The epoch is the low 30 bits of a per-launch 64-bit
// count kept on the host, so flags of earlier launches are never mistaken for this one's and the workspace
// needs zero-filling only once. When the count passes a multiple of 2^30 the tags repeat: the first launch
// on each workspace after that clears its flags (a stream-ordered memset) before it runs. Every wait is
// bounded by a globaltimer deadline; a wait that runs out sets the workspace error word and publishes
// "aborted", which the tiles that wait on it propagate at once.
#include "common.cuh"
#include "multi.cuh"
#include "tc.cuh"

#include <atomic>
#include <mutex>
#include <vector>

namespace up {

constexpr int kScanThreads = 256;
constexpr int kLaneChunks = 16;                                  // 16-byte chunks per lane
constexpr int kScanTile = kScanThreads * kLaneChunks * 4;        // 16384 elements
constexpr int kWarpChunks = 32 * kLaneChunks;                    // 512 chunks = 2048 elements per warp
constexpr int kTileBytes = kScanTile * 4;                        // 64 KiB
constexpr size_t kScanSmem = kTileBytes;

struct ScanHeader {
  uint32_t ticket;  // the general form's next tile; the CTA that takes the last tile sets it back to 0
  uint32_t reserved1, reserved2;
  uint32_t error;   // byte 12: set when a bounded wait ran out
  uint32_t pad[12];
};
static_assert(sizeof(ScanHeader) == 64, "header is one 64-byte line");

enum : uint32_t { kFlagInvalid = 0, kFlagAgg = 1, kFlagIncl = 2, kFlagErr = 3 };

__device__ __forceinline__ uint64_t make_flag(uint32_t epoch, uint32_t status, int32_t v) {
  return ((uint64_t)(epoch & 0x3fffffffu) << 34) | ((uint64_t)status << 32) | (uint64_t)(uint32_t)v;
}
__device__ __forceinline__ uint32_t flag_status(uint64_t f, uint32_t epoch) {
  return ((uint32_t)(f >> 34) == (epoch & 0x3fffffffu)) ? (uint32_t)((f >> 32) & 3u) : kFlagInvalid;
}

template <int OP>
__device__ __forceinline__ int32_t ident() {
  return OP == UP_OP_SUM ? 0 : (OP == UP_OP_MAX ? INT32_MIN : INT32_MAX);
}
template <int OP>
__device__ __forceinline__ int32_t comb(int32_t a, int32_t b) {
  if (OP == UP_OP_SUM) return (int32_t)((uint32_t)a + (uint32_t)b);
  if (OP == UP_OP_MAX) return a > b ? a : b;
  return a < b ? a : b;
}

template <int OP>
__device__ __forceinline__ int32_t warp_reduce(int32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = comb<OP>(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Inclusive scan across the 32 lanes (Kogge-Stone).
template <int OP>
__device__ __forceinline__ int32_t warp_incl_scan(int32_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t w = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v = comb<OP>(w, v);
  }
  return v;
}

// The tile in shared memory, in scan order, read and written by chunk (elements 4g .. 4g+3); `cnt` valid
// elements, the rest read as the identity.
template <int OP>
struct TileView {
  int32_t* buf;
  int cnt;
  __device__ __forceinline__ void load(int g, int32_t (&v)[4]) const {
    const int e0 = 4 * g;
    if (e0 + 4 <= cnt) {
      const int4 c = reinterpret_cast<const int4*>(buf)[g];
      v[0] = c.x; v[1] = c.y; v[2] = c.z; v[3] = c.w;
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) v[c] = (e0 + c < cnt) ? buf[e0 + c] : ident<OP>();
    }
  }
  __device__ __forceinline__ void store(int g, const int32_t (&o)[4]) const {
    const int e0 = 4 * g;
    if (e0 + 4 <= cnt) {
      reinterpret_cast<int4*>(buf)[g] = make_int4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (e0 + c < cnt) buf[e0 + c] = o[c];
    }
  }
};

// General form: CTA i scans tile i (16384 elements of one row; the row's last tile may be short). The tile
// is read with element loads into shared memory in scan order; in shared memory, warp w owns 2048 elements
// and lane l handles the 16-byte chunks i*32 + l (i = 0..15), which keeps every access conflict-free.
// Pass 1 folds the tile; the aggregate goes out as a look-back flag; warp 0 walks back 32 predecessors
// per step until an inclusive prefix; pass 2 rescans with the prefix and writes the result. A CTA takes its
// tile from a ticket counter in the workspace header, not from blockIdx.x: tickets go out in the order CTAs
// start, so a tile only ever waits on tiles whose CTAs are already running, whatever order the hardware
// dispatches CTAs in and however many SMs other work holds.
template <int OP>
__global__ void __launch_bounds__(kScanThreads) scan_i32_kernel(const int32_t* __restrict__ x,
                                                                int32_t* __restrict__ y, int64_t k,
                                                                int64_t tiles_per_row, int exclusive, int reverse,
                                                                const int32_t* carry_in, ScanHeader* hdr,
                                                                uint64_t* flags, uint32_t epoch, uint64_t wait_ns,
                                                                int withhold) {
  extern __shared__ __align__(128) uint8_t smem[];
  int32_t* buf = reinterpret_cast<int32_t*>(smem);
  __shared__ int32_t s_warp_tot[kScanThreads / 32];
  __shared__ int32_t s_prefix;
  __shared__ int s_abort;
  __shared__ uint32_t s_ticket;

  if (threadIdx.x == 0) {
    const uint32_t tk = atomicAdd(&hdr->ticket, 1u);
    if (tk == gridDim.x - 1) atomicExch(&hdr->ticket, 0u);  // every CTA has its tile: ready for the next launch
    s_ticket = tk;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = s_ticket;
  const int64_t row = t / tiles_per_row;
  const int64_t q = t - row * tiles_per_row;
  const int64_t lo = q * kScanTile;
  const int cnt = (int)((k - lo) < kScanTile ? (k - lo) : kScanTile);
  const int32_t* xr = x + row * k;
  int32_t* yr = y + row * k;
  const int32_t id = ident<OP>();

  // ---- bring the tile into shared memory, in scan order (a reversed row is read back to front) ----
  if (threadIdx.x == 0) s_abort = 0;
  for (int e = threadIdx.x; e < cnt; e += kScanThreads) buf[e] = __ldg(xr + (reverse ? (k - 1 - (lo + e)) : (lo + e)));
  __syncthreads();
  const TileView<OP> tile{buf, cnt};

  // ---- pass 1: fold the tile ----
  int32_t acc = id;
#pragma unroll 4
  for (int i = 0; i < kLaneChunks; ++i) {
    int32_t v[4];
    tile.load(warp * kWarpChunks + i * 32 + lane, v);
    acc = comb<OP>(acc, comb<OP>(comb<OP>(v[0], v[1]), comb<OP>(v[2], v[3])));
  }
  acc = warp_reduce<OP>(acc);
  if (lane == 0) s_warp_tot[warp] = acc;
  __syncthreads();
  int32_t wpre = id, agg = id;
#pragma unroll
  for (int w = 0; w < kScanThreads / 32; ++w) {
    if (w < warp) wpre = comb<OP>(wpre, s_warp_tot[w]);
    agg = comb<OP>(agg, s_warp_tot[w]);
  }

  // ---- look-back (warp 0) ----
  if (warp == 0) {
    const int32_t cin = carry_in ? *carry_in : id;
    int32_t excl = id;
    bool abort = s_abort != 0;
    if (q == 0) {
      excl = cin;
      if (lane == 0 && !(withhold && t == 0))
        st_relaxed_u64(flags + t, make_flag(epoch, abort ? kFlagErr : kFlagIncl, comb<OP>(cin, agg)));
    } else if (!abort) {
      if (lane == 0) st_relaxed_u64(flags + t, make_flag(epoch, kFlagAgg, agg));
      const int64_t row_first = row * tiles_per_row;
      int64_t pred = t - 1;
      while (true) {
        const int64_t j = pred - lane;
        const bool mine = j >= row_first;
        uint64_t f = 0;
        uint32_t st = kFlagIncl;  // lanes before the row's first tile are never read
        const uint64_t t0 = globaltimer_ns();
        while (true) {
          if (mine) {
            f = ld_relaxed_u64(flags + j);
            st = flag_status(f, epoch);
          }
          if (__all_sync(0xffffffffu, st != kFlagInvalid)) break;
          const bool late = __shfl_sync(0xffffffffu, (globaltimer_ns() - t0) > wait_ns, 0);
          if (late) {
            abort = true;
            break;
          }
          __nanosleep(32);
        }
        if (abort) break;
        if (__any_sync(0xffffffffu, mine && st == kFlagErr)) {
          abort = true;
          break;
        }
        const unsigned incl = __ballot_sync(0xffffffffu, mine && st == kFlagIncl);
        const int stop = incl ? (__ffs(incl) - 1) : 32;
        const int32_t val = (mine && lane <= stop) ? (int32_t)(uint32_t)f : id;
        excl = comb<OP>(excl, warp_reduce<OP>(val));
        if (incl) break;
        pred -= 32;
      }
      if (lane == 0) {
        if (abort) atomicOr(&hdr->error, 1u);
        st_relaxed_u64(flags + t, abort ? make_flag(epoch, kFlagErr, 0) : make_flag(epoch, kFlagIncl, comb<OP>(excl, agg)));
      }
    } else if (lane == 0) {
      st_relaxed_u64(flags + t, make_flag(epoch, kFlagErr, 0));
    }
    if (lane == 0) {
      s_prefix = excl;
      s_abort = abort ? 1 : 0;
    }
  }
  __syncthreads();
  if (s_abort) return;  // uniform: nothing written, the error word is set

  // ---- pass 2: rescan with the tile's prefix, in place ----
  const int32_t base = comb<OP>(s_prefix, wpre);
  int32_t carry = id;
#pragma unroll 2
  for (int i = 0; i < kLaneChunks; ++i) {
    const int g = warp * kWarpChunks + i * 32 + lane;
    int32_t v[4];
    tile.load(g, v);
    v[1] = comb<OP>(v[0], v[1]);
    v[2] = comb<OP>(v[1], v[2]);
    v[3] = comb<OP>(v[2], v[3]);
    const int32_t inc = warp_incl_scan<OP>(v[3], lane);
    int32_t exc = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 0) exc = id;
    const int32_t pre = comb<OP>(comb<OP>(base, carry), exc);
    int32_t o[4];
    if (exclusive) {
      o[0] = pre;
      o[1] = comb<OP>(pre, v[0]);
      o[2] = comb<OP>(pre, v[1]);
      o[3] = comb<OP>(pre, v[2]);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) o[c] = comb<OP>(pre, v[c]);
    }
    tile.store(g, o);
    carry = comb<OP>(carry, __shfl_sync(0xffffffffu, inc, 31));
  }

  // ---- write the tile back ----
  __syncthreads();
  for (int e = threadIdx.x; e < cnt; e += kScanThreads) yr[reverse ? (k - 1 - (lo + e)) : (lo + e)] = buf[e];
}

// ===================================================================================================
// Persistent form, for rows that are 16-byte aligned and whole 16-byte chunks long (the common case).
//
// One CTA per SM; CTA b scans the 8192-element tiles b, b + P, b + 2P, ... (P = grid size) in that order.
//  * Copy warp: one thread keeps a ring of kQStages tiles loading into shared memory by bulk copies and sends
//    each scanned tile back out with bulk stores, so HBM reads stay in flight while tiles are scanned.
//  * Compute warps (512 threads): thread r owns the 4 consecutive 16-byte chunks 4r .. 4r+3 of a tile. It
//    folds a tile as soon as it lands (pass 1: chunk sums, their prefixes in scan order, a warp scan, the
//    tile aggregate, which is published at once as the tile's look-back flag) and rescans it (pass 2) once its
//    prefix is known. Folding runs kQFold tiles ahead of rescanning. A thread visits its chunks in a rotated
//    order, (i + (lane / 2)) mod 4, which spreads each 8-lane phase of a warp over all eight 16-byte bank
//    groups, so every shared-memory access is conflict-free; chunk prefixes are rotated into scan order and
//    back by a two-step barrel shift.
//  * Look-back warp: computes the exclusive prefix of each of the CTA's tiles from the published aggregates
//    alone. For tile t whose previous tile t - P (this CTA's) is in the same row,
//        prefix(t) = prefix(t - P) + aggregate(t - P) + ... + aggregate(t - 1),
//    P flags read in one batch (up to 5 per lane); otherwise it sums the row from its first tile. Every flag
//    it reads is an aggregate, which depends only on its own tile's data: there is no chain of prefixes across
//    CTAs, and this warp runs ahead of the rescans as far as the aggregates allow, so the round trips to L2
//    overlap the scanning instead of stalling it.
// Forward progress: every CTA is resident (one per SM, grid <= SMs; the host checks that one CTA fits on an SM
// before it launches this form); a tile's aggregate needs only its data, and a stage is refilled only after its
// tile's rescan, whose prefix needs aggregates of smaller tiles only. Work that holds SMs while this kernel runs
// (a concurrent kernel, a context limited to part of the GPU) can keep a CTA off the device until the others
// finish; they cannot finish without it, so their bounded waits run out and the launch reports
// UP_ERR_DEVICE_TIMEOUT with a partly written output, not a hang.
// Aborts: a wait that runs out (or an aborted tile in a window) makes the CTA publish "aborted" for its
// remaining tiles, stop loading, let the loads in flight land, and exit; the error word is set.
constexpr int kQTile = 8192;                        // elements per tile
constexpr int kQTileBytes = kQTile * 4;             // 32 KiB
constexpr int kQStages = 6;
constexpr int kQRowChunks = 4;                      // 16-byte chunks per compute thread
constexpr int kQCompute = kQTile / (4 * kQRowChunks);  // 512 compute threads
constexpr int kQCWarps = kQCompute / 32;            // 16
constexpr int kQCopyWarp = kQCWarps, kQLookWarp = kQCWarps + 1;
constexpr int kQThreads = kQCompute + 64;           // + copy warp + look-back warp
constexpr int kQPubWarp = kQLookWarp + 1;           // block-cyclic form: CTA 0's stripe publisher
constexpr int kQThreadsMulti = kQThreads + 32;
constexpr int kQFold = 3;                           // tiles folded ahead of the rescan
constexpr int kQRing = 5;                           // prefix and warp-total ring (>= kQFold + 2)
constexpr int kQMaxWin = 5;                         // look-back flags per lane: grids of up to 160 CTAs
constexpr int kQMaxGrid = 32 * kQMaxWin;
constexpr size_t kQSmem = (size_t)kQStages * kQTileBytes + 256;
static_assert(kQRing >= kQFold + 2, "warp-total ring");
static_assert(kQStages >= kQFold + 2, "stages");
// The block-cyclic form folds one tile further ahead: its rescans also wait for other GPUs' stripe aggregates, and
// the fold look-ahead is the slack that hides their arrival. A seventh stage keeps two tiles loading ahead.
constexpr int kQStagesMulti = 7, kQFoldMulti = 4, kQRingMulti = 6;
constexpr size_t kQSmemMulti = (size_t)kQStagesMulti * kQTileBytes + 256;
static_assert(kQRingMulti >= kQFoldMulti + 2 && kQStagesMulti >= kQFoldMulti + 2, "block-cyclic pipeline");
static_assert(kQSmemMulti <= 227 * 1024 - 1024, "block-cyclic stages fit the opt-in shared memory");

// Barrier `id` over `n` threads that also returns whether any of them passed `v`.
__device__ __forceinline__ bool named_bar_or(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// a[j] <- a[(j - k) mod 4] (rotate toward higher index by k), k in [0, 4), as two conditional steps.
__device__ __forceinline__ void rot_up4(int32_t (&a)[4], int k) {
#pragma unroll
  for (int step = 1; step < 4; step <<= 1) {
    const bool on = (k & step) != 0;
    int32_t t[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] = on ? a[(j - step) & 3] : a[j];
#pragma unroll
    for (int j = 0; j < 4; ++j) a[j] = t[j];
  }
}
// a[j] <- a[(j + k) mod 4], the inverse of rot_up4.
__device__ __forceinline__ void rot_down4(int32_t (&a)[4], int k) {
#pragma unroll
  for (int step = 1; step < 4; step <<= 1) {
    const bool on = (k & step) != 0;
    int32_t t[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] = on ? a[(j + step) & 3] : a[j];
#pragma unroll
    for (int j = 0; j < 4; ++j) a[j] = t[j];
  }
}

// This CTA's j-th tile t = b + j*P as (row, tile within the row), advanced by additions.
struct QCursor {
  int64_t t, row, q;
  __device__ __forceinline__ void init(int64_t t0, int64_t tpr) {
    t = t0;
    row = t0 / tpr;
    q = t0 - row * tpr;
  }
  __device__ __forceinline__ void next(int64_t P, int64_t tpr) {
    t += P;
    q += P;
    if (q >= tpr) {  // crossed into a later row (only when rows are shorter than P tiles, or at a row's end)
      const int64_t dr = q / tpr;
      row += dr;
      q -= dr * tpr;
    }
  }
};

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// What pass 1 leaves for pass 2 of one tile, per thread.
struct QFold {
  int32_t cp[kQRowChunks];  // slot i: exclusive prefix, within this thread's row, of chunk (i + R) mod 4
  int32_t texcl;            // exclusive prefix of this thread's row within its warp
};

template <int OP, bool REV, bool MULTI = false>
__global__ void __launch_bounds__(MULTI ? kQThreadsMulti : kQThreads, 1)
    scan_i32_persist_kernel(const int32_t* __restrict__ x, int32_t* __restrict__ y, int64_t k, int64_t tiles_per_row,
                            int64_t n_tiles, int exclusive, const int32_t* carry_in, ScanHeader* hdr, uint64_t* flags,
                            uint32_t epoch, uint64_t wait_ns, int withhold, MultiScan ms) {
  static_assert(!(MULTI && REV), "the block-cyclic form scans forward");
  constexpr int STAGES = MULTI ? kQStagesMulti : kQStages;  // shared-memory tile stages
  constexpr int FOLD = MULTI ? kQFoldMulti : kQFold;        // tiles folded ahead of the rescan
  constexpr int RING = MULTI ? kQRingMulti : kQRing;        // prefix and warp-total ring
  constexpr bool reverse = REV;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)STAGES * kQTileBytes);  // [stages] data landed
  uint64_t* done = full + STAGES;      // [stages] rescanned (one arrival per compute warp)
  uint64_t* pfull = done + STAGES;     // [ring] prefix delivered (look-back lane 0)
  uint64_t* pempty = pfull + RING;     // [ring] prefix consumed (one arrival per compute warp)
  __shared__ int32_t s_wt[RING][kQCWarps];
  __shared__ int32_t s_prefix[RING];
  __shared__ int s_abort_mem;
  volatile int* s_abort = &s_abort_mem;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t P = gridDim.x, b = blockIdx.x;
  const int64_t n_mine = (n_tiles - b + P - 1) / P;  // >= 1: the grid is at most n_tiles
  const int32_t id = ident<OP>();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&done[s], kQCWarps);
    }
    for (int s = 0; s < RING; ++s) {
      tc::mbar_init(&pfull[s], 1);
      tc::mbar_init(&pempty[s], kQCWarps);
    }
    *s_abort = 0;
    tc::mbar_fence_init();
  }
  __syncthreads();

  auto count_of = [&](const QCursor& c) {  // elements in the tile (the row's last tile may be short)
    const int64_t lo = c.q * kQTile;
    return (int)((k - lo) < kQTile ? (k - lo) : kQTile);
  };
  auto start_of = [&](const QCursor& c, int cnt) {  // first physical element of the tile
    const int64_t lo = c.q * kQTile;
    return c.row * k + (reverse ? (k - lo - cnt) : lo);
  };
  auto stage = [&](int64_t j) { return smem + (size_t)(j % STAGES) * kQTileBytes; };
  auto sphase = [&](int64_t j) { return (uint32_t)((j / STAGES) & 1); };
  auto rphase = [&](int64_t j) { return (uint32_t)((j / RING) & 1); };
  // Marks this CTA's tiles from `from` on as aborted, so that no other CTA waits for them.
  auto abort_from = [&](int64_t from) {
    if (!*s_abort) atomicOr(&hdr->error, 1u);
    *s_abort = 1;
    for (int64_t jj = from; jj < n_mine; ++jj) st_relaxed_u64(flags + b + jj * P, make_flag(epoch, kFlagErr, 0));
  };

  // Folds the m aggregates flags[t - m .. t - 1] into *sum once all have been published (bounded wait). False
  // when one of them is aborted, the CTA is aborting, or the wait ran out.
  auto window = [&](int64_t t, int m, int32_t* sum) -> bool {
    *sum = id;
    if (m <= 0) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
      uint64_t f[kQMaxWin];
#pragma unroll
      for (int i = 0; i < kQMaxWin; ++i) {  // all loads first: one round trip
        const int d = lane + 32 * i + 1;
        f[i] = d <= m ? ld_relaxed_u64(flags + (t - d)) : 0;
      }
      bool ready = true, err = false;
#pragma unroll
      for (int i = 0; i < kQMaxWin; ++i) {
        const int d = lane + 32 * i + 1;
        if (d <= m) {
          const uint32_t st = flag_status(f[i], epoch);
          ready = ready && st == kFlagAgg;
          err = err || st == kFlagErr;
        }
      }
      if (__any_sync(0xffffffffu, err) || __shfl_sync(0xffffffffu, *s_abort, 0)) return false;
      if (__all_sync(0xffffffffu, ready)) {
        int32_t v = id;
#pragma unroll
        for (int i = 0; i < kQMaxWin; ++i) {
          const int d = lane + 32 * i + 1;
          if (d <= m) v = comb<OP>(v, (int32_t)(uint32_t)f[i]);
        }
        *sum = warp_reduce<OP>(v);
        return true;
      }
      if (__shfl_sync(0xffffffffu, globaltimer_ns() - t0 > wait_ns, 0)) return false;
      __nanosleep(32);
    }
  };

  // MULTI, CTA 0: sends the aggregate of local stripe `ls` to every other rank (global stripe ls * G + r), or
  // "aborted" for local stripes ls onward, so that no rank waits for them.
  auto publish_stripe = [&](int64_t ls, int32_t agg, bool aborted) {
    if (!MULTI || b != 0) return;
    const int64_t n_stripes = (n_tiles + P - 1) / P;
    for (int64_t q = ls; q < (aborted ? n_stripes : ls + 1); ++q)
      if (lane < ms.G && lane != ms.r)
        st_relaxed_sys_u64(ms.peers[lane] + q * ms.G + ms.r,
                           make_flag(ms.tag, aborted ? kFlagErr : kFlagAgg, aborted ? 0 : agg));
  };

  if (MULTI && warp == kQPubWarp) {
    // ---------------- stripe publisher (block-cyclic form, CTA 0) ----------------
    // A stripe's aggregate depends only on its tiles' aggregates, which the compute warps of every CTA publish as
    // soon as they fold a tile (three tiles ahead of the rescans). Publishing it from here, not from the look-back
    // warp (whose loop also waits on the other ranks), keeps every cross-GPU dependency on data alone: no rank's
    // publication ever waits for another rank.
    if (b == 0) {
      const int64_t n_stripes = (n_tiles + P - 1) / P;
      for (int64_t q = 0; q < n_stripes; ++q) {
        const int64_t hi = (q + 1) * P < n_tiles ? (q + 1) * P : n_tiles;
        int32_t sum = id;
        if (!window(hi, (int)(hi - q * P), &sum)) {
          publish_stripe(q, 0, true);
          break;
        }
        publish_stripe(q, sum, false);
      }
    }
    return;
  }

  if (warp == kQCopyWarp) {
    // ---------------- copy warp ----------------
    if (lane == 0) {
      QCursor lc, sc;  // the next tile to load, the next tile to store
      lc.init(b, tiles_per_row);
      sc = lc;
      auto store = [&](int64_t j) {
        const int cnt = count_of(sc);
        const uint32_t bytes = (uint32_t)cnt * 4u;
        char* dst = reinterpret_cast<char*>(y + start_of(sc, cnt));
        for (uint32_t off = 0; off < bytes; off += 16384u)
          tc::bulk_store(dst + off, stage(j) + off, (bytes - off) < 16384u ? (bytes - off) : 16384u);
        tc::bulk_commit();
        sc.next(P, tiles_per_row);
      };
      int64_t issued = 0, stored = 0;
      bool ok = true;
      while (issued < n_mine && !*s_abort) {
        const int64_t j = issued;
        if (j >= STAGES) {  // the stage's previous tile must be rescanned and sent out first
          const int64_t jo = j - STAGES;
          if (!tc::mbar_wait(&done[jo % STAGES], sphase(jo), wait_ns, s_abort)) {
            ok = false;
            break;
          }
          store(jo);
          stored = jo + 1;
          tc::bulk_wait_read();  // the stage has been read out: it may be refilled
        }
        const int cnt = count_of(lc);
        const uint32_t bytes = (uint32_t)cnt * 4u;
        uint64_t* bar = &full[j % STAGES];
        tc::mbar_arrive_expect_tx(bar, bytes);
        const char* src = reinterpret_cast<const char*>(x + start_of(lc, cnt));
        for (uint32_t off = 0; off < bytes; off += 16384u)
          tc::bulk_load(stage(j) + off, src + off, (bytes - off) < 16384u ? (bytes - off) : 16384u, bar);
        lc.next(P, tiles_per_row);
        issued = j + 1;
      }
      for (int64_t jo = stored; ok && jo < issued && !*s_abort; ++jo) {
        if (!tc::mbar_wait(&done[jo % STAGES], sphase(jo), wait_ns, s_abort)) {
          ok = false;
          break;
        }
        store(jo);
      }
      if (!ok && !*s_abort) abort_from(stored);
      if (*s_abort) {
        // loads still in flight must land before this CTA's shared memory is released
        for (int64_t j = (issued > STAGES ? issued - STAGES : 0); j < issued; ++j)
          tc::mbar_wait(&full[j % STAGES], sphase(j), wait_ns, nullptr);
      }
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    return;
  }

  if (warp == kQLookWarp) {
    // ---------------- look-back warp ----------------
    const int32_t cin = carry_in ? *carry_in : id;
    int32_t pre_prev = id;
      // MULTI: `window` and the other ranks' stripe aggregates of global stripes [lo, hi) (at most kMaxRanks - 1)
    // in one round trip: both sets of loads are issued together and tested together (bounded wait). The ops are
    // commutative, so the stripes fold in any order.
    auto window_remote = [&](int64_t t, int m, int64_t lo, int64_t hi, int32_t* sum, int32_t* rsum) -> bool {
      *sum = id;
      *rsum = id;
      const int n = (int)(hi - lo);
      const uint64_t t0 = globaltimer_ns();
      while (true) {
        uint64_t f[kQMaxWin];
#pragma unroll
        for (int i = 0; i < kQMaxWin; ++i) {
          const int d = lane + 32 * i + 1;
          f[i] = d <= m ? ld_relaxed_u64(flags + (t - d)) : 0;
        }
        const uint64_t g = lane < n ? ld_relaxed_sys_u64(ms.sflags + lo + lane) : 0;
        bool ready = true, err = false;
#pragma unroll
        for (int i = 0; i < kQMaxWin; ++i) {
          const int d = lane + 32 * i + 1;
          if (d <= m) {
            const uint32_t st = flag_status(f[i], epoch);
            ready = ready && st == kFlagAgg;
            err = err || st == kFlagErr;
          }
        }
        if (lane < n) {
          const uint32_t st = flag_status(g, ms.tag);
          ready = ready && st == kFlagAgg;
          err = err || st == kFlagErr;
        }
        if (__any_sync(0xffffffffu, err) || __shfl_sync(0xffffffffu, *s_abort, 0)) return false;
        if (__all_sync(0xffffffffu, ready)) {
          int32_t v = id;
#pragma unroll
          for (int i = 0; i < kQMaxWin; ++i) {
            const int d = lane + 32 * i + 1;
            if (d <= m) v = comb<OP>(v, (int32_t)(uint32_t)f[i]);
          }
          *sum = warp_reduce<OP>(v);
          *rsum = warp_reduce<OP>(lane < n ? (int32_t)(uint32_t)g : id);
          return true;
        }
        if (__shfl_sync(0xffffffffu, globaltimer_ns() - t0 > wait_ns, 0)) return false;
        __nanosleep(32);
      }
    };
    QCursor c;
    c.init(b, tiles_per_row);
    for (int64_t j = 0; j < n_mine; ++j, c.next(P, tiles_per_row)) {
      int32_t pre = cin;
      bool good = true;
      const bool chain = j > 0 && c.q >= P;        // this CTA's previous tile is in the same row
      const int m = c.q == 0 ? 0 : (int)(chain ? P : c.q);  // aggregates to add: tiles t - m .. t - 1
      if (!MULTI) {
        if (m > 0) {
          int32_t sum = id;
          good = window(c.t, m, &sum);
          if (good) pre = comb<OP>(chain ? pre_prev : cin, sum);
        }
      } else {
        // the other ranks' stripes between this CTA's previous tile and this one: local stripe j - 1's successors
        // on ranks r + 1 .. G - 1 and local stripe j's predecessors on ranks 0 .. r - 1 (for j = 0, the latter)
        const int64_t lo = j == 0 ? 0 : (j - 1) * ms.G + ms.r + 1, hi = j * ms.G + ms.r;
        int32_t sum = id, rs = id;
        good = window_remote(c.t, m, lo, hi, &sum, &rs);
        if (good) pre = comb<OP>(m > 0 ? comb<OP>(chain ? pre_prev : cin, sum) : cin, rs);
      }
      if (!good) {  // the publisher sees the abort and marks this rank's remaining stripes for the others
        if (lane == 0) abort_from(j);
        return;
      }
      pre_prev = pre;
      if (lane == 0) {
        if (j >= RING && !tc::mbar_wait(&pempty[j % RING], rphase(j - RING), wait_ns, s_abort)) {
          abort_from(j);
          return;
        }
        s_prefix[j % RING] = pre;
        tc::mbar_arrive(&pfull[j % RING]);
      }
      __syncwarp();
    }
    return;
  }

  // ---------------- compute warps ----------------
  const int r = threadIdx.x;      // owns logical chunks 4r .. 4r+3 of every tile
  const int R = (lane >> 1) & 3;  // rotation of this thread's visiting order: lanes 2l and 2l+1 sit 64 bytes
                                  // apart, so this spreads each 8-lane phase over all 8 bank groups
  QCursor fc, rc;                 // the next tile to fold, the next tile to rescan
  fc.init(b, tiles_per_row);
  rc = fc;

  // Loads this thread's chunks of tile j (visiting order); chunks past the tile's end read as the identity.
  auto load_row = [&](int64_t j, int cnt, int32_t (&v)[kQRowChunks][4]) {
    const int4* buf = reinterpret_cast<const int4*>(stage(j));
    const int nch = cnt >> 2;  // whole 16-byte chunks (cnt % 4 == 0 here)
#pragma unroll
    for (int i = 0; i < kQRowChunks; ++i) {
      const int g = kQRowChunks * r + ((i + R) & 3);
      if (g < nch) {
        const int4 c = buf[REV ? nch - 1 - g : g];
        if (REV) { v[i][0] = c.w; v[i][1] = c.z; v[i][2] = c.y; v[i][3] = c.x; }
        else { v[i][0] = c.x; v[i][1] = c.y; v[i][2] = c.z; v[i][3] = c.w; }
      } else {
        v[i][0] = v[i][1] = v[i][2] = v[i][3] = id;
      }
    }
  };
  // Pass 1 on loaded chunks: chunk prefixes within the row, the row's warp-exclusive prefix, the warp total.
  auto fold_math = [&](int64_t j, const int32_t (&v)[kQRowChunks][4], QFold& st) {
#pragma unroll
    for (int i = 0; i < kQRowChunks; ++i) st.cp[i] = comb<OP>(comb<OP>(v[i][0], v[i][1]), comb<OP>(v[i][2], v[i][3]));
    rot_up4(st.cp, R);  // cp[c] = sum of chunk c of the row
    int32_t run = id;
#pragma unroll
    for (int c = 0; c < kQRowChunks; ++c) {
      const int32_t s = st.cp[c];
      st.cp[c] = run;
      run = comb<OP>(run, s);
    }
    rot_down4(st.cp, R);  // back to visiting order
    const int32_t inc = warp_incl_scan<OP>(run, lane);
    st.texcl = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 0) st.texcl = id;
    if (lane == 31) s_wt[j % RING][warp] = inc;
  };
  // After the barrier that follows fold_math: the tile's aggregate goes out as its look-back flag, and the
  // warp totals are replaced by their exclusive prefixes, which the tile's rescan reads one per warp.
  auto publish = [&](int64_t j, int64_t t) {
    if (threadIdx.x == 0) {
      int32_t run = id;
#pragma unroll
      for (int w = 0; w < kQCWarps; ++w) {
        const int32_t v = s_wt[j % RING][w];
        s_wt[j % RING][w] = run;
        run = comb<OP>(run, v);
      }
      if (!(withhold && t == 0)) st_relaxed_u64(flags + t, make_flag(epoch, kFlagAgg, run));
    }
  };

  QFold st[FOLD + 1];  // st[0]: the tile to rescan next; st[i]: the tile folded i tiles after it
  int64_t j = 0;
  bool ok = true;
  // prologue: fold the first FOLD tiles (unrolled, so the states stay in registers)
#pragma unroll
  for (int jf = 0; jf < FOLD; ++jf) {
    if (ok && jf < n_mine) {
      const int cnt = count_of(fc);
      const int64_t t = fc.t;
      fc.next(P, tiles_per_row);
      const bool landed = tc::mbar_wait(&full[jf % STAGES], sphase(jf), wait_ns, s_abort);
      int32_t v[kQRowChunks][4];
      load_row(jf, cnt, v);
      fold_math(jf, v, st[jf]);
      if (named_bar_or(1, kQCompute, !landed || *s_abort)) ok = false;
      else publish(jf, t);
    }
  }
  // Steady state: iteration j folds tile j + FOLD (publishing its aggregate as early as possible), then
  // rescans tile j. One barrier per iteration; it also settles whether any warp's wait for the previous
  // prefix ran out (such a warp releases nothing and has flagged the abort).
  bool good_prev = true;
  for (; ok && j < n_mine; ++j) {
    const bool fold_next = j + FOLD < n_mine;
    const int64_t jf = j + FOLD;
    bool good_f = true;
    int64_t ft = 0;
    if (fold_next) {
      const int fcnt = count_of(fc);
      ft = fc.t;
      fc.next(P, tiles_per_row);
      good_f = tc::mbar_wait(&full[jf % STAGES], sphase(jf), wait_ns, s_abort);
      int32_t fv[kQRowChunks][4];
      load_row(jf, fcnt, fv);
      fold_math(jf, fv, st[FOLD]);
    }
    if (named_bar_or(1, kQCompute, !good_f || !good_prev || *s_abort)) {
      ok = false;
      break;
    }
    if (fold_next) publish(jf, ft);

    // pass 2 of tile j
    const int rcnt = count_of(rc);
    rc.next(P, tiles_per_row);
    const bool gr = tc::mbar_wait(&pfull[j % RING], rphase(j), wait_ns, s_abort);
    int32_t rv[kQRowChunks][4];
    load_row(j, rcnt, rv);
    const int32_t pre = s_prefix[j % RING];
    const int32_t wpre = s_wt[j % RING][warp];  // exclusive prefix of this warp's rows (see publish)
    const int32_t base = comb<OP>(comb<OP>(pre, wpre), st[0].texcl);
    int4* wbuf = reinterpret_cast<int4*>(stage(j));
    const int nch = rcnt >> 2;
#pragma unroll
    for (int i = 0; i < kQRowChunks; ++i) {
      const int g = kQRowChunks * r + ((i + R) & 3);
      const int32_t p = comb<OP>(base, st[0].cp[i]);
      int32_t o[4];
      if (exclusive) {
        o[0] = p;
        o[1] = comb<OP>(p, rv[i][0]);
        o[2] = comb<OP>(o[1], rv[i][1]);
        o[3] = comb<OP>(o[2], rv[i][2]);
      } else {
        o[0] = comb<OP>(p, rv[i][0]);
        o[1] = comb<OP>(o[0], rv[i][1]);
        o[2] = comb<OP>(o[1], rv[i][2]);
        o[3] = comb<OP>(o[2], rv[i][3]);
      }
      if (g < nch) wbuf[REV ? nch - 1 - g : g] = REV ? make_int4(o[3], o[2], o[1], o[0]) : make_int4(o[0], o[1], o[2], o[3]);
    }
    tc::fence_proxy_async_smem();  // this thread's writes are visible to the bulk store
    const bool wgood = __all_sync(0xffffffffu, gr);
    if (lane == 0) {
      if (wgood) {  // one arrival per warp
        tc::mbar_arrive(&done[j % STAGES]);
        tc::mbar_arrive(&pempty[j % RING]);
      } else {
        abort_from(j);  // stops the copy and look-back warps; the next barrier stops the compute warps
      }
    }
    good_prev = wgood;
#pragma unroll
    for (int q = 0; q < FOLD; ++q) st[q] = st[q + 1];
  }
  if (!ok && threadIdx.x == 0) abort_from(j);
}

// ---- per-launch epochs ----
//
// The flags carry the low 30 bits of a 64-bit launch count. Within one span of 2^30 launches (a "cycle") the tags
// are distinct, so a flag left by an earlier launch never matches a later one. Across a cycle boundary they
// repeat, so the first launch on a workspace in each cycle after the first clears the workspace's flags first.
// Workspaces cleared in the current cycle are remembered by address and size (a larger size clears again).
static std::mutex g_epoch_mu;
static uint64_t g_epoch64 = 0;
static uint64_t g_epoch_cycle = 0;
struct ClearedWs {
  const void* ws;
  size_t bytes;
};
static std::vector<ClearedWs> g_cleared;

static cudaError_t launch_epoch(void* workspace, size_t workspace_bytes, cudaStream_t s, uint32_t* epoch) {
  std::lock_guard<std::mutex> lk(g_epoch_mu);
  const uint64_t e = ++g_epoch64;
  const uint64_t cycle = e >> 30;
  *epoch = (uint32_t)(e & 0x3fffffffu);
  if (cycle != g_epoch_cycle) {
    g_epoch_cycle = cycle;
    g_cleared.clear();
  }
  if (cycle == 0) return cudaSuccess;  // the caller's zero-fill holds no tag of this cycle
  for (const ClearedWs& c : g_cleared)
    if (c.ws == workspace && c.bytes >= workspace_bytes) return cudaSuccess;
  // the flags only: the header keeps an unreported error word, and its ticket is already zero
  const cudaError_t r = cudaMemsetAsync(static_cast<char*>(workspace) + sizeof(ScanHeader), 0,
                                        workspace_bytes - sizeof(ScanHeader), s);
  if (r != cudaSuccess) return r;
  for (ClearedWs& c : g_cleared)
    if (c.ws == workspace) {
      c.bytes = workspace_bytes;
      return cudaSuccess;
    }
  g_cleared.push_back({workspace, workspace_bytes});
  return cudaSuccess;
}

// rows x ceil(k / tile) into *out when it is at most `cap`, without overflowing on any int64 extents.
static bool tile_count(int64_t rows, int64_t k, int64_t tile, int64_t cap, int64_t* out) {
  if (rows <= 0 || k <= 0) {
    *out = 0;
    return true;
  }
  const int64_t per_row = (k - 1) / tile + 1;
  if (per_row > cap / rows) return false;
  *out = rows * per_row;
  return true;
}
constexpr int64_t kMaxScanTiles = 0x7ffffffeLL;  // a grid dimension and a 32-bit ticket

}  // namespace up

using namespace up;

extern "C" size_t up_sm100_scan_workspace_bytes(int64_t rows, int64_t k) {
  // one flag per tile of the persistent form (8192 elements); the one-tile-per-CTA form needs fewer
  int64_t tiles = 0;
  if (!tile_count(rows, k, kQTile, kMaxScanTiles, &tiles)) return SIZE_MAX;  // refused by up_sm100_scan_i32
  return sizeof(ScanHeader) + (size_t)tiles * sizeof(uint64_t);
}

template <int OP>
static cudaError_t launch_scan(unsigned grid, cudaStream_t s, const int32_t* x, int32_t* y, int64_t k, int64_t tpr,
                               int exclusive, int reverse, const int32_t* carry_in, ScanHeader* hdr, uint64_t* flags,
                               uint32_t epoch, uint64_t wns, int withhold) {
  cudaError_t e = ensure_smem_attr((const void*)scan_i32_kernel<OP>, (int)kScanSmem);
  if (e != cudaSuccess) return e;
  scan_i32_kernel<OP><<<grid, kScanThreads, kScanSmem, s>>>(x, y, k, tpr, exclusive, reverse, carry_in, hdr, flags,
                                                            epoch, wns, withhold);
  return cudaGetLastError();
}

template <int OP, bool REV>
static cudaError_t launch_scan_persist_dir(unsigned grid, cudaStream_t s, const int32_t* x, int32_t* y, int64_t k,
                                           int64_t tpr, int64_t tiles, int exclusive, const int32_t* carry_in,
                                           ScanHeader* hdr, uint64_t* flags, uint32_t epoch, uint64_t wns,
                                           int withhold) {
  cudaError_t e = ensure_smem_attr((const void*)scan_i32_persist_kernel<OP, REV>, (int)kQSmem);
  if (e != cudaSuccess) return e;
  scan_i32_persist_kernel<OP, REV><<<grid, kQThreads, kQSmem, s>>>(x, y, k, tpr, tiles, exclusive, carry_in, hdr,
                                                                   flags, epoch, wns, withhold, MultiScan{});
  return cudaGetLastError();
}

template <int OP>
static cudaError_t launch_scan_persist(unsigned grid, cudaStream_t s, const int32_t* x, int32_t* y, int64_t k,
                                       int64_t tpr, int64_t tiles, int exclusive, int reverse,
                                       const int32_t* carry_in, ScanHeader* hdr, uint64_t* flags, uint32_t epoch,
                                       uint64_t wns, int withhold) {
  return reverse ? launch_scan_persist_dir<OP, true>(grid, s, x, y, k, tpr, tiles, exclusive, carry_in, hdr, flags,
                                                     epoch, wns, withhold)
                 : launch_scan_persist_dir<OP, false>(grid, s, x, y, k, tpr, tiles, exclusive, carry_in, hdr, flags,
                                                      epoch, wns, withhold);
}

namespace up {
// Sets every scan kernel's shared-memory limit in the current context, and answers whether one CTA of the
// persistent form fits on an SM (it needs 197 KiB of shared memory and 576 threads; a context whose carveout or
// register budget is smaller cannot hold it, and the scan then takes the general form).
static cudaError_t scan_setup(bool* persistent_fits) {
  const void* general[3] = {(const void*)scan_i32_kernel<UP_OP_SUM>, (const void*)scan_i32_kernel<UP_OP_MAX>,
                            (const void*)scan_i32_kernel<UP_OP_MIN>};
  const void* persist[6] = {
      (const void*)scan_i32_persist_kernel<UP_OP_SUM, false>, (const void*)scan_i32_persist_kernel<UP_OP_SUM, true>,
      (const void*)scan_i32_persist_kernel<UP_OP_MAX, false>, (const void*)scan_i32_persist_kernel<UP_OP_MAX, true>,
      (const void*)scan_i32_persist_kernel<UP_OP_MIN, false>, (const void*)scan_i32_persist_kernel<UP_OP_MIN, true>};
  for (const void* f : general) {
    const cudaError_t e = ensure_smem_attr(f, (int)kScanSmem);
    if (e != cudaSuccess) return e;
  }
  bool fits = true;
  for (const void* f : persist) {
    cudaError_t e = ensure_smem_attr(f, (int)kQSmem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, kQThreads, kQSmem);
    if (e != cudaSuccess) return e;
    fits = fits && per_sm >= 1;
  }
  *persistent_fits = fits;
  return cudaSuccess;
}

// scan_setup once per context: whether the persistent form can run here.
static int persistent_form_fits(bool* fits) {
  static std::mutex mu;
  static uint64_t ctx_done[64] = {0};
  static bool fit[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  const uint64_t ctx = context_id();
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && ctx != 0 && ctx_done[dev] == ctx) {
    *fits = fit[dev];
    return UP_OK;
  }
  bool f = false;
  e = scan_setup(&f);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev >= 0 && dev < 64) {
    ctx_done[dev] = ctx;
    fit[dev] = f;
  }
  *fits = f;
  return UP_OK;
}
}  // namespace up

extern "C" int up_sm100_scan_i32(const int32_t* x, int32_t* y, int64_t rows, int64_t k, int op, int exclusive,
                                 int reverse, const int32_t* carry_in, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  UP_CHECK_ARG(rows >= 0 && k >= 0);
  if (op != UP_OP_SUM && op != UP_OP_MAX && op != UP_OP_MIN) return UP_ERR_UNSUPPORTED;
  if (rows == 0 || k == 0) return UP_OK;
  UP_CHECK_ARG(x != nullptr && y != nullptr && workspace != nullptr);
  UP_CHECK_ARG(aligned(workspace, 64));
  int64_t qtiles = 0, tiles = 0;
  if (!tile_count(rows, k, kQTile, kMaxScanTiles, &qtiles) || !tile_count(rows, k, kScanTile, kMaxScanTiles, &tiles))
    return fail_with(UP_ERR_UNSUPPORTED, "scan_i32: more than 2^31 - 2 tiles");
  if (workspace_bytes < up_sm100_scan_workspace_bytes(rows, k)) return UP_ERR_INVALID;
  const int64_t tpr = tiles / rows;
  auto* hdr = static_cast<ScanHeader*>(workspace);
  auto* flags = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + sizeof(ScanHeader));
  bool fits = false;
  int st = persistent_form_fits(&fits);
  if (st != UP_OK) return st;
  // bulk copies need 16-byte aligned rows of whole 16-byte chunks
  const int bulk = fits && aligned(x, 16) && aligned(y, 16) && (k % 4 == 0);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t epoch = 0;
  cudaError_t e = launch_epoch(workspace, workspace_bytes, s, &epoch);
  if (e != cudaSuccess) return cuda_status(e);
  const int withhold = take_withhold_flag();
  const uint64_t wns = wait_limit_ns();
  if (bulk) {
    const int64_t qtpr = qtiles / rows;
    int64_t grid = sm_count();
    if (grid > kQMaxGrid) grid = kQMaxGrid;
    if (grid > qtiles) grid = qtiles;
    const unsigned g = (unsigned)grid;
    if (op == UP_OP_SUM)
      e = launch_scan_persist<UP_OP_SUM>(g, s, x, y, k, qtpr, qtiles, exclusive, reverse, carry_in, hdr, flags, epoch,
                                         wns, withhold);
    else if (op == UP_OP_MAX)
      e = launch_scan_persist<UP_OP_MAX>(g, s, x, y, k, qtpr, qtiles, exclusive, reverse, carry_in, hdr, flags, epoch,
                                         wns, withhold);
    else
      e = launch_scan_persist<UP_OP_MIN>(g, s, x, y, k, qtpr, qtiles, exclusive, reverse, carry_in, hdr, flags, epoch,
                                         wns, withhold);
    note_launch();
    return cuda_status(e);
  }
  if (op == UP_OP_SUM)
    e = launch_scan<UP_OP_SUM>((unsigned)tiles, s, x, y, k, tpr, exclusive, reverse, carry_in, hdr, flags, epoch, wns,
                               withhold);
  else if (op == UP_OP_MAX)
    e = launch_scan<UP_OP_MAX>((unsigned)tiles, s, x, y, k, tpr, exclusive, reverse, carry_in, hdr, flags, epoch, wns,
                               withhold);
  else
    e = launch_scan<UP_OP_MIN>((unsigned)tiles, s, x, y, k, tpr, exclusive, reverse, carry_in, hdr, flags, epoch, wns,
                               withhold);
  note_launch();
  return cuda_status(e);
}

namespace up {
// One rank's pass of a scan over an array sharded block-cyclically across a communicator's ranks (stripes of
// kStripeTiles tiles of 8192 elements, stripe s on rank s % G): a single pass over the shard, with the cross-GPU
// look-back through the stripe words in `m`. Forward scans of one 16-byte aligned row of whole 16-byte chunks and
// at least kStripeTiles tiles, on a device that holds kStripeTiles persistent CTAs at once. Every rank launches it
// with the same k, op and exclusive flag.
int scan_i32_block_cyclic(const int32_t* x, int32_t* y, int64_t k, int op, int exclusive, const int32_t* carry_in,
                          void* workspace, size_t workspace_bytes, const MultiScan& m, cudaStream_t s) {
  if (op != UP_OP_SUM && op != UP_OP_MAX && op != UP_OP_MIN) return UP_ERR_UNSUPPORTED;
  if (x == nullptr || y == nullptr || workspace == nullptr || !aligned(workspace, 64)) return UP_ERR_INVALID;
  if (!aligned(x, 16) || !aligned(y, 16) || k % 4 != 0)
    return fail_with(UP_ERR_UNSUPPORTED, "block-cyclic scan: 16-byte aligned shards of whole 16-byte chunks");
  int64_t tiles = 0;
  if (!tile_count(1, k, kQTile, kMaxScanTiles, &tiles) || tiles < kStripeTiles)
    return fail_with(UP_ERR_UNSUPPORTED, "block-cyclic scan: a shard holds at least 148 tiles of 8192 elements");
  if (workspace_bytes < up_sm100_scan_workspace_bytes(1, k)) return UP_ERR_INVALID;
  bool fits = false;
  int st = persistent_form_fits(&fits);
  if (st != UP_OK) return st;
  if (!fits || sm_count() < kStripeTiles)
    return fail_with(UP_ERR_UNSUPPORTED, "block-cyclic scan: the device must hold 148 persistent CTAs at once");
  auto* hdr = static_cast<ScanHeader*>(workspace);
  auto* flags = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + sizeof(ScanHeader));
  uint32_t epoch = 0;
  cudaError_t e = launch_epoch(workspace, workspace_bytes, s, &epoch);
  if (e != cudaSuccess) return cuda_status(e);
  const void* fn = op == UP_OP_SUM   ? (const void*)scan_i32_persist_kernel<UP_OP_SUM, false, true>
                   : op == UP_OP_MAX ? (const void*)scan_i32_persist_kernel<UP_OP_MAX, false, true>
                                     : (const void*)scan_i32_persist_kernel<UP_OP_MIN, false, true>;
  e = ensure_smem_attr(fn, (int)kQSmemMulti);
  if (e != cudaSuccess) return cuda_status(e);
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kQThreadsMulti, kQSmemMulti);
  if (e != cudaSuccess) return cuda_status(e);
  if (per_sm < 1) return fail_with(UP_ERR_UNSUPPORTED, "block-cyclic scan: its CTA does not fit on an SM");
  const uint64_t wns = wait_limit_ns();
  const int withhold = take_withhold_flag();
  if (op == UP_OP_SUM)
    scan_i32_persist_kernel<UP_OP_SUM, false, true><<<kStripeTiles, kQThreadsMulti, kQSmemMulti, s>>>(
        x, y, k, tiles, tiles, exclusive, carry_in, hdr, flags, epoch, wns, withhold, m);
  else if (op == UP_OP_MAX)
    scan_i32_persist_kernel<UP_OP_MAX, false, true><<<kStripeTiles, kQThreadsMulti, kQSmemMulti, s>>>(
        x, y, k, tiles, tiles, exclusive, carry_in, hdr, flags, epoch, wns, withhold, m);
  else
    scan_i32_persist_kernel<UP_OP_MIN, false, true><<<kStripeTiles, kQThreadsMulti, kQSmemMulti, s>>>(
        x, y, k, tiles, tiles, exclusive, carry_in, hdr, flags, epoch, wns, withhold, m);
  note_launch();
  return check_launch();
}

// Stripe words a block-cyclic scan of a shard of k elements needs on each of G ranks: one per global stripe.
int64_t block_cyclic_stripe_words(int64_t k, int G) {
  const int64_t tiles = (k + kQTile - 1) / kQTile;
  return ((tiles + kStripeTiles - 1) / kStripeTiles) * G;
}
}  // namespace up

extern "C" void up_sm100_set_test_scan_epoch(uint64_t next) {
  std::lock_guard<std::mutex> lk(g_epoch_mu);
  g_epoch64 = next - 1;
}

extern "C" int up_sm100_workspace_status(void* workspace, void* stream) {
  UP_CHECK_ARG(workspace != nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* hdr = static_cast<ScanHeader*>(workspace);
  uint32_t err = 0;
  cudaError_t e = cudaMemcpyAsync(&err, &hdr->error, sizeof(err), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e);
  if (err) {
    const uint32_t zero = 0;
    e = cudaMemcpyAsync(&hdr->error, &zero, sizeof(zero), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e);
    return UP_ERR_DEVICE_TIMEOUT;
  }
  return UP_OK;
}

// ---- scan with built-in scratch, for callers that cannot allocate ----
//
// The look-back flags and the error word live in one file-scope device array instead of a caller's
// workspace. Each device holds its own copy of the array, zero from module load. What must be zero is
// the error word, and it is cleared again whenever a timeout is reported; the flags are epoch-tagged
// (and cleared by the launch that follows a wrap of the tag, as for any workspace). Every call on a device
// uses the same array: calls that overlap in time race, through concurrent streams or host threads, and
// must be serialized by the caller.
namespace up {
constexpr int64_t kNoAllocMaxTiles = 32768;  // rows x ceil(k / 8192) tiles, e.g. one row of 2^28 elements
static __device__ __align__(256) uint64_t g_noalloc_scratch[sizeof(ScanHeader) / 8 + kNoAllocMaxTiles];
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {};
static uint64_t g_noalloc_ctx[64] = {};

// Set-up, once per device and context, with that device current: the device address of this device's copy of
// the scratch, and every scan kernel's shared-memory limit. A cudaDeviceReset ends the context the address
// belongs to; the next call sees a new context and does the set-up again.
static int noalloc_setup(int dev, void** out) {
  const uint64_t ctx = context_id();
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (ctx == 0 || g_noalloc_ctx[dev] != ctx || g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    bool fits = false;
    const int st = persistent_form_fits(&fits);
    if (st != UP_OK) return st;
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return UP_OK;
}
}  // namespace up

extern "C" int up_sm100_scan_i32_noalloc(const int32_t* x, int32_t* y, int64_t rows, int64_t k, int op,
                                         int exclusive, int reverse, const int32_t* carry_in, int sync,
                                         void* stream) {
  UP_CHECK_ARG(rows >= 0 && k >= 0);
  if (op != UP_OP_SUM && op != UP_OP_MAX && op != UP_OP_MIN) return UP_ERR_UNSUPPORTED;
  if (rows == 0 || k == 0) return UP_OK;
  int64_t tiles = 0;
  if (!tile_count(rows, k, kQTile, kNoAllocMaxTiles, &tiles))
    return fail_with(UP_ERR_UNSUPPORTED,
                     "up_sm100_scan_i32_noalloc: rows * ceil(k / 8192) exceeds the built-in scratch's 32768 "
                     "tiles; use up_sm100_scan_i32 with a workspace");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 64) return fail_with(UP_ERR_UNSUPPORTED, "up_sm100_scan_i32_noalloc: device index >= 64");
  void* scratch = nullptr;
  int st = noalloc_setup(dev, &scratch);
  if (st != UP_OK) return st;
  st = up_sm100_scan_i32(x, y, rows, k, op, exclusive, reverse, carry_in, scratch, sizeof(g_noalloc_scratch),
                         stream);
  if (st != UP_OK || !sync) return st;
  return up_sm100_workspace_status(scratch, stream);
}

namespace up {
size_t scan_persist_smem_bytes() { return kQSmem; }  // for the kernel interface
}  // namespace up

UP_DEFINE_REVISION(scan)
