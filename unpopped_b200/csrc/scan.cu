// scan.cu — single-pass int32 scans (inclusive / exclusive; SUM wrapping, MAX, MIN; forward / reverse)
// by decoupled look-back, for sm_100a.
//
// Semantics: `Access::Scan` (crates/unpopped/src/ir.rs:2153-2195) as the oracle evaluates it
// (crates/unpopped/src/oracle/plan_window.rs:10-238): per row of k elements, an inclusive scan writes
// after the combine, an exclusive scan before it (so element 0 gets the monoid identity: 0, INT32_MIN,
// INT32_MAX); Sum wraps at 32 bits; a reverse scan walks from the row's end. Integer combines are exact
// and associative, so the tile decomposition below produces the serial walk's bytes.
//
// Decomposition: a tile is 16384 consecutive elements (64 KiB) of one row (the row's last tile may be
// short); CTA i scans tile i. One thread moves the tile into shared memory with bulk copies
// (cp.async.bulk, no multicast) and back out with bulk stores, so the loads in flight cost no registers and
// three tiles per SM stream concurrently. In shared memory, warp w owns 2048 elements; lane l handles the
// 16-byte chunks i*32 + l (i = 0..15), which keeps every shared-memory access conflict-free. Pass 1 folds
// the tile; the tile's aggregate goes out as a look-back flag; pass 2 rescans from shared memory with the
// prefix found by the look-back and writes the result in place.
//
// Look-back: one 64-bit flag per tile = epoch(30) | status(2) | value(32), written and read with relaxed
// gpu-scope atomics (the value travels inside the flag word). Status: 1 = aggregate of this tile,
// 2 = inclusive prefix through this tile, 3 = aborted. Warp 0 examines 32 predecessors per step. CTAs are
// dispatched in index order, so a tile only ever waits on tiles whose CTAs have started. The epoch is a
// per-launch number chosen on the host, so flags of earlier launches are never mistaken for this one's and
// the workspace needs zero-filling only once. Every wait is bounded by a globaltimer deadline; a wait that
// runs out sets the workspace error word and publishes "aborted", which successors propagate at once.
#include "common.cuh"
#include "tc.cuh"

#include <atomic>
#include <mutex>

namespace up {

constexpr int kScanThreads = 256;
constexpr int kLaneChunks = 16;                                  // 16-byte chunks per lane
constexpr int kScanTile = kScanThreads * kLaneChunks * 4;        // 16384 elements
constexpr int kWarpChunks = 32 * kLaneChunks;                    // 512 chunks = 2048 elements per warp
constexpr int kTileBytes = kScanTile * 4;                        // 64 KiB
constexpr size_t kScanSmem = kTileBytes + 64;                    // + the tile's mbarrier

struct ScanHeader {
  uint32_t reserved0, reserved1, reserved2;
  uint32_t error;  // byte 12: set when a bounded wait ran out
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

// The tile in shared memory, read and written by logical chunk (elements 4g .. 4g+3 in scan order).
// `rev`: the tile is stored back to front (a reverse scan that was bulk-loaded); `cnt`: valid elements.
template <int OP>
struct TileView {
  int32_t* buf;
  int cnt;
  bool rev;
  __device__ __forceinline__ void load(int g, int32_t (&v)[4]) const {
    const int e0 = 4 * g;
    if (e0 + 4 <= cnt) {
      const int4 c = rev ? reinterpret_cast<const int4*>(buf)[(cnt >> 2) - 1 - g] : reinterpret_cast<const int4*>(buf)[g];
      if (rev) { v[0] = c.w; v[1] = c.z; v[2] = c.y; v[3] = c.x; }
      else { v[0] = c.x; v[1] = c.y; v[2] = c.z; v[3] = c.w; }
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) v[c] = (e0 + c < cnt) ? buf[e0 + c] : ident<OP>();  // only unreversed here
    }
  }
  __device__ __forceinline__ void store(int g, const int32_t (&o)[4]) const {
    const int e0 = 4 * g;
    if (e0 + 4 <= cnt) {
      if (rev) reinterpret_cast<int4*>(buf)[(cnt >> 2) - 1 - g] = make_int4(o[3], o[2], o[1], o[0]);
      else reinterpret_cast<int4*>(buf)[g] = make_int4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (e0 + c < cnt) buf[e0 + c] = o[c];
    }
  }
};

template <int OP>
__global__ void __launch_bounds__(kScanThreads) scan_i32_kernel(const int32_t* __restrict__ x,
                                                                int32_t* __restrict__ y, int64_t k,
                                                                int64_t tiles_per_row, int exclusive, int reverse,
                                                                const int32_t* carry_in, ScanHeader* hdr,
                                                                uint64_t* flags, uint32_t epoch, uint64_t wait_ns,
                                                                int withhold, int bulk) {
  extern __shared__ __align__(128) uint8_t smem[];
  int32_t* buf = reinterpret_cast<int32_t*>(smem);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kTileBytes);
  __shared__ int32_t s_warp_tot[kScanThreads / 32];
  __shared__ int32_t s_prefix;
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x;
  const int64_t row = t / tiles_per_row;
  const int64_t q = t - row * tiles_per_row;
  const int64_t lo = q * kScanTile;
  const int cnt = (int)((k - lo) < kScanTile ? (k - lo) : kScanTile);
  const int32_t* xr = x + row * k;
  int32_t* yr = y + row * k;
  const int64_t pstart = reverse ? (k - lo - cnt) : lo;  // first physical element of the tile
  const int32_t id = ident<OP>();

  // ---- bring the tile into shared memory ----
  if (threadIdx.x == 0) s_abort = 0;
  if (bulk) {
    if (threadIdx.x == 0) {
      tc::mbar_init(bar, 1);
      tc::mbar_fence_init();
      const uint32_t bytes = (uint32_t)cnt * 4u;
      tc::mbar_arrive_expect_tx(bar, bytes);
      const char* src = reinterpret_cast<const char*>(xr + pstart);
      for (uint32_t off = 0; off < bytes; off += 16384u)
        tc::bulk_load(smem + off, src + off, (bytes - off) < 16384u ? (bytes - off) : 16384u, bar);
    }
    __syncthreads();
    const bool ok = tc::mbar_wait(bar, 0, wait_ns, nullptr);
    if (__syncthreads_or(!ok)) {
      // the copy did not land in time: report, and let it land before this CTA's shared memory is released
      if (threadIdx.x == 0) {
        atomicOr(&hdr->error, 1u);
        s_abort = 1;
        tc::mbar_wait(bar, 0, wait_ns, nullptr);
      }
    }
  } else {
    // any alignment: element loads, stored in scan order (a reversed row is read back to front)
    for (int e = threadIdx.x; e < cnt; e += kScanThreads) buf[e] = __ldg(xr + (reverse ? (k - 1 - (lo + e)) : (lo + e)));
  }
  __syncthreads();
  const TileView<OP> tile{buf, cnt, bulk && reverse};

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
  if (bulk) {
    tc::fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t bytes = (uint32_t)cnt * 4u;
      char* dst = reinterpret_cast<char*>(yr + pstart);
      for (uint32_t off = 0; off < bytes; off += 16384u)
        tc::bulk_store(dst + off, smem + off, (bytes - off) < 16384u ? (bytes - off) : 16384u);
      tc::bulk_commit();
      tc::bulk_wait_read();
    }
  } else {
    __syncthreads();
    for (int e = threadIdx.x; e < cnt; e += kScanThreads) yr[reverse ? (k - 1 - (lo + e)) : (lo + e)] = buf[e];
  }
}

static std::atomic<uint32_t> g_epoch{0};

}  // namespace up

using namespace up;

extern "C" size_t up_sm100_scan_workspace_bytes(int64_t rows, int64_t k) {
  if (rows <= 0 || k <= 0) return sizeof(ScanHeader);
  const int64_t tiles = rows * ((k + kScanTile - 1) / kScanTile);
  return sizeof(ScanHeader) + (size_t)tiles * sizeof(uint64_t);
}

template <int OP>
static cudaError_t launch_scan(unsigned grid, cudaStream_t s, const int32_t* x, int32_t* y, int64_t k, int64_t tpr,
                               int exclusive, int reverse, const int32_t* carry_in, ScanHeader* hdr, uint64_t* flags,
                               uint32_t epoch, uint64_t wns, int withhold, int bulk) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  static bool attr_set[64] = {false};
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      e = cudaFuncSetAttribute(scan_i32_kernel<OP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kScanSmem);
      if (e != cudaSuccess) return e;
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
  }
  scan_i32_kernel<OP><<<grid, kScanThreads, kScanSmem, s>>>(x, y, k, tpr, exclusive, reverse, carry_in, hdr, flags,
                                                            epoch, wns, withhold, bulk);
  return cudaGetLastError();
}

extern "C" int up_sm100_scan_i32(const int32_t* x, int32_t* y, int64_t rows, int64_t k, int op, int exclusive,
                                 int reverse, const int32_t* carry_in, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  UP_CHECK_ARG(rows >= 0 && k >= 0);
  if (op != UP_OP_SUM && op != UP_OP_MAX && op != UP_OP_MIN) return UP_ERR_UNSUPPORTED;
  if (rows == 0 || k == 0) return UP_OK;
  UP_CHECK_ARG(x != nullptr && y != nullptr && workspace != nullptr);
  UP_CHECK_ARG(aligned(workspace, 64));
  const int64_t tpr = (k + kScanTile - 1) / kScanTile;
  const int64_t tiles = rows * tpr;
  if (tiles >= (int64_t)0x7fffffff) return UP_ERR_UNSUPPORTED;
  if (workspace_bytes < up_sm100_scan_workspace_bytes(rows, k)) return UP_ERR_INVALID;
  auto* hdr = static_cast<ScanHeader*>(workspace);
  auto* flags = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + sizeof(ScanHeader));
  // bulk copies need 16-byte aligned rows of whole 16-byte chunks
  const int bulk = aligned(x, 16) && aligned(y, 16) && (k % 4 == 0);
  const int withhold = take_withhold_flag();
  const uint32_t epoch = ++g_epoch;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint64_t wns = wait_limit_ns();
  cudaError_t e;
  if (op == UP_OP_SUM)
    e = launch_scan<UP_OP_SUM>((unsigned)tiles, s, x, y, k, tpr, exclusive, reverse, carry_in, hdr, flags, epoch, wns,
                               withhold, bulk);
  else if (op == UP_OP_MAX)
    e = launch_scan<UP_OP_MAX>((unsigned)tiles, s, x, y, k, tpr, exclusive, reverse, carry_in, hdr, flags, epoch, wns,
                               withhold, bulk);
  else
    e = launch_scan<UP_OP_MIN>((unsigned)tiles, s, x, y, k, tpr, exclusive, reverse, carry_in, hdr, flags, epoch, wns,
                               withhold, bulk);
  note_launch();
  return cuda_status(e);
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
// the error word, and it is cleared again whenever a timeout is reported. The flags are epoch-tagged,
// so they never need clearing. Every call on a device uses the same array: calls that overlap in time
// race, through concurrent streams or host threads, and must be serialized by the caller.
namespace up {
constexpr int64_t kNoAllocMaxTiles = 16384;  // rows x ceil(k / 16384) tiles, e.g. one row of 2^28 elements
static __device__ __align__(256) uint64_t g_noalloc_scratch[sizeof(ScanHeader) / 8 + kNoAllocMaxTiles];
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {};

// The device address of this device's copy of the scratch, looked up once per device (with it current).
static cudaError_t noalloc_scratch(int dev, void** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}
}  // namespace up

extern "C" int up_sm100_scan_i32_noalloc(const int32_t* x, int32_t* y, int64_t rows, int64_t k, int op,
                                         int exclusive, int reverse, const int32_t* carry_in, int sync,
                                         void* stream) {
  UP_CHECK_ARG(rows >= 0 && k >= 0);
  if (op != UP_OP_SUM && op != UP_OP_MAX && op != UP_OP_MIN) return UP_ERR_UNSUPPORTED;
  if (rows == 0 || k == 0) return UP_OK;
  const int64_t tpr = (k + kScanTile - 1) / kScanTile;
  if (rows > kNoAllocMaxTiles || rows * tpr > kNoAllocMaxTiles)
    return fail_with(UP_ERR_UNSUPPORTED,
                     "up_sm100_scan_i32_noalloc: rows * ceil(k / 16384) exceeds the built-in scratch's 16384 "
                     "tiles; use up_sm100_scan_i32 with a workspace");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 64) return fail_with(UP_ERR_UNSUPPORTED, "up_sm100_scan_i32_noalloc: device index >= 64");
  void* scratch = nullptr;
  e = noalloc_scratch(dev, &scratch);
  if (e != cudaSuccess) return cuda_status(e);
  const int st = up_sm100_scan_i32(x, y, rows, k, op, exclusive, reverse, carry_in, scratch,
                                   sizeof(g_noalloc_scratch), stream);
  if (st != UP_OK || !sync) return st;
  return up_sm100_workspace_status(scratch, stream);
}
