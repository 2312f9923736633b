// scan.cu — single-pass int32 scans (inclusive / exclusive; SUM wrapping, MAX, MIN; forward / reverse)
// by decoupled look-back, for sm_100a.
//
// Semantics: `Access::Scan` (crates/unpopped/src/ir.rs:2153-2195) as the oracle evaluates it
// (crates/unpopped/src/oracle/plan_window.rs:10-238): per row of k elements, an inclusive scan writes
// after the combine, an exclusive scan before it (so element 0 gets the monoid identity: 0, INT32_MIN,
// INT32_MAX); Sum wraps at 32 bits; a reverse scan walks from the row's end. Integer combines are exact
// and associative, so the tile decomposition below produces the serial walk's bytes.
//
// Decomposition: a tile is 4096 consecutive elements of one row (the row's last tile may be short).
// CTAs take tiles in ticket order (an atomic counter), so every tile's predecessors belong to CTAs that
// are already running or done — the look-back cannot wait on a CTA that has not started.
// Within a tile, warp w owns elements [w*512, w*512+512); lane l holds the int4 groups i*32 + l
// (i = 0..3), which makes every load and store one contiguous 512-byte warp access.
//
// Look-back flags: one 64-bit word per tile = epoch(30) | status(2) | value(32), written and read with
// relaxed gpu-scope atomics (the value travels inside the flag word, so no separate fence is needed).
// Status: 1 = aggregate of this tile, 2 = inclusive prefix through this tile, 3 = aborted. The epoch is
// bumped by the last CTA of every launch, which also resets the ticket counters, so the workspace needs
// zero-filling only once. Every wait is bounded by a globaltimer deadline; a wait that runs out sets the
// workspace error word and publishes "aborted", which its successors propagate at once.
#include "common.cuh"

namespace up {

constexpr int kScanThreads = 256;
constexpr int kScanVecs = 4;                                    // int4 per thread
constexpr int kScanTile = kScanThreads * kScanVecs * 4;         // 4096 elements
constexpr int kWarpSeg = kScanVecs * 4 * 32;                    // 512 elements per warp

struct ScanHeader {
  uint32_t ticket;
  uint32_t done;
  uint32_t epoch;
  uint32_t error;
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

template <int OP>
__global__ void __launch_bounds__(kScanThreads) scan_i32_kernel(const int32_t* __restrict__ x,
                                                                int32_t* __restrict__ y, int64_t k,
                                                                int64_t tiles_per_row, int64_t num_tiles,
                                                                int exclusive, int reverse,
                                                                const int32_t* carry_in, ScanHeader* hdr,
                                                                uint64_t* flags, uint64_t wait_ns,
                                                                int withhold, int vec_ok) {
  __shared__ int64_t s_tile;
  __shared__ uint32_t s_epoch;
  __shared__ int32_t s_warp_tot[kScanThreads / 32];
  __shared__ int32_t s_prefix;
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    s_tile = (int64_t)atomicAdd(&hdr->ticket, 1u);
    s_epoch = ld_relaxed_u32(&hdr->epoch);
    s_abort = 0;
  }
  __syncthreads();
  const int64_t t = s_tile;
  const uint32_t epoch = s_epoch;
  const int64_t row = t / tiles_per_row;
  const int64_t q = t - row * tiles_per_row;
  const int64_t lo = q * kScanTile;
  const bool full = (lo + kScanTile <= k) && vec_ok;
  const int32_t* xr = x + row * k;
  int32_t* yr = y + row * k;
  const int32_t id = ident<OP>();

  // ---- load (logical order; reversed rows are read back to front) ----
  int32_t v[kScanVecs][4];
#pragma unroll
  for (int i = 0; i < kScanVecs; ++i) {
    const int64_t e0 = lo + warp * kWarpSeg + (i * 32 + lane) * 4;
    if (full) {
      if (!reverse) {
        const uint4 u = ld_nc_na_v4(xr + e0);
        v[i][0] = (int32_t)u.x; v[i][1] = (int32_t)u.y; v[i][2] = (int32_t)u.z; v[i][3] = (int32_t)u.w;
      } else {
        const uint4 u = ld_nc_na_v4(xr + (k - e0 - 4));
        v[i][0] = (int32_t)u.w; v[i][1] = (int32_t)u.z; v[i][2] = (int32_t)u.y; v[i][3] = (int32_t)u.x;
      }
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int64_t e = e0 + c;
        v[i][c] = e < k ? __ldg(xr + (reverse ? k - 1 - e : e)) : id;
      }
    }
  }

  // ---- thread-local scans of each 4-group, warp scans of the group totals ----
  int32_t gex[kScanVecs];  // exclusive prefix of group (i, lane) within the warp segment
  int32_t carry = id;      // warp-uniform running total over i
#pragma unroll
  for (int i = 0; i < kScanVecs; ++i) {
    v[i][1] = comb<OP>(v[i][0], v[i][1]);
    v[i][2] = comb<OP>(v[i][1], v[i][2]);
    v[i][3] = comb<OP>(v[i][2], v[i][3]);
    const int32_t inc = warp_incl_scan<OP>(v[i][3], lane);
    int32_t exc = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 0) exc = id;
    gex[i] = comb<OP>(carry, exc);
    carry = comb<OP>(carry, __shfl_sync(0xffffffffu, inc, 31));
  }
  if (lane == 0) s_warp_tot[warp] = carry;
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
    bool abort = false;
    if (q == 0) {
      excl = cin;
      if (lane == 0 && !(withhold && t == 0)) st_relaxed_u64(flags + t, make_flag(epoch, kFlagIncl, comb<OP>(cin, agg)));
    } else {
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
          __nanosleep(64);
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
        if (abort) {
          atomicOr(&hdr->error, 1u);
          st_relaxed_u64(flags + t, make_flag(epoch, kFlagErr, 0));
        } else {
          st_relaxed_u64(flags + t, make_flag(epoch, kFlagIncl, comb<OP>(excl, agg)));
        }
      }
    }
    if (lane == 0) {
      s_prefix = excl;
      s_abort = abort ? 1 : 0;
    }
  }
  __syncthreads();

  // ---- store ----
  if (!s_abort) {
    const int32_t base = comb<OP>(s_prefix, wpre);
#pragma unroll
    for (int i = 0; i < kScanVecs; ++i) {
      const int32_t pre = comb<OP>(base, gex[i]);
      int32_t o[4];
      if (exclusive) {
        o[0] = pre;
        o[1] = comb<OP>(pre, v[i][0]);
        o[2] = comb<OP>(pre, v[i][1]);
        o[3] = comb<OP>(pre, v[i][2]);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) o[c] = comb<OP>(pre, v[i][c]);
      }
      const int64_t e0 = lo + warp * kWarpSeg + (i * 32 + lane) * 4;
      if (full) {
        if (!reverse) st_cs_v4(yr + e0, make_uint4((uint32_t)o[0], (uint32_t)o[1], (uint32_t)o[2], (uint32_t)o[3]));
        else st_cs_v4(yr + (k - e0 - 4), make_uint4((uint32_t)o[3], (uint32_t)o[2], (uint32_t)o[1], (uint32_t)o[0]));
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int64_t e = e0 + c;
          if (e < k) yr[reverse ? k - 1 - e : e] = o[c];
        }
      }
    }
  }

  // ---- the last CTA of the launch re-arms the workspace for the next one ----
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t d = atomicAdd(&hdr->done, 1u);
    if ((int64_t)d == num_tiles - 1) {
      atomicExch(&hdr->ticket, 0u);
      atomicExch(&hdr->done, 0u);
      __threadfence();
      atomicAdd(&hdr->epoch, 1u);
    }
  }
}

}  // namespace up

using namespace up;

extern "C" size_t up_sm100_scan_workspace_bytes(int64_t rows, int64_t k) {
  if (rows <= 0 || k <= 0) return sizeof(ScanHeader);
  const int64_t tiles = rows * ((k + kScanTile - 1) / kScanTile);
  return sizeof(ScanHeader) + (size_t)tiles * sizeof(uint64_t);
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
  const int vec_ok = aligned(x, 16) && aligned(y, 16) && (k % 4 == 0);
  const int withhold = take_withhold_flag();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint64_t wns = wait_limit_ns();
  if (op == UP_OP_SUM)
    scan_i32_kernel<UP_OP_SUM><<<(unsigned)tiles, kScanThreads, 0, s>>>(x, y, k, tpr, tiles, exclusive, reverse,
                                                                       carry_in, hdr, flags, wns, withhold, vec_ok);
  else if (op == UP_OP_MAX)
    scan_i32_kernel<UP_OP_MAX><<<(unsigned)tiles, kScanThreads, 0, s>>>(x, y, k, tpr, tiles, exclusive, reverse,
                                                                       carry_in, hdr, flags, wns, withhold, vec_ok);
  else
    scan_i32_kernel<UP_OP_MIN><<<(unsigned)tiles, kScanThreads, 0, s>>>(x, y, k, tpr, tiles, exclusive, reverse,
                                                                       carry_in, hdr, flags, wns, withhold, vec_ok);
  note_launch();
  return check_launch();
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
