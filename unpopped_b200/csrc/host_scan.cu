// host_scan.cu — the int32 scan over HOST memory (up_sm100_scan_i32_host).
//
// The reference evaluates a scan over host buffers (crates/unpopped/src/oracle/plan_window.rs:10-238, the same
// semantics as up_sm100_scan_i32). This entry takes those same host buffers. The array streams
// through a ring of device slots: a copy-in stream, a scan stream and a copy-out stream, ordered by events,
// so the host-to-device copy of chunk i+1, the scan of chunk i and the device-to-host copy of chunk i-1
// run at once. Both directions of the host link are busy together.
//
// Chunks: rows longer than a slot are cut along the row; each later chunk of a row starts from the carry
// of the chunk before it (its edge output, combined with its edge input when the scan is exclusive), which
// a one-thread kernel derives on the device, so the host never waits inside a row. Shorter rows travel as
// groups of whole rows, each group one launch with the caller's carry.
#include <mutex>
#include <vector>

#include "common.cuh"

namespace up {
namespace {

constexpr int kSlots = 4;
constexpr int64_t kSlotElems = int64_t(1) << 23;  // 32 MiB of int32 per slot and direction
constexpr int64_t kMaxTiles = 65536;              // look-back tiles per launch (scan workspace of 512 KiB)

// The inclusive total through a chunk: its edge output, combined with its edge input for an exclusive scan.
__global__ void scan_chunk_carry_kernel(int op, const int32_t* y_edge, const int32_t* x_edge, int32_t* carry) {
  int32_t v = *y_edge;
  if (x_edge != nullptr) {
    const int32_t a = *x_edge;
    v = op == UP_OP_SUM ? (int32_t)((uint32_t)v + (uint32_t)a) : op == UP_OP_MAX ? (a > v ? a : v) : (a < v ? a : v);
  }
  *carry = v;
}

struct Chunk {
  int64_t row0, nrow;  // rows [row0, row0 + nrow)
  int64_t k0, len;     // columns [k0, k0 + len) of each of those rows
  bool carry_from_prev;
  bool carry_to_next;
};

struct Streamer {
  bool ready = false;
  uint64_t ctx = 0;  // the context the slots and streams belong to
  cudaStream_t h2d = nullptr, comp = nullptr, d2h = nullptr;
  int32_t* xs = nullptr;  // kSlots x kSlotElems
  int32_t* ys = nullptr;
  int32_t* carry = nullptr;  // [0] the caller's carry, [1], [2] the carries between chunks (alternating)
  void* ws = nullptr;
  size_t ws_bytes = 0;
  cudaEvent_t h2d_done[kSlots], scan_done[kSlots], d2h_done[kSlots];
};

std::mutex g_mu;
Streamer g_st[64];

// Allocates the slots, streams and events once per device and context. After a cudaDeviceReset the old ones died
// with their context, so a new context starts from nothing.
int setup(Streamer& st) {
  const uint64_t ctx = context_id();
  if (st.ready && (ctx == 0 || st.ctx == ctx)) return UP_OK;
  st = Streamer{};
  cudaError_t e = cudaSuccess;
  auto ok = [&](cudaError_t r) {
    if (e == cudaSuccess) e = r;
    return e == cudaSuccess;
  };
  ok(cudaStreamCreateWithFlags(&st.h2d, cudaStreamNonBlocking));
  ok(cudaStreamCreateWithFlags(&st.comp, cudaStreamNonBlocking));
  ok(cudaStreamCreateWithFlags(&st.d2h, cudaStreamNonBlocking));
  ok(cudaMalloc(&st.xs, sizeof(int32_t) * kSlots * kSlotElems));
  ok(cudaMalloc(&st.ys, sizeof(int32_t) * kSlots * kSlotElems));
  ok(cudaMalloc(&st.carry, 64));
  st.ws_bytes = 64 + 8 * (size_t)kMaxTiles;
  ok(cudaMalloc(&st.ws, st.ws_bytes));
  ok(cudaMemset(st.ws, 0, st.ws_bytes));
  for (int s = 0; s < kSlots; ++s) {
    ok(cudaEventCreateWithFlags(&st.h2d_done[s], cudaEventDisableTiming));
    ok(cudaEventCreateWithFlags(&st.scan_done[s], cudaEventDisableTiming));
    ok(cudaEventCreateWithFlags(&st.d2h_done[s], cudaEventDisableTiming));
  }
  ok(cudaDeviceSynchronize());
  if (e != cudaSuccess) return cuda_status(e);
  st.ready = true;
  st.ctx = ctx;
  return UP_OK;
}

std::vector<Chunk> plan_chunks(int64_t rows, int64_t k, bool reverse) {
  std::vector<Chunk> cs;
  if (k > kSlotElems) {
    const int64_t n = (k + kSlotElems - 1) / kSlotElems;
    for (int64_t r = 0; r < rows; ++r)
      for (int64_t j = 0; j < n; ++j) {
        const int64_t q = reverse ? n - 1 - j : j;  // a reverse scan starts from the row's end
        const int64_t k0 = q * kSlotElems;
        cs.push_back({r, 1, k0, (k - k0 < kSlotElems ? k - k0 : kSlotElems), j > 0, j + 1 < n});
      }
  } else {
    const int64_t tiles_per_row = (k + 8191) / 8192;
    int64_t per = kSlotElems / k;
    if (per > kMaxTiles / tiles_per_row) per = kMaxTiles / tiles_per_row;
    for (int64_t r0 = 0; r0 < rows; r0 += per) cs.push_back({r0, rows - r0 < per ? rows - r0 : per, 0, k, false, false});
  }
  return cs;
}

}  // namespace
}  // namespace up

using namespace up;

extern "C" int up_sm100_scan_i32_host(const int32_t* x, int32_t* y, int64_t rows, int64_t k, int op, int exclusive,
                                      int reverse, const int32_t* carry_in) {
  if (rows < 0 || k < 0) return fail_with(UP_ERR_INVALID, "scan_i32_host: negative extent");
  if (op != UP_OP_SUM && op != UP_OP_MAX && op != UP_OP_MIN)
    return fail_with(UP_ERR_UNSUPPORTED, "scan_i32_host: op must be SUM, MAX or MIN");
  if (rows == 0 || k == 0) return UP_OK;
  if (x == nullptr || y == nullptr) return fail_with(UP_ERR_INVALID, "scan_i32_host: null buffer");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail_with(UP_ERR_CUDA, "scan_i32_host: no current device");
  std::lock_guard<std::mutex> lock(g_mu);
  Streamer& st = g_st[dev];
  int status = setup(st);
  if (status != UP_OK) return status;

  cudaError_t e = cudaSuccess;
  auto ok = [&](cudaError_t r) {
    if (e == cudaSuccess) e = r;
    return e == cudaSuccess;
  };
  const int32_t* user_carry = nullptr;
  if (carry_in != nullptr) {
    const int32_t c = *carry_in;
    ok(cudaMemcpyAsync(st.carry, &c, sizeof(c), cudaMemcpyHostToDevice, st.comp));
    user_carry = st.carry;
  }
  const std::vector<Chunk> cs = plan_chunks(rows, k, reverse != 0);
  for (size_t i = 0; i < cs.size() && e == cudaSuccess; ++i) {
    const Chunk& c = cs[i];
    const int s = (int)(i % kSlots);
    int32_t* xs = st.xs + (size_t)s * kSlotElems;
    int32_t* ys = st.ys + (size_t)s * kSlotElems;
    const int64_t off = c.row0 * k + c.k0;  // the chunk is contiguous: whole rows, or a piece of one row
    const size_t bytes = sizeof(int32_t) * (size_t)(c.nrow * c.len);
    // copy in, once the scan that last read this slot is done
    if (i >= (size_t)kSlots) ok(cudaStreamWaitEvent(st.h2d, st.scan_done[s], 0));
    ok(cudaMemcpyAsync(xs, x + off, bytes, cudaMemcpyHostToDevice, st.h2d));
    ok(cudaEventRecord(st.h2d_done[s], st.h2d));
    // scan, once the input has landed and the slot's last output has been copied out
    ok(cudaStreamWaitEvent(st.comp, st.h2d_done[s], 0));
    if (i >= (size_t)kSlots) ok(cudaStreamWaitEvent(st.comp, st.d2h_done[s], 0));
    if (e != cudaSuccess) break;
    const int32_t* cin = c.carry_from_prev ? st.carry + 1 + (i & 1) : user_carry;
    status = up_sm100_scan_i32(xs, ys, c.nrow, c.len, op, exclusive, reverse, cin, st.ws, st.ws_bytes, st.comp);
    if (status != UP_OK) break;
    if (c.carry_to_next) {
      const int64_t edge = reverse ? 0 : c.len - 1;
      scan_chunk_carry_kernel<<<1, 1, 0, st.comp>>>(op, ys + edge, exclusive ? xs + edge : nullptr,
                                                    st.carry + 1 + ((i + 1) & 1));
      note_launch();
      ok(cudaGetLastError());
    }
    ok(cudaEventRecord(st.scan_done[s], st.comp));
    // copy out
    ok(cudaStreamWaitEvent(st.d2h, st.scan_done[s], 0));
    ok(cudaMemcpyAsync(y + off, ys, bytes, cudaMemcpyDeviceToHost, st.d2h));
    ok(cudaEventRecord(st.d2h_done[s], st.d2h));
  }
  // Drain every stream before returning, whatever happened, so no copy is left reading or writing the caller's
  // buffers.
  const cudaError_t e1 = cudaStreamSynchronize(st.h2d);
  const cudaError_t e2 = cudaStreamSynchronize(st.comp);
  const cudaError_t e3 = cudaStreamSynchronize(st.d2h);
  if (e == cudaSuccess) e = e1 != cudaSuccess ? e1 : e2 != cudaSuccess ? e2 : e3;
  if (e != cudaSuccess) return cuda_status(e);
  if (status != UP_OK) return status;
  return up_sm100_workspace_status(st.ws, st.comp);  // a bounded device wait that ran out, if any
}

UP_DEFINE_REVISION(host_scan)
