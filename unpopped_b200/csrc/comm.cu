// comm.cu — the multi-GPU side of libunpopped_sm100: communicators over the GPUs of one node, the exchange of the
// peer addresses the cross-GPU scan writes to, and up_sm100_launch_multi (one rank's shard of a lift, with the
// exchange step that lift has).
//
// The reference models a launch over several devices as the same kernel run per device on its slice of the launch
// (crates/unpopped/src/oracle/kernel_launch.rs:100-129, run_launch_devices; crates/unpopped/src/exec.rs:119-143,
// LaunchShape::devices). Here one process (or one host thread) drives each GPU; each call runs that rank's shard,
// and NCCL over NVLink carries only the exchanges the lifts have: the shard totals of a scan over contiguous
// shards, the output slices of the W4A16 GEMM. The block-cyclic scan needs no collective: its look-back reads
// stripe aggregates that the other ranks write into this rank's memory over NVLink (plain peer stores; no TMA,
// no multicast).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, preferring the copy the process already has, e.g. the one
// PyTorch loaded), so the library links no NCCL and loads without it; the communicator entry points return
// UP_ERR_COMM when it is missing.
#include "common.cuh"
#include "multi.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

namespace up {
namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
};

const NcclApi* nccl() {
  static NcclApi api{};
  static bool ok = false;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the NCCL this process already loaded
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) return;
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
    api.CommInitAll = reinterpret_cast<decltype(api.CommInitAll)>(dlsym(h, "ncclCommInitAll"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
    api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    ok = api.GetUniqueId && api.CommInitRank && api.CommInitAll && api.CommDestroy && api.AllGather &&
         api.AllReduce && api.GetErrorString;
  });
  return ok ? &api : nullptr;
}

int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return UP_OK;
  char buf[200];
  const NcclApi* api = nccl();
  std::snprintf(buf, sizeof(buf), "%s: %s", what, api ? api->GetErrorString(r) : "NCCL error");
  return fail_with(UP_ERR_COMM, buf);
}

// Sets a device current for the life of the object, and puts the previous one back.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (dev != prev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace up

using namespace up;

// A communicator: this rank's NCCL communicator and device, and the buffers of the exchanges.
struct up_comm {
  int nranks = 0, rank = 0, dev = 0;
  ncclComm_t nc = nullptr;
  bool single = false;                       // one process drives every rank (up_sm100_comm_init)
  std::vector<up_comm*>* group = nullptr;    // single process: every rank's communicator, by rank
  bool distinct = false;                     // every rank is on its own GPU
  uint64_t* sflags = nullptr;                // this rank's stripe words (block-cyclic scan)
  int64_t sflag_words = 0;
  uint64_t* peers[kMaxRanks] = {};           // every rank's stripe words, as this rank addresses them
  bool peer_ipc[kMaxRanks] = {};             // peers[i] was opened from a CUDA IPC handle
  uint64_t launches = 0;                     // block-cyclic launches (the same count on every rank)
  int32_t* scratch = nullptr;                // device: [0] this shard's total, [1 .. G] all totals, [G + 1] carry
};

namespace up {
namespace {

// Fold of the shard totals before this rank in scan order (after it, for a reverse scan) into *carry.
__global__ void shard_carry_kernel(const int32_t* totals, int G, int r, int op, int reverse, int32_t* carry) {
  int32_t acc = op == UP_OP_SUM ? 0 : (op == UP_OP_MAX ? INT32_MIN : INT32_MAX);
  const int lo = reverse ? r + 1 : 0, hi = reverse ? G : r;
  for (int q = lo; q < hi; ++q) {
    const int32_t v = totals[q];
    acc = op == UP_OP_SUM ? (int32_t)((uint32_t)acc + (uint32_t)v) : op == UP_OP_MAX ? (v > acc ? v : acc)
                                                                                     : (v < acc ? v : acc);
  }
  *carry = acc;
}

// The all-gathered [G][M][Nl] output slices into the [M][G * Nl] output.
__global__ void slices_to_rows_kernel(const uint16_t* __restrict__ parts, int G, int64_t M, int64_t Nl,
                                      uint16_t* __restrict__ out, int64_t out_stride) {
  const int64_t total = (int64_t)G * M * Nl;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = i / (M * Nl), rem = i - g * M * Nl, m = rem / Nl, j = rem - m * Nl;
    out[m * out_stride + g * Nl + j] = parts[i];
  }
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Every rank's PCI bus id through an all-gather; true when no two ranks share a GPU.
int ranks_on_distinct_gpus(up_comm* c, bool* distinct) {
  char mine[64] = {0};
  cudaError_t e = cudaDeviceGetPCIBusId(mine, sizeof(mine), c->dev);
  if (e != cudaSuccess) return cuda_status(e);
  char* d = nullptr;
  e = cudaMalloc(&d, (size_t)64 * (c->nranks + 1));
  if (e != cudaSuccess) return cuda_status(e);
  std::vector<char> all((size_t)64 * c->nranks);
  cudaStream_t s = nullptr;
  int st = UP_OK;
  e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMemcpyAsync(d, mine, 64, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) st = cuda_status(e);
  if (st == UP_OK) st = nccl_status(nccl()->AllGather(d, d + 64, 64, ncclUint8, c->nc, s), "all-gather of devices");
  if (st == UP_OK) {
    e = cudaMemcpyAsync(all.data(), d + 64, all.size(), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) st = cuda_status(e);
  }
  if (s) cudaStreamDestroy(s);
  cudaFree(d);
  if (st != UP_OK) return st;
  bool ok = true;
  for (int a = 0; a < c->nranks; ++a)
    for (int b = a + 1; b < c->nranks; ++b)
      if (std::strncmp(&all[(size_t)64 * a], &all[(size_t)64 * b], 64) == 0) ok = false;
  *distinct = ok;
  return UP_OK;
}

void release_stripes(up_comm* c) {
  DeviceGuard g(c->dev);
  for (int q = 0; q < kMaxRanks; ++q) {
    if (c->peer_ipc[q] && c->peers[q]) cudaIpcCloseMemHandle(c->peers[q]);
    c->peers[q] = nullptr;
    c->peer_ipc[q] = false;
  }
  if (c->sflags) cudaFree(c->sflags);
  c->sflags = nullptr;
  c->sflag_words = 0;
}

// Makes every rank's stripe words hold at least `words` (a collective: every rank calls it with the same count).
// Multi-process: each rank allocates its own words and the ranks all-gather their CUDA IPC handles; single
// process: the words of every rank's device are allocated here and addressed directly (peer access enabled).
int ensure_stripes(up_comm* c, int64_t words, cudaStream_t s) {
  if (c->single) {
    bool enough = true;
    for (up_comm* o : *c->group) enough = enough && o->sflag_words >= words;
    if (enough) return UP_OK;
    for (up_comm* o : *c->group) {
      DeviceGuard g(o->dev);
      cudaError_t e = cudaDeviceSynchronize();
      if (e != cudaSuccess) return cuda_status(e);
      release_stripes(o);
      e = cudaMalloc(&o->sflags, (size_t)words * 8);
      if (e == cudaSuccess) e = cudaMemset(o->sflags, 0, (size_t)words * 8);
      if (e == cudaSuccess) e = cudaDeviceSynchronize();
      if (e != cudaSuccess) return cuda_status(e);
      o->sflag_words = words;
    }
    for (up_comm* o : *c->group)
      for (int q = 0; q < o->nranks; ++q) o->peers[q] = (*c->group)[q]->sflags;
    return UP_OK;
  }
  if (c->sflag_words >= words) return UP_OK;
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e);
  release_stripes(c);
  e = cudaMalloc(&c->sflags, (size_t)words * 8);
  if (e == cudaSuccess) e = cudaMemset(c->sflags, 0, (size_t)words * 8);
  cudaIpcMemHandle_t h{};
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->sflags);
  char* d = nullptr;
  if (e == cudaSuccess) e = cudaMalloc(&d, sizeof(h) * (c->nranks + 1));
  if (e == cudaSuccess) e = cudaMemcpy(d, &h, sizeof(h), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (d) cudaFree(d);
    return cuda_status(e);
  }
  int st = nccl_status(nccl()->AllGather(d, d + sizeof(h), sizeof(h), ncclUint8, c->nc, s), "all-gather of handles");
  std::vector<cudaIpcMemHandle_t> hs(c->nranks);
  if (st == UP_OK) {
    e = cudaMemcpyAsync(hs.data(), d + sizeof(h), sizeof(h) * c->nranks, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) st = cuda_status(e);
  }
  cudaFree(d);
  if (st != UP_OK) return st;
  for (int q = 0; q < c->nranks; ++q) {
    if (q == c->rank) {
      c->peers[q] = c->sflags;
      continue;
    }
    void* p = nullptr;
    e = cudaIpcOpenMemHandle(&p, hs[q], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_status(e);
    c->peers[q] = static_cast<uint64_t*>(p);
    c->peer_ipc[q] = true;
  }
  c->sflag_words = words;
  return UP_OK;
}

// The launch tag of the next block-cyclic scan on `c`. When the 30-bit tag wraps (once in 2^30 launches), every
// rank clears its stripe words and the ranks meet before any of them launches again, so no stale word of the
// previous cycle is read as current.
int next_tag(up_comm* c, cudaStream_t s, uint32_t* tag) {
  const uint64_t before = c->launches >> 30;
  const uint64_t n = ++c->launches;
  *tag = (uint32_t)(n & 0x3fffffffu);
  if ((n >> 30) == before) return UP_OK;
  if (c->single) {
    for (up_comm* o : *c->group) {
      DeviceGuard g(o->dev);
      cudaError_t e = cudaDeviceSynchronize();
      if (e == cudaSuccess && o->sflags) e = cudaMemset(o->sflags, 0, (size_t)o->sflag_words * 8);
      if (e == cudaSuccess) e = cudaDeviceSynchronize();
      if (e != cudaSuccess) return cuda_status(e);
    }
    return UP_OK;
  }
  cudaError_t e = cudaMemsetAsync(c->sflags, 0, (size_t)c->sflag_words * 8, s);
  if (e != cudaSuccess) return cuda_status(e);
  return nccl_status(nccl()->AllReduce(c->scratch, c->scratch, 1, ncclInt32, ncclMax, c->nc, s), "wrap barrier");
}

int64_t numel(const up_tensor& t) {
  int64_t n = 1;
  for (int d = 0; d < t.rank; ++d) n *= t.shape[d];
  return n;
}

bool dense(const up_tensor& t) {
  int64_t s = 1;
  for (int d = t.rank - 1; d >= 0; --d) {
    if (t.shape[d] != 1 && t.stride[d] != s) return false;
    s *= t.shape[d];
  }
  return true;
}

const char* elem_at(const up_tensor& t, int bytes) { return static_cast<const char*>(t.ptr) + t.base * bytes; }

}  // namespace
}  // namespace up

extern "C" int up_sm100_comm_unique_id(unsigned char* id) {
  if (id == nullptr) return UP_ERR_INVALID;
  const NcclApi* api = nccl();
  if (api == nullptr) return fail_with(UP_ERR_COMM, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  const int st = nccl_status(api->GetUniqueId(&u), "ncclGetUniqueId");
  if (st != UP_OK) return st;
  std::memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
  return UP_OK;
}

extern "C" int up_sm100_comm_init_rank(int nranks, int rank, const unsigned char* id, up_comm** out) {
  if (out == nullptr || id == nullptr || nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
    return UP_ERR_INVALID;
  *out = nullptr;
  const NcclApi* api = nccl();
  if (api == nullptr) return fail_with(UP_ERR_COMM, "libnccl.so.2 could not be loaded");
  auto* c = new up_comm();
  c->nranks = nranks;
  c->rank = rank;
  cudaError_t e = cudaGetDevice(&c->dev);
  if (e != cudaSuccess) {
    delete c;
    return cuda_status(e);
  }
  ncclUniqueId u;
  std::memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
  int st = nccl_status(api->CommInitRank(&c->nc, nranks, u, rank), "ncclCommInitRank");
  if (st == UP_OK) {
    e = cudaMalloc(&c->scratch, 4096);
    if (e == cudaSuccess) e = cudaMemset(c->scratch, 0, 4096);
    st = cuda_status(e);
  }
  if (st == UP_OK) st = ranks_on_distinct_gpus(c, &c->distinct);
  if (st != UP_OK) {
    if (c->scratch) cudaFree(c->scratch);
    if (c->nc) api->CommDestroy(c->nc);
    delete c;
    return st;
  }
  *out = c;
  return UP_OK;
}

extern "C" int up_sm100_comm_init(int n_gpus, const int* devs, up_comm** comms) {
  if (comms == nullptr || devs == nullptr || n_gpus < 1 || n_gpus > kMaxRanks) return UP_ERR_INVALID;
  for (int i = 0; i < n_gpus; ++i) comms[i] = nullptr;
  const NcclApi* api = nccl();
  if (api == nullptr) return fail_with(UP_ERR_COMM, "libnccl.so.2 could not be loaded");
  std::vector<ncclComm_t> ncs(n_gpus, nullptr);
  int st = nccl_status(api->CommInitAll(ncs.data(), n_gpus, devs), "ncclCommInitAll");
  if (st != UP_OK) return st;
  bool distinct = true;
  for (int a = 0; a < n_gpus; ++a)
    for (int b = a + 1; b < n_gpus; ++b) distinct = distinct && devs[a] != devs[b];
  auto* group = new std::vector<up_comm*>(n_gpus, nullptr);
  for (int i = 0; i < n_gpus && st == UP_OK; ++i) {
    auto* c = new up_comm();
    c->nranks = n_gpus;
    c->rank = i;
    c->dev = devs[i];
    c->nc = ncs[i];
    c->single = true;
    c->group = group;
    c->distinct = distinct;
    (*group)[i] = c;
    DeviceGuard g(devs[i]);
    cudaError_t e = cudaMalloc(&c->scratch, 4096);
    if (e == cudaSuccess) e = cudaMemset(c->scratch, 0, 4096);
    for (int j = 0; j < n_gpus && e == cudaSuccess; ++j) {
      if (devs[j] == devs[i]) continue;
      const cudaError_t p = cudaDeviceEnablePeerAccess(devs[j], 0);
      if (p != cudaSuccess && p != cudaErrorPeerAccessAlreadyEnabled) e = p;
      cudaGetLastError();  // an already-enabled peer leaves its error code behind
    }
    st = cuda_status(e);
  }
  if (st != UP_OK) {
    for (int i = 0; i < n_gpus; ++i) {
      up_comm* c = (*group)[i];
      if (c == nullptr) {
        if (ncs[i]) api->CommDestroy(ncs[i]);
        continue;
      }
      DeviceGuard g(c->dev);
      if (c->scratch) cudaFree(c->scratch);
      api->CommDestroy(c->nc);
      delete c;
    }
    delete group;
    return st;
  }
  for (int i = 0; i < n_gpus; ++i) comms[i] = (*group)[i];
  return UP_OK;
}

extern "C" int up_sm100_comm_destroy(up_comm* c) {
  if (c == nullptr) return UP_ERR_INVALID;
  const NcclApi* api = nccl();
  release_stripes(c);
  {
    DeviceGuard g(c->dev);
    if (c->scratch) cudaFree(c->scratch);
  }
  int st = UP_OK;
  if (api && c->nc) st = nccl_status(api->CommDestroy(c->nc), "ncclCommDestroy");
  if (c->single && c->group) {
    (*c->group)[c->rank] = nullptr;
    bool empty = true;
    for (up_comm* o : *c->group) empty = empty && o == nullptr;
    if (empty) delete c->group;
  }
  delete c;
  return st;
}

extern "C" int up_sm100_comm_rank(const up_comm* c, int* rank, int* nranks) {
  if (c == nullptr || rank == nullptr || nranks == nullptr) return UP_ERR_INVALID;
  *rank = c->rank;
  *nranks = c->nranks;
  return UP_OK;
}

extern "C" void up_sm100_comm_set_test_launches(up_comm* c, uint64_t launches) {
  if (c != nullptr) c->launches = launches;
}

extern "C" int up_sm100_workspace_bytes_multi(int kernel_id, const up_tensor* ins, int n_in, const up_tensor* outs,
                                              int n_out, const int64_t* scalars, int n_scalars, const up_comm* comm,
                                              size_t* bytes) {
  if (bytes == nullptr || comm == nullptr) return UP_ERR_INVALID;
  *bytes = 0;
  if (kernel_id == UP_K_W4A16_GEMM) {
    if (!ins || n_in < 3 || !scalars || n_scalars < 1) return UP_ERR_INVALID;
    const int64_t m = ins[2].shape[0], nl = ins[0].shape[0];
    *bytes = align256(up_sm100_w4a16_workspace_bytes(m, nl, ins[0].shape[1], scalars[0])) +
             align256((size_t)m * nl * 2) + (size_t)comm->nranks * m * nl * 2;
    return UP_OK;
  }
  return up_sm100_workspace_bytes(kernel_id, ins, n_in, outs, n_out, scalars, n_scalars, bytes);
}

extern "C" int up_sm100_launch_multi(int kernel_id, const up_tensor* ins, int n_in, const up_tensor* outs, int n_out,
                                     const int64_t* scalars, int n_scalars, void* workspace, size_t workspace_bytes,
                                     void* stream, up_comm* comm) {
  if (comm == nullptr || ins == nullptr || outs == nullptr) return UP_ERR_INVALID;
  auto sc = [&](int i, int64_t dflt) { return (scalars && i < n_scalars) ? scalars[i] : dflt; };
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int G = comm->nranks, r = comm->rank;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != comm->dev)
    return fail_with(UP_ERR_INVALID, "launch_multi: the communicator's device must be current");
  switch (kernel_id) {
    case UP_K_SCAN_I32: {
      if (n_in < 1 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &y = outs[0];
      if (x.dtype != UP_EK_I32 || y.dtype != UP_EK_I32 || !dense(x) || !dense(y) || numel(x) != numel(y))
        return UP_ERR_UNSUPPORTED;
      const int64_t k = numel(x);
      const int op = (int)sc(0, UP_OP_SUM), excl = (int)sc(1, 0), rev = (int)sc(2, 0), layout = (int)sc(3, 0);
      if (op != UP_OP_SUM && op != UP_OP_MAX && op != UP_OP_MIN) return UP_ERR_UNSUPPORTED;
      const int32_t* xp = reinterpret_cast<const int32_t*>(elem_at(x, 4));
      int32_t* yp = (int32_t*)elem_at(y, 4);
      if (layout == 0) {
        // contiguous shards in rank order: fold the shard, all-gather the G totals, scan seeded with the carry
        int st = up_sm100_reduce_i32(xp, k, op, comm->scratch, stream);
        if (st != UP_OK) return st;
        st = nccl_status(nccl()->AllGather(comm->scratch, comm->scratch + 1, 1, ncclInt32, comm->nc, s),
                         "all-gather of shard totals");
        if (st != UP_OK) return st;
        shard_carry_kernel<<<1, 1, 0, s>>>(comm->scratch + 1, G, r, op, rev, comm->scratch + G + 1);
        note_launch();
        st = check_launch();
        if (st != UP_OK) return st;
        return up_sm100_scan_i32(xp, yp, 1, k, op, excl, rev, comm->scratch + G + 1, workspace, workspace_bytes,
                                 stream);
      }
      if (layout != 1)
        return fail_with(UP_ERR_UNSUPPORTED, "launch_multi scan: layout 0 (contiguous) or 1 (block-cyclic)");
      if (rev) return fail_with(UP_ERR_UNSUPPORTED, "block-cyclic scan: forward only");
      if (!comm->distinct)
        return fail_with(UP_ERR_UNSUPPORTED, "block-cyclic scan: every rank needs its own GPU (the ranks wait on "
                                             "one another inside the kernel)");
      int st = ensure_stripes(comm, block_cyclic_stripe_words(k, G), s);
      if (st != UP_OK) return st;
      MultiScan m{};
      m.sflags = comm->sflags;
      for (int q = 0; q < G; ++q) m.peers[q] = comm->peers[q];
      m.G = G;
      m.r = r;
      st = next_tag(comm, s, &m.tag);
      if (st != UP_OK) return st;
      return scan_i32_block_cyclic(xp, yp, k, op, excl, nullptr, workspace, workspace_bytes, m, s);
    }
    case UP_K_W4A16_GEMM: {
      // this rank's weight rows [Nl, K]; the output [M, G * Nl] is assembled from every rank's slice
      if (n_in < 3 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &w = ins[0], &sl = ins[1], &x = ins[2], &o = outs[0];
      if (w.dtype != UP_EK_I4 || sl.dtype != UP_EK_F16 || x.dtype != UP_EK_BF16 || o.dtype != UP_EK_BF16)
        return UP_ERR_UNSUPPORTED;
      if (w.rank != 2 || x.rank != 2 || o.rank != 2 || sl.rank != 2 || !dense(w) || !dense(sl) || !dense(x) ||
          !dense(o) || w.base % 2)
        return UP_ERR_UNSUPPORTED;
      const int64_t nl = w.shape[0], kk = w.shape[1], m = x.shape[0], group = sc(0, 128);
      if (group <= 0 || kk % group || sl.shape[0] != nl || sl.shape[1] != kk / group || x.shape[1] != kk ||
          o.shape[0] != m || o.shape[1] != nl * G)
        return UP_ERR_UNSUPPORTED;
      size_t need = 0;
      int st = up_sm100_workspace_bytes_multi(kernel_id, ins, n_in, outs, n_out, scalars, n_scalars, comm, &need);
      if (st != UP_OK) return st;
      if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 256)) return UP_ERR_INVALID;
      const size_t gemm_ws = align256(up_sm100_w4a16_workspace_bytes(m, nl, kk, group));
      char* base = static_cast<char*>(workspace);
      uint16_t* slice = reinterpret_cast<uint16_t*>(base + gemm_ws);
      uint16_t* parts = reinterpret_cast<uint16_t*>(base + gemm_ws + align256((size_t)m * nl * 2));
      st = up_sm100_w4a16_gemm(reinterpret_cast<const uint8_t*>(w.ptr) + w.base / 2,
                               reinterpret_cast<const uint16_t*>(elem_at(sl, 2)),
                               reinterpret_cast<const uint16_t*>(elem_at(x, 2)), m, nl, kk, group, slice, workspace,
                               gemm_ws, stream);
      if (st != UP_OK) return st;
      st = nccl_status(nccl()->AllGather(slice, parts, (size_t)m * nl, ncclBfloat16, comm->nc, s),
                       "all-gather of output slices");
      if (st != UP_OK) return st;
      const int64_t total = (int64_t)G * m * nl;
      int64_t blocks = (total + 255) / 256;
      if (blocks > (int64_t)sm_count() * 8) blocks = (int64_t)sm_count() * 8;
      if (blocks > 0) {
        slices_to_rows_kernel<<<(unsigned)blocks, 256, 0, s>>>(parts, G, m, nl, (uint16_t*)elem_at(o, 2), o.stride[0]);
        note_launch();
      }
      return check_launch();
    }
    case UP_K_ROW_SUM_F32:
    case UP_K_ROW_MAX_ARGMAX_BF16:
    case UP_K_GATHER_ROWS:
    case UP_K_DEQUANT_I4:
      // independent (output) rows: each rank runs its shard, no collective on the data path
      return up_sm100_launch(kernel_id, ins, n_in, outs, n_out, scalars, n_scalars, workspace, workspace_bytes, stream);
    default:
      return fail_with(UP_ERR_UNSUPPORTED, "launch_multi: a kernel this library does not shard");
  }
}

UP_DEFINE_REVISION(comm)
