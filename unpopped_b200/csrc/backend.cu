// backend.cu — host side of libunpopped_sm100: the Backend-seam answers (name, provider, supports_dtype,
// plan classification) and the generic descriptor-based launch, plus the library's shared host state.
//
// Mirrors the reference trait `unpopped::Backend` (crates/unpopped/src/backend.rs:668-835) for the plans
// this backend lowers, and its refusal rule "refuse rather than approximate" (backend.rs:700-707): every
// plan outside the table below is declined with a typed LowerError, never run some other way.
#include "common.cuh"

#include <cuda.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

namespace up {

static std::atomic<uint64_t> g_launches{0};
static std::atomic<uint64_t> g_wait_ns{1000000000ull};
static std::atomic<int> g_withhold{0};
static thread_local char g_last_error[256] = "";
static std::mutex g_sm_mu;
static int g_sm_count[64] = {0};

void note_launch(uint64_t k) { g_launches.fetch_add(k, std::memory_order_relaxed); }

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return UP_OK;
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return UP_ERR_CUDA;
}

int check_launch() { return cuda_status(cudaGetLastError()); }

int fail_with(int status, const char* text) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", text);
  return status;
}

uint64_t wait_limit_ns() { return g_wait_ns.load(std::memory_order_relaxed); }

int take_withhold_flag() { return g_withhold.exchange(0); }

uint64_t context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static std::once_flag once;
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  if (get_current == nullptr || get_id == nullptr) return 0;
  cudaFree(nullptr);  // makes the device's primary context current if no context is yet
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (get_current(&c) != CUDA_SUCCESS || c == nullptr || get_id(c, &id) != CUDA_SUCCESS) return 0;
  return (uint64_t)id;
}

cudaError_t ensure_smem_attr(const void* func, int bytes) {
  struct Entry {
    const void* func;
    uint64_t ctx;
    int bytes;
  };
  static std::mutex mu;
  static std::vector<Entry> done;
  const uint64_t ctx = context_id();
  std::lock_guard<std::mutex> lk(mu);
  if (ctx != 0)
    for (const Entry& en : done)
      if (en.func == func && en.ctx == ctx && en.bytes >= bytes) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess || ctx == 0) return e;
  for (Entry& en : done)
    if (en.func == func && en.ctx == ctx) {
      en.bytes = bytes;
      return e;
    }
  done.push_back({func, ctx, bytes});
  return e;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(g_sm_mu);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

static bool is_our_target(const char* t) {
  if (!t) return false;
  return !std::strcmp(t, "cuda:sm_100a") || !std::strcmp(t, "cuda:sm100a") || !std::strcmp(t, "cuda:sm100") ||
         !std::strcmp(t, "cuda:sm_100");
}

static size_t elem_bits(int ek) {
  switch (ek) {
    case UP_EK_F16: case UP_EK_BF16: case UP_EK_I16: case UP_EK_U16: return 16;
    case UP_EK_F32: case UP_EK_F32_STRICT: case UP_EK_I32: case UP_EK_U32: return 32;
    case UP_EK_F64: case UP_EK_I64: case UP_EK_U64: case UP_EK_COMPLEX64: return 64;
    case UP_EK_COMPLEX128: return 128;
    case UP_EK_I8: case UP_EK_U8: case UP_EK_BOOL: case UP_EK_FP8_E4M3FN: case UP_EK_FP8_E5M2:
    case UP_EK_F8_E8M0: case UP_EK_F8_E6M2: return 8;
    case UP_EK_I4: case UP_EK_U4: return 4;
    default: return 0;
  }
}

static const char* k_name(int id) {
  switch (id) {
    case UP_K_ROW_SUM_F32: return "up_sm100_row_sum_f32";
    case UP_K_ROW_MAX_ARGMAX_BF16: return "up_sm100_row_max_argmax_bf16";
    case UP_K_SCAN_I32: return "up_sm100_scan_i32";
    case UP_K_GATHER_ROWS: return "up_sm100_gather_rows";
    case UP_K_DEQUANT_I4: return "up_sm100_dequant_i4_bf16";
    case UP_K_W4A16_GEMM: return "up_sm100_w4a16_gemm";
    case UP_K_REDUCE2D_F32: return "up_sm100_reduce2d_f32";
    case UP_K_REDUCE2D_I32: return "up_sm100_reduce2d_i32";
    case UP_K_REDUCE_F32: return "up_sm100_reduce3d_f32";
    case UP_K_REDUCE_I32: return "up_sm100_reduce3d_i32";
    case UP_K_ROW_REDUCE_F32: return "up_sm100_row_reduce_f32";
    case UP_K_COL_SUM_SPLITK: return "up_sm100_col_sum_f32_splitk";
    case UP_K_WINDOW: return "up_sm100_window";
    case UP_K_IM2COL: return "up_sm100_im2col";
    case UP_K_SCATTER: return "up_sm100_scatter";
    case UP_K_BINCOUNT: return "up_sm100_bincount";
    default: return "";
  }
}

static int refuse(up_lowered* out, int err, const char* detail) {
  out->kernel_id = UP_K_NONE;
  out->lower_error = err;
  out->name[0] = '\0';
  std::snprintf(out->detail, sizeof(out->detail), "%s", detail);
  out->n_scalars = 0;
  return UP_ERR_UNSUPPORTED;
}

static int accept(up_lowered* out, int id, std::initializer_list<int64_t> scalars) {
  out->kernel_id = id;
  out->lower_error = UP_LOWER_OK;
  std::snprintf(out->name, sizeof(out->name), "%s", k_name(id));
  out->detail[0] = '\0';
  out->n_scalars = 0;
  for (int64_t v : scalars) out->scalars[out->n_scalars++] = v;
  return UP_OK;
}

// A rank-r operand is row-contiguous on its last axis and its rows stack without overlap.
static bool last_axis_contiguous(const up_tensor& t) { return t.rank >= 1 && t.stride[t.rank - 1] == 1; }

static bool dense_row_major(const up_tensor& t) {
  int64_t s = 1;
  for (int d = t.rank - 1; d >= 0; --d) {
    if (t.shape[d] != 1 && t.stride[d] != s) return false;
    s *= t.shape[d];
  }
  return true;
}

// Axes [a, b) of t as one axis: its element count and the stride of its innermost non-unit axis (1 when all are
// unit). False when they do not flatten (an axis's stride is not the next one's stride times its extent).
static bool flat_run(const up_tensor& t, int a, int b, int64_t* n, int64_t* st) {
  int64_t count = 1, expect = 0, inner = 1;
  bool any = false;
  for (int d = b - 1; d >= a; --d) {
    count *= t.shape[d];
    if (t.shape[d] == 1) continue;
    if (any && t.stride[d] != expect) return false;
    if (!any) inner = t.stride[d];
    any = true;
    expect = t.stride[d] * t.shape[d];
  }
  *n = count;
  *st = inner;
  return true;
}

// A reduction over one run of adjacent axes [i, j) of a rank-r input seen as [A, R, C]: A the kept leading axes
// (batch stride sA), R the reduced run (step sR), C the kept trailing axes (contiguous). kind: 1 when C == 1 (a
// last-axis reduction of A rows of R), 0 when A == 1 (the outer axis of [R, C]), 2 otherwise (the middle axis).
struct RedGeo {
  int kind;
  int64_t A, R, C, sA, sR;
};
static bool reduction_geometry(const up_tensor& in, uint32_t mask, RedGeo* g) {
  const int r = in.rank;
  if (r < 1 || r > 8) return false;
  if (mask == 0) mask = 1u << (r - 1);  // the legacy last-axis default (ir.rs:2094-2097)
  if (mask >> r) return false;
  int i = 0;
  while (!(mask >> i & 1u)) ++i;
  int j = i;
  while (j < r && (mask >> j & 1u)) ++j;
  if (mask >> j) return false;  // the reduced axes are not one run
  int64_t sC = 1;
  if (!flat_run(in, 0, i, &g->A, &g->sA) || !flat_run(in, i, j, &g->R, &g->sR) || !flat_run(in, j, r, &g->C, &sC))
    return false;
  if (g->C > 1 && sC != 1) return false;  // the kept trailing axes are contiguous
  if (g->C == 1) {
    if (g->R > 1 && g->sR != 1) return false;  // a last-axis reduction reads contiguous rows
    if (g->A <= 1) g->sA = g->R;
    g->kind = 1;
  } else {
    if (g->R <= 1) g->sR = g->C;
    if (g->A <= 1) g->sA = g->R * g->sR;
    g->kind = g->A == 1 ? 0 : 2;
  }
  return g->sA >= 0 && g->sR >= 0;
}

static int64_t numel(const up_tensor& t) {
  int64_t n = 1;
  for (int d = 0; d < t.rank; ++d) n *= t.shape[d];
  return n;
}

}  // namespace up

using namespace up;

extern "C" int up_sm100_version(void) { return UP_SM100_ABI_VERSION; }
extern "C" const char* up_sm100_name(void) { return "cuda_sm100"; }
extern "C" const char* up_sm100_provider(void) { return "unpopped-cuda-sm100"; }
extern "C" uint64_t up_sm100_launch_count(void) { return g_launches.load(); }
extern "C" const char* up_sm100_last_error(void) { return g_last_error; }
extern "C" void up_sm100_set_wait_limit_ns(uint64_t ns) { g_wait_ns.store(ns ? ns : 1); }
extern "C" void up_sm100_set_test_withhold_flag(int enable) { g_withhold.store(enable ? 1 : 0); }

extern "C" int up_sm100_supports_dtype(int dtype, const char* target) {
  if (!is_our_target(target)) return 1;  // Unsupported: not this backend's target
  if (dtype < 0 || dtype >= UP_EK_COUNT) return 1;
  // Reserved tokens (no computation semantics at this schema version, element.rs:1112-1135): decline.
  if (dtype == UP_EK_FP8_E4M3FNUZ || dtype == UP_EK_FP8_E5M2FNUZ) return 1;
  // Every dtype a kernel of this backend takes in some role: f32 (sum), bf16 (max/argmax, W4A16, dequant
  // output), f16 (group scales), i32/i64/u32 (scans, indices, argmax), i4 (packed weights), and every
  // fixed-width storage type of at least one byte, which the row gather moves bit for bit.
  if (dtype == UP_EK_I4) return 0;
  if (dtype == UP_EK_U4 || dtype == UP_EK_B1) return 1;
  if (dtype == UP_EK_F4_E2M1 || dtype == UP_EK_F6_E2M3 || dtype == UP_EK_F6_E3M2) return 1;
  return elem_bits(dtype) >= 8 ? 0 : 1;
}

extern "C" int up_sm100_classify(const up_plan_desc* p, up_lowered* out) {
  if (!p || !out) return UP_ERR_INVALID;
  std::memset(out, 0, sizeof(*out));
  if (!is_our_target(p->target)) return refuse(out, UP_LOWER_UNSUPPORTED_SCHEDULE, "target is not cuda:sm_100a");
  if (p->n_operands < 0 || p->n_operands > 8) return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "operand count");
  const up_tensor* ops = p->operands;
  switch (p->schedule) {
    case UP_SCHED_REDUCTION: {
      if (p->n_operands < 2) return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "a reduction has an input and an output");
      const up_tensor& in = ops[0];
      const bool last_axis = p->axes_mask == 0 || (in.rank >= 1 && p->axes_mask == (1u << (in.rank - 1)));
      const bool outer_axis = in.rank == 2 && p->axes_mask == 1u;  // axis 0 of a rank-2 input
      if (!p->identity_body) return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "body/post must be the identity");
      // rank 2 keeps the rank-2 kernels; any other rank, or a middle or multi-axis set, is flattened to [A, R, C]
      const bool general = !(in.rank == 2 && (last_axis || outer_axis));
      RedGeo geo{};
      if (general && !reduction_geometry(in, p->axes_mask, &geo))
        return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE,
                      "the reduced axes are one run of adjacent axes, and the kept and reduced runs each flatten");
      if (!general && !last_axis_contiguous(in))
        return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "rows must be contiguous");
      const int axis = general ? (geo.kind == 1 ? 1 : 0) : (last_axis ? 1 : 0);
      if (p->op == UP_OP_MAX || p->op == UP_OP_ARGMAX) {
        if (p->dtype == UP_EK_BF16 && axis == 1) {
          if (p->op == UP_OP_ARGMAX && p->out_dtype != UP_EK_I64 && p->out_dtype != UP_EK_I32)
            return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "ArgMax needs an I64 (or I32) output");
          if (p->op == UP_OP_MAX && p->out_dtype != UP_EK_F32)
            return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "Max is stored as f32");
          return accept(out, UP_K_ROW_MAX_ARGMAX_BF16, {});
        }
        if (p->op == UP_OP_ARGMAX)
          return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "ArgMax is lowered for bf16 over the last axis");
      }
      if (p->dtype == UP_EK_F32) {
        if (p->op != UP_OP_SUM && p->op != UP_OP_MEAN && p->op != UP_OP_MAX && p->op != UP_OP_MIN)
          return refuse(out, UP_LOWER_UNSUPPORTED_OP, "f32 reductions lowered: Sum, Mean, Max, Min");
        const bool summing = p->op == UP_OP_SUM || p->op == UP_OP_MEAN;
        if (summing && p->accum != UP_ACCUM_AUTO && !(p->accum == UP_ACCUM_F32 && p->op == UP_OP_SUM && axis == 1))
          return refuse(out, UP_LOWER_UNSUPPORTED_OP, "accumulation policy");
        const int b = p->block ? p->block : (axis == 1 ? 256 : 1);
        if (b < 1 || b > 1024 || (b & (b - 1))) return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "block B");
        if (summing && axis == 0 && b > 256)
          return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "an outer-axis Sum/Mean takes a block of at most 256");
        if (p->splitk_chunks > 0) {  // the runtime selector chose the split-K variant
          if (general || axis != 0 || !summing)
            return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "split-K is a variant of the outer-axis Sum/Mean");
          return accept(out, UP_K_COL_SUM_SPLITK, {p->op == UP_OP_MEAN ? 1 : 0, p->splitk_chunks});
        }
        if (general) return accept(out, UP_K_REDUCE_F32, {p->op, p->axes_mask, p->accum, b});
        if (p->op == UP_OP_SUM && axis == 1) return accept(out, UP_K_ROW_SUM_F32, {p->accum, b});
        return accept(out, UP_K_REDUCE2D_F32, {p->op, axis, p->accum, b});
      }
      if (p->dtype == UP_EK_I32) {
        if (p->op != UP_OP_SUM && p->op != UP_OP_PROD && p->op != UP_OP_MAX && p->op != UP_OP_MIN &&
            p->op != UP_OP_AND && p->op != UP_OP_OR && p->op != UP_OP_XOR)
          return refuse(out, UP_LOWER_UNSUPPORTED_OP, "i32 reductions lowered: Sum, Prod, Max, Min, And, Or, Xor");
        if (general) return accept(out, UP_K_REDUCE_I32, {p->op, p->axes_mask});
        return accept(out, UP_K_REDUCE2D_I32, {p->op, axis});
      }
      return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "reductions are lowered for f32, i32 and (Max/ArgMax) bf16");
    }
    case UP_SCHED_ROW_REDUCE: {
      // Access::RowReduce: the lowered forms over f32 rows (kernel_lift/row_reduce_launched.rs:47-84)
      if (p->n_operands < 2) return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "a row reduction has an input and an output");
      if (p->dtype != UP_EK_F32) return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "row reductions are lowered for f32");
      if (p->row_reduce_form < UP_RR_SOFTMAX || p->row_reduce_form > UP_RR_CENTRED)
        return refuse(out, UP_LOWER_UNSUPPORTED_OP, "the stages and epilogue are softmax, RMS norm or the centred quotient");
      const up_tensor& in = ops[0];
      int64_t rows = 0, rstride = 0;
      if (in.rank < 2 || !last_axis_contiguous(in) || !flat_run(in, 0, in.rank - 1, &rows, &rstride))
        return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "a launched row reduction strides blocks over a leading axis");
      const int b = p->block ? p->block : 256;
      if (b < 1 || b > 1024 || (b & (b - 1))) return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "block B");
      int64_t eps_bits = 0;
      std::memcpy(&eps_bits, &p->eps, sizeof(eps_bits));
      return accept(out, UP_K_ROW_REDUCE_F32, {p->row_reduce_form, b, eps_bits});
    }
    case UP_SCHED_WINDOW: {
      // Access::Window (ir.rs:2206-2259): 1-D pooling along one axis of a dense input, identity pre/post
      if (p->n_operands < 2) return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "a window has an input and an output");
      if (p->dtype != UP_EK_F32 && p->dtype != UP_EK_I32)
        return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "windows are lowered for f32 and i32");
      if (p->op != UP_OP_SUM && p->op != UP_OP_MEAN && p->op != UP_OP_MAX && p->op != UP_OP_MIN)
        return refuse(out, UP_LOWER_UNSUPPORTED_OP, "window ops: Sum, Mean, Max, Min");
      if (p->dtype == UP_EK_I32 && p->op == UP_OP_MEAN)
        return refuse(out, UP_LOWER_UNSUPPORTED_OP, "an integer window Mean is not defined");
      if (!p->identity_body) return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "pre/post must be the identity");
      const up_tensor &in = ops[0], &o = ops[1];
      if (p->window_axis < 0 || p->window_axis >= in.rank || o.rank != in.rank || !dense_row_major(in) ||
          !dense_row_major(o))
        return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "a dense input and output, the axis in range");
      if (p->window_size < 1 || p->window_stride < 1 || p->window_dilation < 1 || p->window_pad_lo < 0)
        return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "size, stride, dilation >= 1");
      return accept(out, UP_K_WINDOW, {p->op, p->window_size, p->window_stride, p->window_dilation, p->window_pad_lo,
                                       p->count_include_pad, p->window_axis});
    }
    case UP_SCHED_IM2COL: {
      if (p->n_operands < 2) return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "im2col has an input and an output");
      const up_tensor &in = ops[0], &o = ops[1];
      const int bits = elem_bits(in.dtype);
      if (bits < 8 || (bits != 8 && bits != 16 && bits != 32 && bits != 64))
        return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "im2col moves elements of 1, 2, 4 or 8 bytes");
      if (in.rank != 4 || o.rank != 3 || !dense_row_major(in) || !dense_row_major(o) || o.dtype != in.dtype)
        return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "a dense NCHW input into a dense [N, C*kh*kw, oH*oW]");
      return accept(out, UP_K_IM2COL, {p->im2col_kernel[0], p->im2col_kernel[1], p->im2col_stride[0],
                                       p->im2col_stride[1], p->im2col_pad[0], p->im2col_pad[1],
                                       p->im2col_dilation[0], p->im2col_dilation[1]});
    }
    case UP_SCHED_SCAN: {
      if (p->n_operands < 2) return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "a scan has an input and an output");
      if (p->dtype != UP_EK_I32) return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "scans are lowered for i32");
      if (p->op != UP_OP_SUM && p->op != UP_OP_MAX && p->op != UP_OP_MIN)
        return refuse(out, UP_LOWER_UNSUPPORTED_OP, "scan op");
      if (p->scan_axis != ops[0].rank - 1) return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "only the last axis is scanned");
      if (!dense_row_major(ops[0]) || !dense_row_major(ops[1]))
        return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "scan operands must be dense row-major");
      return accept(out, UP_K_SCAN_I32, {p->op, p->exclusive ? 1 : 0, p->reverse ? 1 : 0});
    }
    case UP_SCHED_STRIDED: {
      if (p->has_write_index) {
        // scatter / index_add / bincount: operands (updates, ids, out) or, for bincount, (x, counts)
        if (p->scatter_axis != 0) return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "scatter along axis 0 only");
        if (p->index_dtype != UP_EK_I32 && p->index_dtype != UP_EK_I64 && p->index_dtype != UP_EK_U32)
          return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "index dtype");
        if (p->combine == UP_COMBINE_ASSIGN)
          return refuse(out, UP_LOWER_UNSUPPORTED_OP, "a launched Assign: repeated targets order the stores");
        if (p->count) {
          if (p->n_operands < 2 || ops[1].dtype != UP_EK_I32 || p->combine != UP_COMBINE_ADD)
            return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "bincount adds into I32 counts");
          return accept(out, UP_K_BINCOUNT, {});
        }
        if (p->n_operands < 3) return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "updates, ids and output");
        const up_tensor &u = ops[0], &ix = ops[1], &o = ops[2];
        if (u.rank != 2 || o.rank != 2 || u.stride[1] != 1 || o.stride[1] != 1 || u.shape[1] != o.shape[1])
          return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "rank-2 updates and destination with contiguous rows");
        const bool full = ix.rank == 2 && ix.stride[1] == 1 && ix.shape[0] == u.shape[0] && ix.shape[1] == u.shape[1];
        const bool row = (ix.rank == 1 && ix.shape[0] == u.shape[0]) ||
                         (ix.rank == 2 && ix.stride[1] == 0 && ix.shape[0] == u.shape[0]);
        if (!full && !row) return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "a full-shape or a 1-D row index");
        const int dt = p->dtype;
        const bool integer = dt == UP_EK_I32 || dt == UP_EK_U32 || dt == UP_EK_I64;
        const bool fp = dt == UP_EK_F32 || dt == UP_EK_F64;
        if (!integer && !fp) return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "scatter dtypes: I32, U32, I64, F32, F64");
        if (fp && p->combine != UP_COMBINE_ADD)
          return refuse(out, UP_LOWER_UNSUPPORTED_OP, "float Max/Min scatter: integers only");
        return accept(out, UP_K_SCATTER, {p->combine, full ? 1 : 0});
      }
      if (!p->has_read_index) return refuse(out, UP_LOWER_UNSUPPORTED_SCHEDULE, "only the gather form of Strided");
      if (p->gather_axis != 0) return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "gather along axis 0 only");
      if (p->index_dtype != UP_EK_I32 && p->index_dtype != UP_EK_I64 && p->index_dtype != UP_EK_U32)
        return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "index dtype");
      if (p->n_operands < 3) return refuse(out, UP_LOWER_INADMISSIBLE_PLAN, "table, ids and output");
      if (!dense_row_major(ops[0]) || !dense_row_major(ops[2]))
        return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "table and output must be dense row-major");
      for (int d = 1; d < ops[1].rank; ++d)
        if (ops[1].stride[d] != 0 && ops[1].shape[d] != 1)
          return refuse(out, UP_LOWER_UNSUPPORTED_PLAN_SHAPE, "ids must be 1-D, broadcast over the row");
      if (elem_bits(ops[0].dtype) < 8) return refuse(out, UP_LOWER_UNSUPPORTED_DTYPE, "sub-byte table");
      return accept(out, UP_K_GATHER_ROWS, {p->oob});
    }
    case UP_SCHED_KERNEL_FN: {
      if (p->n_operands == 3 && ops[0].dtype == UP_EK_I4 && ops[1].dtype == UP_EK_F16 && ops[2].dtype == UP_EK_BF16) {
        const int64_t group = ops[1].shape[1] > 0 ? ops[0].shape[1] / ops[1].shape[1] : 0;
        return accept(out, UP_K_DEQUANT_I4, {group});
      }
      if (p->n_operands == 4 && ops[0].dtype == UP_EK_I4 && ops[1].dtype == UP_EK_F16 && ops[2].dtype == UP_EK_BF16 &&
          ops[3].dtype == UP_EK_BF16) {
        const int64_t group = ops[1].shape[1] > 0 ? ops[0].shape[1] / ops[1].shape[1] : 0;
        return accept(out, UP_K_W4A16_GEMM, {group});
      }
      return refuse(out, UP_LOWER_UNSUPPORTED_KERNEL, "kernel-layer function is not the dequant/W4A16 form");
    }
    default:
      return refuse(out, UP_LOWER_UNSUPPORTED_SCHEDULE, "schedule not lowered by this backend");
  }
}

static const char* at(const up_tensor& t) {
  const size_t bits = elem_bits(t.dtype);
  return static_cast<const char*>(t.ptr) + (int64_t)((t.base * (int64_t)bits) / 8);
}

// An output of `n` elements written contiguously: its elements must be exactly those, densely laid out.
static bool dense_vector(const up_tensor& t, int64_t n) {
  int64_t c = 1;
  for (int d = 0; d < t.rank; ++d) c *= t.shape[d];
  return c == n && (n <= 1 || dense_row_major(t));
}

static bool same_shape(const up_tensor& a, const up_tensor& b) {
  if (a.rank != b.rank) return false;
  for (int d = 0; d < a.rank; ++d)
    if (a.shape[d] != b.shape[d]) return false;
  return true;
}

extern "C" int up_sm100_workspace_bytes(int kernel_id, const up_tensor* ins, int n_in, const up_tensor* outs, int n_out,
                                        const int64_t* scalars, int n_scalars, size_t* bytes) {
  (void)outs; (void)n_out;
  if (!bytes) return UP_ERR_INVALID;
  *bytes = 0;
  if (kernel_id == UP_K_SCAN_I32) {
    if (!ins || n_in < 1 || ins[0].rank < 1) return UP_ERR_INVALID;
    int64_t rows = 1;
    for (int d = 0; d < ins[0].rank - 1; ++d) rows *= ins[0].shape[d];
    *bytes = up_sm100_scan_workspace_bytes(rows, ins[0].shape[ins[0].rank - 1]);
  } else if (kernel_id == UP_K_COL_SUM_SPLITK) {
    if (!ins || n_in < 1 || ins[0].rank != 2 || !scalars || n_scalars < 2) return UP_ERR_INVALID;
    *bytes = up_sm100_col_sum_splitk_workspace_bytes(ins[0].shape[0], ins[0].shape[1], scalars[1]);
  } else if (kernel_id == UP_K_W4A16_GEMM) {
    if (!ins || n_in < 3 || !scalars || n_scalars < 1) return UP_ERR_INVALID;
    *bytes = up_sm100_w4a16_workspace_bytes(ins[2].shape[0], ins[0].shape[0], ins[0].shape[1], scalars[0]);
  }
  return UP_OK;
}

extern "C" int up_sm100_launch(int kernel_id, const up_tensor* ins, int n_in, const up_tensor* outs, int n_out,
                               const int64_t* scalars, int n_scalars, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (!ins || !outs) return UP_ERR_INVALID;
  auto sc = [&](int i, int64_t dflt) { return (scalars && i < n_scalars) ? scalars[i] : dflt; };
  switch (kernel_id) {
    case UP_K_ROW_SUM_F32: {
      if (n_in < 1 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &y = outs[0];
      if (x.dtype != UP_EK_F32 || y.dtype != UP_EK_F32 || x.rank != 2 || x.stride[1] != 1) return UP_ERR_UNSUPPORTED;
      if (!dense_vector(y, x.shape[0])) return UP_ERR_UNSUPPORTED;
      return up_sm100_row_sum_f32(reinterpret_cast<const float*>(at(x)), x.shape[0], x.shape[1], x.stride[0],
                                  (float*)at(y), (int)sc(0, UP_ACCUM_F32), (int)sc(1, 256), stream);
    }
    case UP_K_REDUCE2D_F32:
    case UP_K_REDUCE2D_I32: {
      if (n_in < 1 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &y = outs[0];
      const int axis = (int)sc(1, 1);
      const bool f32 = kernel_id == UP_K_REDUCE2D_F32;
      if (x.dtype != (f32 ? UP_EK_F32 : UP_EK_I32) || y.dtype != x.dtype || x.rank != 2 || x.stride[1] != 1)
        return UP_ERR_UNSUPPORTED;
      if (axis != 0 && axis != 1) return UP_ERR_INVALID;
      const int64_t n_out_elems = axis == 1 ? x.shape[0] : x.shape[1];
      if (!dense_vector(y, n_out_elems)) return UP_ERR_UNSUPPORTED;
      if (f32)
        return up_sm100_reduce2d_f32(reinterpret_cast<const float*>(at(x)), x.shape[0], x.shape[1], x.stride[0], axis,
                                     (int)sc(0, UP_OP_SUM), (int)sc(2, UP_ACCUM_AUTO), (int)sc(3, 256), (float*)at(y),
                                     stream);
      return up_sm100_reduce2d_i32(reinterpret_cast<const int32_t*>(at(x)), x.shape[0], x.shape[1], x.stride[0], axis,
                                   (int)sc(0, UP_OP_SUM), (int32_t*)at(y), stream);
    }
    case UP_K_REDUCE_F32:
    case UP_K_REDUCE_I32: {
      if (n_in < 1 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &y = outs[0];
      const bool f32 = kernel_id == UP_K_REDUCE_F32;
      if (x.dtype != (f32 ? UP_EK_F32 : UP_EK_I32) || y.dtype != x.dtype) return UP_ERR_UNSUPPORTED;
      RedGeo g{};
      if (!reduction_geometry(x, (uint32_t)sc(1, 0), &g)) return UP_ERR_UNSUPPORTED;
      if (!dense_row_major(y) || numel(y) != g.A * g.C) return UP_ERR_UNSUPPORTED;  // out [A, C], dense
      const int op = (int)sc(0, UP_OP_SUM);
      if (g.kind == 1) {  // A rows of R
        if (f32 && op == UP_OP_SUM)
          return up_sm100_row_sum_f32(reinterpret_cast<const float*>(at(x)), g.A, g.R, g.sA, (float*)at(y),
                                      (int)sc(2, UP_ACCUM_AUTO), (int)sc(3, 256), stream);
        if (f32)
          return up_sm100_reduce2d_f32(reinterpret_cast<const float*>(at(x)), g.A, g.R, g.sA, 1, op,
                                       (int)sc(2, UP_ACCUM_AUTO), (int)sc(3, 256), (float*)at(y), stream);
        return up_sm100_reduce2d_i32(reinterpret_cast<const int32_t*>(at(x)), g.A, g.R, g.sA, 1, op, (int32_t*)at(y),
                                     stream);
      }
      if (f32)
        return up_sm100_reduce3d_f32(reinterpret_cast<const float*>(at(x)), g.A, g.R, g.C, g.sA, g.sR, op,
                                     (int)sc(2, UP_ACCUM_AUTO), (int)sc(3, 1), (float*)at(y), g.C, stream);
      return up_sm100_reduce3d_i32(reinterpret_cast<const int32_t*>(at(x)), g.A, g.R, g.C, g.sA, g.sR, op,
                                   (int32_t*)at(y), g.C, stream);
    }
    case UP_K_WINDOW: {
      if (n_in < 1 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &y = outs[0];
      const int axis = (int)sc(6, 0);
      if (axis < 0 || axis >= x.rank || y.rank != x.rank || !dense_row_major(x) || !dense_row_major(y) ||
          y.dtype != x.dtype)
        return UP_ERR_UNSUPPORTED;
      int64_t outer = 1, inner = 1;
      for (int d = 0; d < axis; ++d) {
        if (y.shape[d] != x.shape[d]) return UP_ERR_UNSUPPORTED;
        outer *= x.shape[d];
      }
      for (int d = axis + 1; d < x.rank; ++d) {
        if (y.shape[d] != x.shape[d]) return UP_ERR_UNSUPPORTED;
        inner *= x.shape[d];
      }
      return up_sm100_window(at(x), x.dtype, outer, x.shape[axis], inner, (int)sc(0, UP_OP_SUM), (int)sc(1, 1),
                             (int)sc(2, 1), (int)sc(3, 1), (int)sc(4, 0), (int)sc(5, 0), (void*)at(y), y.shape[axis],
                             stream);
    }
    case UP_K_IM2COL: {
      if (n_in < 1 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &y = outs[0];
      if (x.rank != 4 || y.rank != 3 || !dense_row_major(x) || !dense_row_major(y)) return UP_ERR_UNSUPPORTED;
      const int kh = (int)sc(0, 1), kw = (int)sc(1, 1), sh = (int)sc(2, 1), sw = (int)sc(3, 1);
      const int ph = (int)sc(4, 0), pw = (int)sc(5, 0), dh = (int)sc(6, 1), dw = (int)sc(7, 1);
      if (kh < 1 || kw < 1 || sh < 1 || sw < 1 || dh < 1 || dw < 1) return UP_ERR_UNSUPPORTED;
      const int64_t oh = (x.shape[2] + 2 * (int64_t)ph - (int64_t)dh * (kh - 1) - 1) / sh + 1;
      const int64_t ow = (x.shape[3] + 2 * (int64_t)pw - (int64_t)dw * (kw - 1) - 1) / sw + 1;
      if (y.shape[0] != x.shape[0] || y.shape[1] != x.shape[1] * kh * kw || y.shape[2] != oh * ow)
        return UP_ERR_UNSUPPORTED;
      return up_sm100_im2col(at(x), elem_bits(x.dtype) / 8, x.shape[0], x.shape[1], x.shape[2], x.shape[3], kh, kw, sh,
                             sw, ph, pw, dh, dw, (void*)at(y), stream);
    }
    case UP_K_COL_SUM_SPLITK: {
      if (n_in < 1 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &y = outs[0];
      if (x.dtype != UP_EK_F32 || y.dtype != UP_EK_F32 || x.rank != 2 || x.stride[1] != 1) return UP_ERR_UNSUPPORTED;
      if (!dense_row_major(y) || numel(y) != x.shape[1]) return UP_ERR_UNSUPPORTED;
      return up_sm100_col_sum_f32_splitk(reinterpret_cast<const float*>(at(x)), x.shape[0], x.shape[1], x.stride[0],
                                         sc(1, 1), (int)sc(0, 0), workspace, workspace_bytes, (float*)at(y), stream);
    }
    case UP_K_ROW_REDUCE_F32: {
      if (n_in < 1 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &y = outs[0];
      if (x.dtype != UP_EK_F32 || y.dtype != UP_EK_F32 || x.rank < 2 || y.rank != x.rank) return UP_ERR_UNSUPPORTED;
      int64_t rows = 0, xs = 0, yrows = 0, ys = 0;
      if (!last_axis_contiguous(x) || !last_axis_contiguous(y) || !flat_run(x, 0, x.rank - 1, &rows, &xs) ||
          !flat_run(y, 0, y.rank - 1, &yrows, &ys))
        return UP_ERR_UNSUPPORTED;
      const int64_t cols = x.shape[x.rank - 1];
      if (yrows != rows || y.shape[y.rank - 1] != cols) return UP_ERR_UNSUPPORTED;
      if (rows <= 1) xs = ys = cols;  // one row: its stride is never used
      double eps = 0.0;
      const int64_t eps_bits = sc(2, 0);
      std::memcpy(&eps, &eps_bits, sizeof(eps));
      return up_sm100_row_reduce_f32(reinterpret_cast<const float*>(at(x)), rows, cols, xs, (int)sc(0, 0),
                                     (int)sc(1, 256), eps, (float*)at(y), ys, stream);
    }
    case UP_K_ROW_MAX_ARGMAX_BF16: {
      if (n_in < 1 || n_out < 2) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &mx = outs[0], &am = outs[1];
      if (x.dtype != UP_EK_BF16 || x.rank != 2 || x.stride[1] != 1) return UP_ERR_UNSUPPORTED;
      if (mx.ptr && (mx.dtype != UP_EK_F32 || !dense_vector(mx, x.shape[0]))) return UP_ERR_UNSUPPORTED;
      if (am.ptr && ((am.dtype != UP_EK_I32 && am.dtype != UP_EK_I64) || !dense_vector(am, x.shape[0])))
        return UP_ERR_UNSUPPORTED;
      return up_sm100_row_max_argmax_bf16(reinterpret_cast<const uint16_t*>(at(x)), x.shape[0], x.shape[1], x.stride[0],
                                          mx.ptr ? (float*)at(mx) : nullptr,
                                          (am.ptr && am.dtype == UP_EK_I32) ? (int32_t*)at(am) : nullptr,
                                          (am.ptr && am.dtype == UP_EK_I64) ? (int64_t*)at(am) : nullptr, stream);
    }
    case UP_K_SCATTER: {
      if (n_in < 2 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &u = ins[0], &ix = ins[1], &o = outs[0];
      if (u.rank != 2 || o.rank != 2 || u.dtype != o.dtype) return UP_ERR_UNSUPPORTED;
      const int64_t ids_stride = sc(1, 0) ? ix.stride[0] : 0;
      const int64_t ids_elem_stride = (ix.rank >= 1 && !sc(1, 0)) ? ix.stride[0] : 1;
      if (!sc(1, 0) && ids_elem_stride != 1) return UP_ERR_UNSUPPORTED;  // a 1-D index must be contiguous
      return up_sm100_scatter(at(u), u.shape[0], u.shape[1], u.stride[0], u.dtype, at(ix), ix.dtype, ids_stride,
                              (int)sc(0, UP_COMBINE_ADD), (void*)at(o), o.shape[0], o.stride[0], stream);
    }
    case UP_K_BINCOUNT: {
      if (n_in < 1 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &c = outs[0];
      int64_t nx = 1;
      for (int d = 0; d < x.rank; ++d) nx *= x.shape[d];
      if (c.dtype != UP_EK_I32 || (x.rank > 1 && !dense_row_major(x))) return UP_ERR_UNSUPPORTED;
      return up_sm100_bincount(at(x), nx, x.dtype, (int32_t*)at(c), c.rank >= 1 ? c.shape[0] : 1, stream);
    }
    case UP_K_SCAN_I32: {
      if (n_in < 1 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &x = ins[0], &y = outs[0];
      if (x.dtype != UP_EK_I32 || y.dtype != UP_EK_I32 || x.rank < 1) return UP_ERR_UNSUPPORTED;
      if (!dense_row_major(x) || !dense_row_major(y) || !same_shape(x, y)) return UP_ERR_UNSUPPORTED;
      int64_t rows = 1;
      for (int d = 0; d < x.rank - 1; ++d) rows *= x.shape[d];
      return up_sm100_scan_i32(reinterpret_cast<const int32_t*>(at(x)), (int32_t*)at(y), rows, x.shape[x.rank - 1],
                               (int)sc(0, UP_OP_SUM), (int)sc(1, 0), (int)sc(2, 0), nullptr, workspace,
                               workspace_bytes, stream);
    }
    case UP_K_GATHER_ROWS: {
      if (n_in < 2 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &tab = ins[0], &ids = ins[1], &o = outs[0];
      if (tab.rank < 1 || tab.dtype != o.dtype || !dense_row_major(tab) || !dense_row_major(o) || o.rank != tab.rank)
        return UP_ERR_UNSUPPORTED;
      int64_t row_elems = 1;
      for (int d = 1; d < tab.rank; ++d) {
        if (o.shape[d] != tab.shape[d]) return UP_ERR_UNSUPPORTED;
        row_elems *= tab.shape[d];
      }
      const int64_t row_bytes = row_elems * (int64_t)elem_bits(tab.dtype) / 8;
      const int64_t n = o.shape[0];
      if (ids.rank < 1 || ids.shape[0] != n || ids.stride[0] != 1) return UP_ERR_UNSUPPORTED;
      return up_sm100_gather_rows(at(tab), tab.shape[0], row_bytes, at(ids), ids.dtype, n, (int)sc(0, UP_OOB_SKIP),
                                  (void*)at(o), stream);
    }
    case UP_K_DEQUANT_I4: {
      if (n_in < 2 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &w = ins[0], &s = ins[1], &o = outs[0];
      if (w.dtype != UP_EK_I4 || s.dtype != UP_EK_F16 || o.dtype != UP_EK_BF16) return UP_ERR_UNSUPPORTED;
      if (!dense_row_major(w) || !dense_row_major(s) || !dense_row_major(o) || w.base % 2) return UP_ERR_UNSUPPORTED;
      const int64_t group = sc(0, 128);
      if (w.rank != 2 || s.rank != 2 || !same_shape(w, o) || group <= 0 || w.shape[1] % group ||
          s.shape[0] != w.shape[0] || s.shape[1] != w.shape[1] / group)
        return UP_ERR_UNSUPPORTED;
      return up_sm100_dequant_i4_bf16(reinterpret_cast<const uint8_t*>(at(w)), reinterpret_cast<const uint16_t*>(at(s)),
                                      w.shape[0], w.shape[1], sc(0, 128), (uint16_t*)at(o), stream);
    }
    case UP_K_W4A16_GEMM: {
      if (n_in < 3 || n_out < 1) return UP_ERR_INVALID;
      const up_tensor &w = ins[0], &s = ins[1], &x = ins[2], &o = outs[0];
      if (w.dtype != UP_EK_I4 || s.dtype != UP_EK_F16 || x.dtype != UP_EK_BF16 || o.dtype != UP_EK_BF16)
        return UP_ERR_UNSUPPORTED;
      if (!dense_row_major(w) || !dense_row_major(s) || !dense_row_major(x) || !dense_row_major(o) || w.base % 2)
        return UP_ERR_UNSUPPORTED;
      const int64_t group = sc(0, 128);
      if (w.rank != 2 || s.rank != 2 || x.rank != 2 || o.rank != 2 || group <= 0 || w.shape[1] % group ||
          s.shape[0] != w.shape[0] || s.shape[1] != w.shape[1] / group || x.shape[1] != w.shape[1] ||
          o.shape[0] != x.shape[0] || o.shape[1] != w.shape[0])
        return UP_ERR_UNSUPPORTED;
      return up_sm100_w4a16_gemm(reinterpret_cast<const uint8_t*>(at(w)), reinterpret_cast<const uint16_t*>(at(s)),
                                 reinterpret_cast<const uint16_t*>(at(x)), x.shape[0], w.shape[0], w.shape[1], sc(0, 128),
                                 (uint16_t*)at(o), workspace, workspace_bytes, stream);
    }
    default:
      return UP_ERR_UNSUPPORTED;
  }
}

UP_DEFINE_REVISION(backend)
