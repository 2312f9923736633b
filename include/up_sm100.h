/*
 * up_sm100.h — C ABI of libunpopped_sm100.so, the sm_100a (B200) execution backend for Unpopped's lifted
 * kernel families: row reductions (sum, max, argmax), inclusive/exclusive scans, row gather, int4
 * group-wise dequant and the W4A16 GEMM.
 *
 * The reference (Unpopped, Rust) has no execution step of its own: its `Backend` trait
 * (crates/unpopped/src/backend.rs:668-835) lowers a `KernelPlan` to kernel source and its oracle
 * (crates/unpopped/src/oracle/plan_eval.rs) evaluates plans on the CPU. This library is what a Rust
 * `unpopped-cuda-sm100` crate binds through `extern "C"`: the dtype answer of `Backend::supports_dtype`
 * (backend.rs:779), the plan classification behind `Backend::lower` (backend.rs:708) and the launch of
 * the kernel the plan lowered to, on caller-owned device buffers.
 *
 * Conventions
 *  - Every entry point returns an `up_status` (an int). 0 is success. Values 1 and 2 follow the C ABI the
 *    reference's C99 emitter gives its kernels (crates/unpopped-cpu-c/src/kernel.rs:7-18: 1 = out of
 *    bounds, 2 = zero step); the rest extend it. No entry point aborts or traps on caller input.
 *  - Pointers are device pointers unless a parameter says "host". Launches are stream-ordered on the
 *    `stream` argument (a cudaStream_t; NULL is the legacy default stream) and return once enqueued.
 *  - Device-side waits (scan look-back, split-K fix-up) are bounded. A wait that runs out sets an error
 *    word in the caller's workspace; `up_sm100_workspace_status` reports it as UP_ERR_DEVICE_TIMEOUT.
 *  - Elements are addressed as `ptr + base + sum(coord[d] * stride[d])`, in elements, as in the
 *    reference's `TypedBuffer` (crates/unpopped/src/oracle/buffers.rs:16) and the C99 emitter's buffer
 *    arguments (crates/unpopped-cpu-c/src/base.rs:81-86).
 */
#ifndef UP_SM100_H
#define UP_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UP_SM100_ABI_VERSION 1

/* Exported from libunpopped_sm100.so (built with hidden visibility for everything else). */
#if defined(__GNUC__)
#define UP_API __attribute__((visibility("default")))
#else
#define UP_API
#endif
#define UP_MAX_RANK 8

/* Status codes. */
typedef enum up_status {
  UP_OK = 0,
  UP_ERR_OOB = 1,              /* an extent or offset leaves its buffer (cpu-c ABI value 1) */
  UP_ERR_ZERO_STEP = 2,        /* a zero loop step (cpu-c ABI value 2) */
  UP_ERR_UNSUPPORTED = 3,      /* the backend declines this dtype / shape / op (LowerError) */
  UP_ERR_DEVICE_TIMEOUT = 4,   /* a bounded device-side wait ran out */
  UP_ERR_CUDA = 5,             /* a CUDA runtime/driver call failed */
  UP_ERR_COMM = 6,             /* a collective failed */
  UP_ERR_INVALID = 7           /* a null pointer, a negative extent or a too-small workspace */
} up_status;

/* ElementKind, by ordinal in the reference enum (crates/unpopped-vocab/src/element.rs:1052-1206). */
typedef enum up_element_kind {
  UP_EK_F16 = 0, UP_EK_BF16 = 1, UP_EK_F32 = 2, UP_EK_F32_STRICT = 3, UP_EK_F64 = 4,
  UP_EK_I8 = 5, UP_EK_I16 = 6, UP_EK_U8 = 7, UP_EK_U16 = 8, UP_EK_I32 = 9, UP_EK_I64 = 10,
  UP_EK_BOOL = 11, UP_EK_FP8_E4M3FN = 12, UP_EK_FP8_E4M3FNUZ = 13, UP_EK_FP8_E5M2 = 14,
  UP_EK_F8_E8M0 = 15, UP_EK_F8_E6M2 = 16, UP_EK_FP8_E5M2FNUZ = 17, UP_EK_I4 = 18, UP_EK_U4 = 19,
  UP_EK_B1 = 20, UP_EK_COMPLEX64 = 21, UP_EK_COMPLEX128 = 22, UP_EK_U32 = 23, UP_EK_U64 = 24,
  UP_EK_F4_E2M1 = 25, UP_EK_F6_E2M3 = 26, UP_EK_F6_E3M2 = 27,
  UP_EK_COUNT = 28
} up_element_kind;

/* ReduceOp, by ordinal in the reference enum (crates/unpopped/src/ir.rs:1700-1742). */
typedef enum up_reduce_op {
  UP_OP_SUM = 0, UP_OP_MEAN = 1, UP_OP_MAX = 2, UP_OP_MIN = 3, UP_OP_PROD = 4, UP_OP_AND = 5,
  UP_OP_OR = 6, UP_OP_XOR = 7, UP_OP_MAXNUM = 8, UP_OP_MINNUM = 9, UP_OP_ARGMAX = 10, UP_OP_ARGMIN = 11
} up_reduce_op;

/* OobPolicy (crates/unpopped/src/ir.rs:2582-2599): what an out-of-range gather index writes. The load
 * address is always clamped in range; the policy only decides the store. */
typedef enum up_oob_policy { UP_OOB_SKIP = 0, UP_OOB_CLAMP = 1, UP_OOB_ZERO_FILL = 2 } up_oob_policy;

/* Accumulation policy of a float Sum (crates/unpopped/src/ir.rs:2447-2476, docs/accum-policies.md).
 *  UP_ACCUM_AUTO: f64 accumulator in the launched lift's documented order (logical thread t of a block of
 *                 B folds t, t+B, t+2B, ... ascending; then acc[t] += acc[t+s] for s = B/2 .. 1; one
 *                 rounding at the store) — crates/unpopped/src/kernel_lift/block_reduce.rs:13-23.
 *                 Bit-exact and reproducible for a given B.
 *  UP_ACCUM_F32:  f32 accumulator in this library's fixed order (deterministic; error <= 2^-20 sum|x|). */
typedef enum up_accum { UP_ACCUM_AUTO = 0, UP_ACCUM_F32 = 1 } up_accum;

/* Schedule kind of a plan (crates/unpopped/src/plan/types.rs:14-150), plus the kernel-layer entry
 * (`Backend::lower_kernel`, backend.rs:726-745) for the dequant GEMM. */
typedef enum up_schedule {
  UP_SCHED_VECTORIZED = 0, UP_SCHED_SCALAR = 1, UP_SCHED_STRIDED = 2, UP_SCHED_REDUCTION = 3,
  UP_SCHED_ROW_REDUCE = 4, UP_SCHED_CONTRACTION = 5, UP_SCHED_SCAN = 6, UP_SCHED_WINDOW = 7, UP_SCHED_IM2COL = 8,
  UP_SCHED_KERNEL_FN = 100
} up_schedule;

/* Kernel ids: what `up_sm100_classify` maps a plan to and `up_sm100_launch` runs. */
/* `WriteCombine` (crates/unpopped/src/ir.rs:2723-2732), in declaration order. */
typedef enum up_write_combine {
  UP_COMBINE_ASSIGN = 0, UP_COMBINE_ADD = 1, UP_COMBINE_MAX = 2, UP_COMBINE_MIN = 3
} up_write_combine;

typedef enum up_kernel_id {
  UP_K_NONE = -1,
  UP_K_ROW_SUM_F32 = 1,
  UP_K_ROW_MAX_ARGMAX_BF16 = 2,
  UP_K_SCAN_I32 = 3,
  UP_K_GATHER_ROWS = 4,
  UP_K_DEQUANT_I4 = 5,
  UP_K_W4A16_GEMM = 6,
  UP_K_REDUCE2D_F32 = 7,  /* f32 Sum/Mean/Max/Min over the last or the outer axis of a rank-2 input */
  UP_K_REDUCE2D_I32 = 8,  /* i32 Sum/Prod/Max/Min/And/Or/Xor, same axes */
  UP_K_SCATTER = 9,       /* scatter / index_add with an atomic combine over axis 0 */
  UP_K_BINCOUNT = 10,
  UP_K_REDUCE_F32 = 11,   /* f32 Sum/Mean/Max/Min over one run of adjacent axes of a rank-r input (any class) */
  UP_K_REDUCE_I32 = 12,   /* i32, the seven ops, same geometry */
  UP_K_ROW_REDUCE_F32 = 13, /* a RowReduce form (softmax, RMS norm, centred quotient) over f32 rows */
  UP_K_COL_SUM_SPLITK = 14,  /* the split-K variant of the outer-axis f32 Sum/Mean (needs a workspace) */
  UP_K_WINDOW = 15,          /* 1-D window pooling (Sum/Mean/Max/Min) along one axis, f32 or i32 */
  UP_K_IM2COL = 16           /* the 2-D unfold of an NCHW input, raw bits */
} up_kernel_id;

/* A buffer argument: the reference's TypedBuffer / OperandDesc. `base` and `stride` count elements
 * (for I4/U4: nibbles; packing is two per byte, low nibble = even index, tests/sub_byte_packing.rs:24-40). */
typedef struct up_tensor {
  void* ptr;
  int32_t dtype; /* up_element_kind */
  int32_t rank;
  int64_t shape[UP_MAX_RANK];
  int64_t stride[UP_MAX_RANK];
  int64_t base;
} up_tensor;

/* The parts of a reference `KernelPlan` (plan/types.rs:170-270) the classifier reads. */
typedef struct up_plan_desc {
  int32_t schedule;      /* up_schedule */
  int32_t op;            /* up_reduce_op: the Reduction / Scan op */
  int32_t dtype;         /* plan.dtype, the compute dtype */
  int32_t out_dtype;     /* plan.out_dtype (ArgMax requires I64; I32 is this library's extension) */
  uint32_t axes_mask;    /* Reduction axes; 0 = the legacy last-axis default (ir.rs:2094-2097) */
  int32_t keepdim;
  int32_t identity_body; /* 1 when the body is Input(0) and the post is Reduced(0) */
  int32_t accum;         /* up_accum for a float Sum */
  int32_t block;         /* the launched lift's block size B for UP_ACCUM_AUTO (0 = 256) */
  int32_t scan_axis;     /* Scan: the scanned axis */
  int32_t exclusive;     /* Scan */
  int32_t reverse;       /* Scan */
  int32_t has_read_index;/* Strided with a data-dependent read (a gather) */
  int32_t gather_axis;   /* ReadIndex::Indexed{axis} (ir.rs:2620-2669) */
  int32_t oob;           /* up_oob_policy */
  int32_t index_dtype;   /* up_element_kind of the index operand */
  int32_t n_operands;    /* inputs then outputs, at most 8 */
  up_tensor operands[8]; /* shapes/strides/dtypes only; ptr may be NULL */
  char target[32];       /* TargetId token, e.g. "cuda:sm_100a" or "cuda:sm100a" */
  /* appended: the data-dependent WRITE role (WriteIndex::ScatterIndexed, ir.rs:2787-2850) */
  int32_t has_write_index; /* Strided with a scatter store */
  int32_t scatter_axis;    /* the scattered axis of the destination */
  int32_t combine;         /* up_write_combine */
  int32_t count;           /* bincount: the input is its own index and the increment is the constant 1 */
  /* appended: a RowReduce plan (Access::RowReduce, ir.rs; its stages and epilogue matched to a named form) */
  int32_t row_reduce_form; /* up_row_reduce_form; 0 = not one of the lowered forms */
  double eps;              /* the RMS norm's constant under the square root */
  /* appended: the runtime selector's choice of the split-K variant (ondevice/README.md:185-218) */
  int64_t splitk_chunks;   /* > 0: an outer-axis f32 Sum/Mean runs as split-K over this many row chunks */
  /* appended: Schedule::Window (plan/types.rs; ir.rs:2206-2259) */
  int32_t window_axis, window_size, window_stride, window_dilation, window_pad_lo, window_pad_hi;
  int32_t count_include_pad;
  /* appended: Schedule::Im2Col (ir.rs:2286-2324): (h, w) pairs */
  int32_t im2col_kernel[2], im2col_stride[2], im2col_pad[2], im2col_dilation[2];
} up_plan_desc;

/* What `Backend::lower` returns (`GeneratedKernel{name, source}` + launch metadata), or why it refused
 * (`LowerError`, backend.rs:386-440). */
typedef enum up_lower_error {
  UP_LOWER_OK = 0, UP_LOWER_UNSUPPORTED_DTYPE = 1, UP_LOWER_UNSUPPORTED_SCHEDULE = 2,
  UP_LOWER_UNSUPPORTED_OP = 3, UP_LOWER_UNSUPPORTED_PLAN_SHAPE = 4, UP_LOWER_INADMISSIBLE_PLAN = 5,
  UP_LOWER_UNSUPPORTED_KERNEL = 6
} up_lower_error;

typedef struct up_lowered {
  int32_t kernel_id;     /* up_kernel_id */
  int32_t lower_error;   /* up_lower_error */
  char name[64];         /* entry symbol, e.g. "up_sm100_scan_i32" */
  char detail[160];      /* the refusal's detail text */
  int64_t scalars[8];    /* launch scalars `up_sm100_launch` expects for this kernel */
  int32_t n_scalars;
} up_lowered;

/* ---- Backend seam ------------------------------------------------------------------------------- */

/* UP_SM100_ABI_VERSION of the loaded library. */
UP_API int up_sm100_version(void);

/* `Backend::name` / `Backend::provider` (backend.rs:668-690): "cuda_sm100" / "unpopped-cuda-sm100". */
UP_API const char* up_sm100_name(void);
UP_API const char* up_sm100_provider(void);

/* `Backend::supports_dtype(dtype, target)` (backend.rs:779): 0 Supported, 1 Unsupported,
 * 2 NotExpressible (DtypeSupport, backend.rs:645-666). Targets "cuda:sm_100a" and "cuda:sm100a" (and
 * "cuda:sm100") are this backend's; any other target answers Unsupported. */
UP_API int up_sm100_supports_dtype(int dtype, const char* target);

/* `Backend::lower` (backend.rs:708) restricted to what this backend maps: fills `out` with the kernel id,
 * entry symbol and launch scalars, or with the LowerError that refuses the plan. Returns UP_OK when a
 * kernel was chosen, UP_ERR_UNSUPPORTED when the plan is refused, UP_ERR_INVALID on a null argument. */
UP_API int up_sm100_classify(const up_plan_desc* plan, up_lowered* out);

/* ---- Generic launch ------------------------------------------------------------------------------ */

/* Workspace bytes `up_sm100_launch(id, ...)` needs (0 when none). The workspace must be zero-filled
 * once before its first use (`cudaMemset`); every launch that completes without an error leaves it ready
 * for the next launch of any shape (the kernels re-arm their counters and clear their partial sums). After
 * UP_ERR_DEVICE_TIMEOUT, zero-fill it again. Launches that overlap on the GPU need separate workspaces. */
UP_API int up_sm100_workspace_bytes(int kernel_id, const up_tensor* ins, int n_in, const up_tensor* outs,
                             int n_out, const int64_t* scalars, int n_scalars, size_t* bytes);

/* Launch kernel `kernel_id` on tensor descriptors. Operand order and scalars per kernel:
 *  ROW_SUM_F32:          ins {x f32 [rows, cols]}, outs {sum f32 [rows]};
 *                        scalars {accum (up_accum), block B (AUTO only; power of two, 1..1024)}
 *  ROW_MAX_ARGMAX_BF16:  ins {x bf16 [rows, cols]}, outs {max f32 [rows] | ptr NULL,
 *                        argmax i32 or i64 [rows] | ptr NULL}
 *  SCAN_I32:             ins {x i32 [rows, k]}, outs {y i32 [rows, k]};
 *                        scalars {op (SUM|MAX|MIN), exclusive, reverse}
 *  GATHER_ROWS:          ins {table [V, D] (any dtype), ids i32/i64/u32 [N]}, outs {out [N, D]};
 *                        scalars {oob (up_oob_policy)}
 *  DEQUANT_I4:           ins {w i4 [N, K], scale f16 [N, K/group]}, outs {out bf16 [N, K]};
 *                        scalars {group}
 *  W4A16_GEMM:           ins {w i4 [N, K], scale f16 [N, K/group], x bf16 [M, K]},
 *                        outs {out bf16 [M, N]}; scalars {group}
 */
UP_API int up_sm100_launch(int kernel_id, const up_tensor* ins, int n_in, const up_tensor* outs, int n_out,
                    const int64_t* scalars, int n_scalars, void* workspace, size_t workspace_bytes,
                    void* stream);

/* Waits for `stream`, then reads and clears the device error word of a workspace: UP_OK, or
 * UP_ERR_DEVICE_TIMEOUT when a bounded wait ran out during an earlier launch on it. */
UP_API int up_sm100_workspace_status(void* workspace, void* stream);

/* ---- Typed entry points (what the generic launch dispatches to) ------------------------------------ */

/* Row sum of a row-major f32 matrix (`ReduceOp::Sum` over the last axis, `Access::Reduction`,
 * ir.rs:2080-2135; oracle fold oracle/plan_eval.rs:501-651). `row_stride` in elements (>= cols). */
UP_API int up_sm100_row_sum_f32(const float* x, int64_t rows, int64_t cols, int64_t row_stride, float* out,
                         int accum, int block, void* stream);

/* The reduction lift's other ops on a row-major rank-2 [rows, cols] input reduced over one axis: axis 1 (the
 * last; `out` has `rows` entries) or axis 0 (the outer; `out` has `cols`). `ReduceOp` (ir.rs:1700-1748) and
 * `Access::Reduction` with an axes mask (ir.rs:2080-2135), evaluated as the oracle does (oracle/plan_eval.rs:
 * 501-651, plan_contract.rs:146-245).
 * f32: op SUM, MEAN, MAX or MIN. Over the last axis Sum/Mean follow `accum` (Mean: Auto only) and the launched
 * lift's documented order for logical block `block` (kernel_lift/block_reduce.rs:13-23); over the outer axis
 * Sum/Mean follow the same documented order down each column for a block of up to 256 (block 1: the serial
 * order; Auto only). Max/Min are NaN-propagating and bit-exact to the
 * serial fold: the last NaN (quiet bit set) if any, else the first element of the extreme value.
 * i32: op SUM or PROD (both wrapping), MAX, MIN, AND, OR or XOR; bit-exact. An empty fold stores 0 (1 for Prod;
 * an f32 Mean: 0/0). */
UP_API int up_sm100_reduce2d_f32(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int axis, int op,
                                 int accum, int block, float* out, void* stream);
UP_API int up_sm100_reduce2d_i32(const int32_t* x, int64_t rows, int64_t cols, int64_t row_stride, int axis,
                                 int op, int32_t* out, void* stream);

/* RowReduce forms, by the stages and epilogue of `Access::RowReduce` (crates/unpopped/src/ir.rs) they stand for:
 * the forms of crates/unpopped/tests/kernel_parallel_row_reduce_agrees.rs:99-131. */
typedef enum up_row_reduce_form {
  UP_RR_NONE = 0,
  UP_RR_SOFTMAX = 1,   /* stages Max(x), Sum(exp(x - r0)); epilogue exp(x - r0) / r1 */
  UP_RR_RMS_NORM = 2,  /* stage Mean(x * x); epilogue x / sqrt(r0 + eps) */
  UP_RR_CENTRED = 3    /* stages Mean(x), Max(x - r0); epilogue (x - r0) / r1 */
} up_row_reduce_form;

/* The launched RowReduce lift (`lift_row_reduce_opdef_launched`, kernel_lift/row_reduce_launched.rs:47-84) over
 * the rows of a [rows, cols] f32 input (contiguous rows) into out (row stride out_stride), for logical block
 * `block` (a power of two up to 1024). Expressions are evaluated in f64; Sum/Mean stages fold in the documented
 * order of `block` (kernel_lift/block_reduce.rs:13-23); Max stages are NaN-keeping; each stage value is rounded
 * once to f32 and the epilogue once on the store (row_reduce_launched.rs:1-24). The reference holds its softmax
 * and RMS norm to a few ulps of its serial lift (kernel_parallel_row_reduce_agrees.rs:371-392). */
UP_API int up_sm100_row_reduce_f32(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int form,
                                   int block, double eps, float* out, int64_t out_stride, void* stream);

/* The split-K variant of the outer-axis f32 Sum/Mean (crates/unpopped/ondevice/README.md:185-218; the harness
 * splitk_validate.cu:40-50): chunk c of chunk_rows = ceil(rows / n_chunks) rows is folded ascending into an f64
 * partial from a 0.0 seed (in the workspace), then the partials are added in chunk order seeded from the first;
 * Mean divides by rows; one rounding. Deterministic for a fixed n_chunks (the reference's ReassociatedDeterministic
 * fidelity); n_chunks = 1 is the serial fold of up_sm100_reduce2d_f32 (axis 0, block 1) bit for bit. n_chunks is
 * clamped to [1, rows]. `workspace` from up_sm100_col_sum_splitk_workspace_bytes, 8-byte aligned. */
UP_API int up_sm100_col_sum_f32_splitk(const float* x, int64_t rows, int64_t cols, int64_t row_stride,
                                       int64_t n_chunks, int mean, void* workspace, size_t workspace_bytes,
                                       float* out, void* stream);
UP_API size_t up_sm100_col_sum_splitk_workspace_bytes(int64_t rows, int64_t cols, int64_t n_chunks);

/* The Window lift (Access::Window, ir.rs:2206-2259) as 1-D pooling along one axis of a dense [outer, k_in, inner]
 * input into [outer, k_out, inner]: output o folds the taps o·stride − pad_lo + kk·dilation (kk ascending) that
 * fall inside [0, k_in), as the oracle does (oracle/plan_window.rs:249-475). f32: Sum/Mean in f64 with one rounding
 * (Mean divides by `size` when count_include_pad, else by the valid taps), Max/Min from the first tap, strictly
 * better replacing, the last NaN kept (quiet bit set). i32: Sum wrapping, Max, Min. A window with no in-bounds tap
 * is refused (UP_ERR_UNSUPPORTED), as the reference's plan declines it. */
UP_API int up_sm100_window(const void* x, int dtype, int64_t outer, int64_t k_in, int64_t inner, int op, int size,
                           int stride, int dilation, int pad_lo, int count_include_pad, void* out, int64_t k_out,
                           void* stream);

/* The Im2Col lift (Access::Im2Col, ir.rs:2286-2324; oracle/plan_window.rs:483-535): a dense NCHW input of
 * elem_bytes-sized elements (1, 2, 4 or 8) into [N, C·kh·kw, oH·oW], oH = (H + 2ph − dh(kh − 1) − 1)/sh + 1 (and the
 * same for W). Cell (n, c·kh·kw + ki·kw + kj, oh·oW + ow) is a raw-bit copy of input (n, c, oh·sh − ph + ki·dh,
 * ow·sw − pw + kj·dw), or zero bytes outside the input. */
UP_API int up_sm100_im2col(const void* x, int elem_bytes, int64_t n, int64_t c, int64_t h, int64_t w, int kh, int kw,
                           int sh, int sw, int ph, int pw, int dh, int dw, void* out, void* stream);

/* Interface artifacts. The `KernelInterface` (crates/unpopped/src/kernel_interface.rs:196-230) of a kernel id as
 * JSON: the entry symbol, the parameters (role, element kind, rank) in the generic launch's operand order and then
 * its scalars, the launch geometry and dynamic shared memory, launch bounds, the cooperative flag, the capabilities
 * the code requires, fidelity notes, the workspace it needs, and its revision hash. A NULL `buf` reports the length
 * (without the terminating NUL) in `len`; UP_ERR_INVALID when `cap` is too small. */
UP_API int up_sm100_kernel_interface(int kernel_id, char* buf, size_t cap, size_t* len);
/* A kernel's source revision: FNV-1a 64 over its source file (`GeneratedKernel::revision_hash`, backend.rs:173-175,
 * revision.rs), the third field of its link-registry row (link.rs:27-42). 0 for an unknown id. */
UP_API uint64_t up_sm100_revision_hash(int kernel_id);

/* The same ops over the middle axis of [outer, rows, cols] (rows contiguous; batch b at x + b·outer_stride) into
 * out[outer][cols] (row stride out_stride): `ReduceAxisClass::Middle` (plan/types.rs:150-165), and every reduced
 * set that flattens to one run of adjacent axes, which the oracle folds in row-major order over the reduced
 * coordinates (oracle/plan_eval.rs:565-605), the order the flattened axis has. Each output cell is the outer-axis
 * fold of up_sm100_reduce2d_* over its batch, with the same orders, bounds and refusals. */
UP_API int up_sm100_reduce3d_f32(const float* x, int64_t outer, int64_t rows, int64_t cols, int64_t outer_stride,
                                 int64_t row_stride, int op, int accum, int block, float* out, int64_t out_stride,
                                 void* stream);
UP_API int up_sm100_reduce3d_i32(const int32_t* x, int64_t outer, int64_t rows, int64_t cols, int64_t outer_stride,
                                 int64_t row_stride, int op, int32_t* out, int64_t out_stride, void* stream);

/* The launched Scatter lift (`WriteIndex::ScatterIndexed`, ir.rs:2787-2850; the oracle's scatter store,
 * oracle/plan_eval.rs:430-490) over axis 0 of a row-major destination [out_rows, cols]: for every element (i, j) of
 * `updates` [n, cols], the target row t is ids[i * ids_stride + j] (`ids_stride` = the index's row stride: a
 * full-shape index, torch `scatter_add`) or ids[i] (`ids_stride` 0: `index_add`), and
 * out[t][j] = combine(out[t][j], updates[i][j]); targets outside [0, out_rows) are skipped. `combine`: ADD, MAX or
 * MIN (ASSIGN is declined, as the reference's launched lift declines it). `dtype`: I32, U32, I64 (every combine;
 * bit-exact, integer add wraps) or F32, F64 (ADD only; within the reassociation band gamma_(n-1) * sum|terms|).
 * `index_dtype`: I32, I64 or U32. Strides in elements. */
UP_API int up_sm100_scatter(const void* updates, int64_t n, int64_t cols, int64_t upd_stride, int dtype,
                            const void* ids, int index_dtype, int64_t ids_stride, int combine, void* out,
                            int64_t out_rows, int64_t out_stride, void* stream);

/* bincount (`OpDef::bincount`; crates/unpopped/tests/kernel_bincount_agrees.rs:1-10): counts[x[i]] += 1 for every
 * in-range x[i] (0 <= x[i] < bins); `counts` (I32) keeps its prior contents. `index_dtype`: I32, I64 or U32. */
UP_API int up_sm100_bincount(const void* x, int64_t n, int index_dtype, int32_t* counts, int64_t bins, void* stream);

/* Row max and argmax of a row-major bf16 matrix: Max is NaN-propagating (oracle/plan_contract.rs:179-210),
 * ArgMax is the first index of the extreme with NaN the greatest value (plan_contract.rs:213-245).
 * Either output may be NULL; `argmax_i64` and `argmax_i32` may both be given. */
UP_API int up_sm100_row_max_argmax_bf16(const uint16_t* x, int64_t rows, int64_t cols, int64_t row_stride,
                                 float* max_out, int32_t* argmax_i32, int64_t* argmax_i64, void* stream);

/* Scan of `rows` independent rows of `k` int32 (`Access::Scan`, ir.rs:2153-2195; oracle
 * oracle/plan_window.rs:10-238): op SUM (wrapping), MAX or MIN; `exclusive` writes the prefix before
 * the element (the first is the identity: 0, INT32_MIN, INT32_MAX); `reverse` runs from the row's end.
 * `carry_in` (device pointer to one int32, or NULL) is combined in front of every row — the carry of a
 * scan sharded over several GPUs. Single-pass decoupled look-back; `workspace` from
 * up_sm100_scan_workspace_bytes, zero-filled before its first use (the launches keep it usable: look-back flags
 * are tagged per launch, and the first launch on a workspace after the 30-bit tag wraps, once in 2^30 launches,
 * clears the flags with a stream-ordered memset first). Shapes beyond 2^31 - 2 tiles return UP_ERR_UNSUPPORTED
 * (up_sm100_scan_workspace_bytes then answers SIZE_MAX). Rows that are 16-byte aligned and whole 16-byte chunks
 * long run as one persistent CTA per SM, which needs every CTA resident at once: a kernel running concurrently
 * on other streams can keep one off the device, and the scan then returns UP_ERR_DEVICE_TIMEOUT (through
 * up_sm100_workspace_status) after the wait limit instead of completing. Other rows take tiles from an atomic
 * ticket and complete whatever runs beside them. */
UP_API int up_sm100_scan_i32(const int32_t* x, int32_t* y, int64_t rows, int64_t k, int op, int exclusive,
                      int reverse, const int32_t* carry_in, void* workspace, size_t workspace_bytes,
                      void* stream);
UP_API size_t up_sm100_scan_workspace_bytes(int64_t rows, int64_t k);

/* No counterpart in the reference: up_sm100_scan_i32 for callers that cannot allocate device memory,
 * for example a host runtime whose allocator must not run on this path. The scratch is a built-in
 * device array (256 KiB per device), so nothing is allocated or freed. It holds at most 32768 tiles:
 * rows * ceil(k / 8192) <= 32768, one row of up to 2^28 elements. Larger shapes return
 * UP_ERR_UNSUPPORTED with the reason in up_sm100_last_error. The first call on each device does set-up
 * (looks up the array's address and sets the shared-memory size of every scan kernel variant), and so does
 * the first call after a cudaDeviceReset (a new context); make that call before any stream capture. Every
 * call on a device shares the array, so calls that overlap in time (other streams, other host threads)
 * race; serialize them. `sync` != 0 waits for the scan (cudaStreamSynchronize, which fails under stream
 * capture: pass 0 there) and returns UP_ERR_DEVICE_TIMEOUT if its look-back ran out of time. The timeout
 * flag is sticky: the report also covers any earlier unreported call on this device, and reporting clears
 * it. `sync` == 0 returns once the scan is enqueued. */
UP_API int up_sm100_scan_i32_noalloc(const int32_t* x, int32_t* y, int64_t rows, int64_t k, int op,
                                     int exclusive, int reverse, const int32_t* carry_in, int sync,
                                     void* stream);

/* No counterpart in the reference as a device entry: up_sm100_scan_i32 over HOST buffers, the buffers the
 * reference's own scan evaluation reads and writes (crates/unpopped/src/oracle/plan_window.rs:10-238). The
 * array streams through a ring of device slots on three streams (copy in, scan, copy out), so both
 * directions of the host link and the scan overlap; pinned host memory gives the full copy rate. Rows longer
 * than a slot are cut along the row with the carry derived on the device. `carry_in`: HOST pointer to one
 * int32, or NULL. Blocks until `y` is written. The first call on each device allocates the slots (256 MiB)
 * and its streams, and keeps them; calls are serialized. Returns UP_ERR_DEVICE_TIMEOUT when a bounded
 * device wait ran out. */
UP_API int up_sm100_scan_i32_host(const int32_t* x, int32_t* y, int64_t rows, int64_t k, int op, int exclusive,
                                  int reverse, const int32_t* carry_in);

/* Fold of a whole int32 array to one value (the first pass of a scan sharded over GPUs): SUM (wrapping),
 * MAX or MIN, written to `total` (device, one int32). Deterministic. */
UP_API int up_sm100_reduce_i32(const int32_t* x, int64_t n, int op, int32_t* total, void* stream);

/* Row gather `out[n, :] = table[ids[n], :]` (ReadIndex::Indexed on axis 0, ir.rs:2620-2669; oracle
 * oracle/plan_eval.rs:363-385): the row is copied bit for bit; an id outside [0, table_rows) writes
 * nothing (SKIP), zeros (ZERO_FILL) or the clamped row (CLAMP). `row_bytes` is the row size in bytes;
 * `index_dtype` is UP_EK_I32, UP_EK_I64 or UP_EK_U32. */
UP_API int up_sm100_gather_rows(const void* table, int64_t table_rows, int64_t row_bytes, const void* ids,
                         int index_dtype, int64_t n, int oob, void* out, void* stream);

/* Group-wise int4 dequant: out[n][k] = bf16(w[n][k] * scale[n][k / group]) with one rounding (RNE).
 * `w` is [N, K] i4 packed two per byte along K (low nibble first), `scale` f16 [N, K/group]. */
UP_API int up_sm100_dequant_i4_bf16(const uint8_t* w, const uint16_t* scale, int64_t n, int64_t k,
                             int64_t group, uint16_t* out, void* stream);

/* W4A16 GEMM: out[m][n] = bf16( sum_k x[m][k] * w[n][k] * scale[n][k / group] ), f32 accumulation on
 * the tcgen05 tensor cores (TMEM accumulator, per-group scale applied in f32). `x` bf16 [M, K]
 * row-major, `out` bf16 [M, N] row-major, M <= 16 per call tile, K % group == 0, group % 128 == 0,
 * N % 128 == 0. `workspace` from up_sm100_w4a16_workspace_bytes (split-K partials and counters),
 * zero-filled before its first use. */
UP_API int up_sm100_w4a16_gemm(const uint8_t* w, const uint16_t* scale, const uint16_t* x, int64_t m,
                        int64_t n, int64_t k, int64_t group, uint16_t* out, void* workspace,
                        size_t workspace_bytes, void* stream);
UP_API size_t up_sm100_w4a16_workspace_bytes(int64_t m, int64_t n, int64_t k, int64_t group);

/* ---- Several GPUs of one node ------------------------------------------------------------------------
 *
 * The reference models a launch over several devices as the same kernel run per device on its slice of the
 * launch (crates/unpopped/src/oracle/kernel_launch.rs:100-129, run_launch_devices; crates/unpopped/src/exec.rs:
 * 119-143, LaunchShape::devices). A communicator joins the ranks of one node (at most 8), one GPU each; each rank
 * calls up_sm100_launch_multi with its own shard, and the library runs the lift's exchange step (NCCL over
 * NVLink, or peer stores for the block-cyclic scan). NCCL is loaded at run time (libnccl.so.2); without it these
 * entry points return UP_ERR_COMM. Calls on one communicator are collectives: every rank makes the same calls
 * in the same order, each on one stream of its own. */
typedef struct up_comm up_comm;

/* A new NCCL unique id (128 bytes) for a multi-process communicator: one rank makes it and the host's own channel
 * (a store, MPI, torch.distributed) carries it to the others. */
UP_API int up_sm100_comm_unique_id(unsigned char id[128]);
/* Joins this process, on the current device, as `rank` of `nranks` (1..8) to the communicator named by `id`.
 * Blocks until every rank has joined. */
UP_API int up_sm100_comm_init_rank(int nranks, int rank, const unsigned char id[128], up_comm** comm);
/* One process driving `n_gpus` devices: comms[i] is rank i on devs[i] (ncclCommInitAll); peer access is enabled
 * between the devices. A call on comms[i] needs devs[i] current. The collective exchanges (the contiguous-shard
 * scan, W4A16) need one process per GPU; the block-cyclic scan and the row-parallel lifts run either way. */
UP_API int up_sm100_comm_init(int n_gpus, const int* devs, up_comm** comms);
UP_API int up_sm100_comm_destroy(up_comm* comm);
UP_API int up_sm100_comm_rank(const up_comm* comm, int* rank, int* nranks);

/* Workspace of up_sm100_launch_multi on this rank's operands (the W4A16 GEMM adds room for the output slices). */
UP_API int up_sm100_workspace_bytes_multi(int kernel_id, const up_tensor* ins, int n_in, const up_tensor* outs,
                                          int n_out, const int64_t* scalars, int n_scalars, const up_comm* comm,
                                          size_t* bytes);
/* This rank's shard of a lift, with the lift's exchange step, on `stream` (the communicator's device current).
 * Operands are this rank's, as for up_sm100_launch:
 *  SCAN_I32:            ins {x i32, this rank's shard}, outs {y}; scalars {op, exclusive, reverse, layout}.
 *                       layout 0: the global array is the shards in rank order. Each rank folds its shard, the
 *                       ranks all-gather the totals (NCCL), and each scans with the fold of the totals before it
 *                       (after it, reverse): two passes over the data. layout 1: block-cyclic. The global array
 *                       is a sequence of stripes of 148 x 8192 elements, stripe s on rank s % G as that rank's
 *                       local stripe s / G. One pass: each rank's CTA 0 stores its local stripes' aggregates into
 *                       the other ranks' memory over NVLink, and the look-back adds those that sit before each
 *                       tile. Forward only; shards of at least 148 x 8192 elements, 16-byte aligned, whole 16-byte
 *                       chunks, the same size on every rank; every rank on its own GPU. Either layout is bit-exact
 *                       to the single-GPU scan of the global array. Status after the fact:
 *                       up_sm100_workspace_status on this rank's workspace.
 *  W4A16_GEMM:          ins {w i4 [Nl, K] (this rank's weight rows), scale f16 [Nl, K/group], x bf16 [M, K]},
 *                       outs {out bf16 [M, G * Nl]}, scalars {group}: the rank's slice, then an NCCL all-gather of
 *                       every slice into the whole output on every rank (rank g's rows are columns g*Nl ..).
 *  ROW_SUM_F32, ROW_MAX_ARGMAX_BF16, GATHER_ROWS, DEQUANT_I4: independent (output) rows; each rank runs its
 *                       shard as up_sm100_launch does, with no collective. */
UP_API int up_sm100_launch_multi(int kernel_id, const up_tensor* ins, int n_in, const up_tensor* outs, int n_out,
                                 const int64_t* scalars, int n_scalars, void* workspace, size_t workspace_bytes,
                                 void* stream, up_comm* comm);

/* ---- Test and tuning hooks ----------------------------------------------------------------------- */

/* Makes `launches` the block-cyclic launch count of `comm` (its low 30 bits tag the stripe words), so that a test
 * can cross a wrap of the tag; every rank must set the same value. */
UP_API void up_sm100_comm_set_test_launches(up_comm* comm, uint64_t launches);

/* Bound, in nanoseconds, of every device-side wait (default 1e9). */
UP_API void up_sm100_set_wait_limit_ns(uint64_t ns);
/* When nonzero, the next scan launches make tile 0 withhold its look-back flag, so every other tile's wait
 * runs out: the host-visible error path of a bounded wait, without hanging or faulting the GPU. */
UP_API void up_sm100_set_test_withhold_flag(int enable);
/* Makes `next` the 64-bit launch count the next scan uses (its flags carry the low 30 bits). Tests use it to
 * cross a wrap of the 30-bit tag without 2^30 launches. */
UP_API void up_sm100_set_test_scan_epoch(uint64_t next);
/* Number of kernels this library has launched since load (all entry points). */
UP_API uint64_t up_sm100_launch_count(void);
/* Last CUDA error text seen by the library (static storage). */
UP_API const char* up_sm100_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* UP_SM100_H */
