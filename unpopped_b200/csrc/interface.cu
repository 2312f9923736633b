// interface.cu — the interface artifacts a consumer binds a lowered kernel by (§ "Contract / interface artifacts"):
// the `KernelInterface` of each kernel id (crates/unpopped/src/kernel_interface.rs:196-230: launch geometry, the
// parameters with role, element kind and rank, dynamic shared memory, the entry symbol, launch bounds, cooperative
// launch, required capabilities, fidelity notes) as JSON, and each kernel's source revision hash (FNV-1a 64 over its
// source file, as `GeneratedKernel::revision_hash`, backend.rs:173-175 and revision.rs), which the link registry's
// rows carry (link.rs:27-42). Host code only.
#include "common.cuh"

#include <cstdio>
#include <cstring>
#include <string>

namespace up {
uint64_t revision_backend();
uint64_t revision_colsplit();
uint64_t revision_dequant();
uint64_t revision_gather();
uint64_t revision_reduce();
uint64_t revision_reduce2d();
uint64_t revision_rowreduce();
uint64_t revision_scan();
uint64_t revision_scatter();
uint64_t revision_w4a16();
uint64_t revision_window();
size_t scan_persist_smem_bytes();
size_t w4a16_smem_bytes();
}  // namespace up

using namespace up;

extern "C" uint64_t up_sm100_revision_hash(int kernel_id) {
  switch (kernel_id) {
    case UP_K_ROW_SUM_F32:
    case UP_K_ROW_MAX_ARGMAX_BF16: return revision_reduce();
    case UP_K_SCAN_I32: return revision_scan();
    case UP_K_GATHER_ROWS: return revision_gather();
    case UP_K_DEQUANT_I4: return revision_dequant();
    case UP_K_W4A16_GEMM: return revision_w4a16();
    case UP_K_REDUCE2D_F32:
    case UP_K_REDUCE2D_I32:
    case UP_K_REDUCE_F32:
    case UP_K_REDUCE_I32: return revision_reduce2d();
    case UP_K_SCATTER:
    case UP_K_BINCOUNT: return revision_scatter();
    case UP_K_ROW_REDUCE_F32: return revision_rowreduce();
    case UP_K_COL_SUM_SPLITK: return revision_colsplit();
    case UP_K_WINDOW:
    case UP_K_IM2COL: return revision_window();
    default: return 0;
  }
}

// The JSON body of one kernel's interface (everything but the revision, added below). Parameters follow the
// generic launch's operand order (inputs, then outputs), then the launch scalars; `rank` -1 is any rank.
static const char* interface_body(int id) {
  switch (id) {
    case UP_K_ROW_SUM_F32:
      return R"J({"entry_symbol":"up_sm100_row_sum_f32","params":[{"name":"x","role":"read","elem":"F32","rank":2},{"name":"out","role":"write","elem":"F32","rank":1},{"name":"accum","role":"scalar","elem":"I32"},{"name":"block","role":"scalar","elem":"I32"}],"launch":{"block":[256,1,1],"grid":"min(rows, 8 per SM) CTAs, a row per CTA at a time","cluster":null,"dynamic_shared_bytes":"rows per CTA x block x 8 (Auto)"},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a"],"fidelity_notes":["F32 policy: a fixed tree order, deterministic, |got - exact| <= 2^-20 sum|x| for cols <= 8192","Auto policy: the launched lift's documented f64 order for the block, bit-exact"],"workspace":null})J";
    case UP_K_ROW_MAX_ARGMAX_BF16:
      return R"J({"entry_symbol":"up_sm100_row_max_argmax_bf16","params":[{"name":"x","role":"read","elem":"BF16","rank":2},{"name":"max","role":"write","elem":"F32","rank":1},{"name":"argmax","role":"write","elem":"I64|I32","rank":1}],"launch":{"block":[256,1,1],"grid":"a CTA per row","cluster":null,"dynamic_shared_bytes":0},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a"],"fidelity_notes":[],"workspace":null})J";
    case UP_K_SCAN_I32:
      return R"J({"entry_symbol":"up_sm100_scan_i32","params":[{"name":"x","role":"read","elem":"I32","rank":-1},{"name":"y","role":"write","elem":"I32","rank":-1},{"name":"op","role":"scalar","elem":"I32"},{"name":"exclusive","role":"scalar","elem":"I32"},{"name":"reverse","role":"scalar","elem":"I32"}],"launch":{"block":[576,1,1],"grid":"persistent, one CTA per SM","cluster":null,"dynamic_shared_bytes":%SMEM%},"launch_bounds":{"max_threads":576,"min_blocks":1},"cooperative":false,"requires":["sm_100a","cp.async.bulk","mbarrier"],"fidelity_notes":["the look-back waits are bounded; a wait that runs out reports UP_ERR_DEVICE_TIMEOUT through the workspace"],"workspace":"look-back flags and an error word: up_sm100_scan_workspace_bytes, zero-filled once"})J";
    case UP_K_GATHER_ROWS:
      return R"J({"entry_symbol":"up_sm100_gather_rows","params":[{"name":"table","role":"read","elem":"any","rank":2},{"name":"ids","role":"read","elem":"I32|I64|U32","rank":1},{"name":"out","role":"write","elem":"any","rank":2},{"name":"oob","role":"scalar","elem":"I32"}],"launch":{"block":[256,1,1],"grid":"a warp per output row, 4 rows in flight per warp","cluster":null,"dynamic_shared_bytes":0},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a"],"fidelity_notes":[],"workspace":null})J";
    case UP_K_DEQUANT_I4:
      return R"J({"entry_symbol":"up_sm100_dequant_i4_bf16","params":[{"name":"w","role":"read","elem":"I4","rank":2},{"name":"scale","role":"read","elem":"F16","rank":2},{"name":"out","role":"write","elem":"BF16","rank":2},{"name":"group","role":"scalar","elem":"I64"}],"launch":{"block":[256,1,1],"grid":"a CTA per row, up to 32 per SM","cluster":null,"dynamic_shared_bytes":0},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a"],"fidelity_notes":[],"workspace":null})J";
    case UP_K_W4A16_GEMM:
      return R"J({"entry_symbol":"up_sm100_w4a16_gemm","params":[{"name":"w","role":"read","elem":"I4","rank":2},{"name":"scale","role":"read","elem":"F16","rank":2},{"name":"x","role":"read","elem":"BF16","rank":2},{"name":"out","role":"write","elem":"BF16","rank":2},{"name":"group","role":"scalar","elem":"I64"}],"launch":{"block":[640,1,1],"grid":"persistent, one CTA per SM, stream-K over 128-row units","cluster":null,"dynamic_shared_bytes":%SMEM%},"launch_bounds":{"max_threads":640,"min_blocks":1},"cooperative":false,"requires":["sm_100a","tcgen05","tensor_memory","tma","mbarrier"],"fidelity_notes":["bf16 output within 1/2 ulp of the exact value plus gamma(K + 2G + 2) sum|x w s| with u = 2^-24 (f32 tensor-core accumulation)","split tiles are fixed up in CTA order: deterministic"],"workspace":"split-tile partials and counters: up_sm100_w4a16_workspace_bytes, zero-filled once"})J";
    case UP_K_REDUCE2D_F32:
    case UP_K_REDUCE_F32:
      return R"J({"entry_symbol":"up_sm100_reduce2d_f32","params":[{"name":"x","role":"read","elem":"F32","rank":-1},{"name":"out","role":"write","elem":"F32","rank":-1},{"name":"op","role":"scalar","elem":"I32"},{"name":"axis_or_mask","role":"scalar","elem":"I32"},{"name":"accum","role":"scalar","elem":"I32"},{"name":"block","role":"scalar","elem":"I32"}],"launch":{"block":[256,1,1],"grid":"last axis: two CTAs per SM over rows; outer/middle axis: 128-column strips x an 8-CTA cluster (Max/Min, documented Sum) or a warp per 32 columns (serial Sum), batches on gridDim.z","cluster":[1,8,1],"dynamic_shared_bytes":"serial Sum: 48 KiB; documented Sum (block < 64): block x 256 B"},"launch_bounds":{"max_threads":512,"min_blocks":0},"cooperative":false,"requires":["sm_100a","thread_block_clusters","distributed_shared_memory","cp.async"],"fidelity_notes":[],"workspace":null})J";
    case UP_K_REDUCE2D_I32:
    case UP_K_REDUCE_I32:
      return R"J({"entry_symbol":"up_sm100_reduce2d_i32","params":[{"name":"x","role":"read","elem":"I32","rank":-1},{"name":"out","role":"write","elem":"I32","rank":-1},{"name":"op","role":"scalar","elem":"I32"},{"name":"axis_or_mask","role":"scalar","elem":"I32"}],"launch":{"block":[256,1,1],"grid":"last axis: two CTAs per SM over rows; outer axis: column strips x row splits, combined by atomics","cluster":null,"dynamic_shared_bytes":0},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a","int32_atomics"],"fidelity_notes":[],"workspace":null})J";
    case UP_K_SCATTER:
      return R"J({"entry_symbol":"up_sm100_scatter","params":[{"name":"updates","role":"read","elem":"I32|U32|I64|F32|F64","rank":2},{"name":"ids","role":"read","elem":"I32|I64|U32","rank":-1},{"name":"out","role":"readwrite","elem":"I32|U32|I64|F32|F64","rank":2},{"name":"combine","role":"scalar","elem":"I32"},{"name":"full_index","role":"scalar","elem":"I32"}],"launch":{"block":[256,1,1],"grid":"a warp per update row","cluster":null,"dynamic_shared_bytes":0},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a","int32_atomics","int64_atomics","float_atomics"],"fidelity_notes":["a float AtomicAdd reassociates: |got - exact| <= gamma(n-1) sum|terms| (kernel_parallel_float_scatter_band.rs)"],"workspace":null})J";
    case UP_K_BINCOUNT:
      return R"J({"entry_symbol":"up_sm100_bincount","params":[{"name":"x","role":"read","elem":"I32|I64|U32","rank":1},{"name":"counts","role":"readwrite","elem":"I32","rank":1}],"launch":{"block":[256,1,1],"grid":"grid-stride, up to 16 CTAs per SM","cluster":null,"dynamic_shared_bytes":0},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a","int32_atomics"],"fidelity_notes":[],"workspace":null})J";
    case UP_K_ROW_REDUCE_F32:
      return R"J({"entry_symbol":"up_sm100_row_reduce_f32","params":[{"name":"x","role":"read","elem":"F32","rank":-1},{"name":"out","role":"write","elem":"F32","rank":-1},{"name":"form","role":"scalar","elem":"I32"},{"name":"block","role":"scalar","elem":"I32"},{"name":"eps","role":"scalar","elem":"F64"}],"launch":{"block":[256,1,1],"grid":"two CTAs per SM over row groups (rows of at most 32 elements per thread), else 8 per SM","cluster":null,"dynamic_shared_bytes":65536},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a","cp.async","fp64"],"fidelity_notes":["exp and sqrt are CUDA's f64 functions; softmax and RMS norm stay within 4 f32 ulps of the serial lift, as the reference states"],"workspace":null})J";
    case UP_K_COL_SUM_SPLITK:
      return R"J({"entry_symbol":"up_sm100_col_sum_f32_splitk","params":[{"name":"x","role":"read","elem":"F32","rank":2},{"name":"out","role":"write","elem":"F32","rank":1},{"name":"mean","role":"scalar","elem":"I32"},{"name":"n_chunks","role":"scalar","elem":"I64"}],"launch":{"block":[256,1,1],"grid":"partial: column strips x n_chunks; combine: a thread per column","cluster":null,"dynamic_shared_bytes":0},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a","fp64"],"fidelity_notes":["ReassociatedDeterministic: f64 chunk partials added in chunk order, a different association than the serial fold; n_chunks = 1 is the serial fold"],"workspace":"n_chunks x cols f64 partials: up_sm100_col_sum_splitk_workspace_bytes"})J";
    case UP_K_WINDOW:
      return R"J({"entry_symbol":"up_sm100_window","params":[{"name":"x","role":"read","elem":"F32|I32","rank":-1},{"name":"out","role":"write","elem":"F32|I32","rank":-1},{"name":"op","role":"scalar","elem":"I32"},{"name":"size","role":"scalar","elem":"I32"},{"name":"stride","role":"scalar","elem":"I32"},{"name":"dilation","role":"scalar","elem":"I32"},{"name":"pad_lo","role":"scalar","elem":"I32"},{"name":"count_include_pad","role":"scalar","elem":"I32"},{"name":"axis","role":"scalar","elem":"I32"}],"launch":{"block":[256,1,1],"grid":"a CTA per row (innermost axis; the row staged by cp.async into 32 KiB of static shared memory) or per group of lines, up to 16 per SM","cluster":null,"dynamic_shared_bytes":0},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a","cp.async"],"fidelity_notes":[],"workspace":null})J";
    case UP_K_IM2COL:
      return R"J({"entry_symbol":"up_sm100_im2col","params":[{"name":"x","role":"read","elem":"any","rank":4},{"name":"out","role":"write","elem":"any","rank":3},{"name":"kh","role":"scalar","elem":"I32"},{"name":"kw","role":"scalar","elem":"I32"},{"name":"sh","role":"scalar","elem":"I32"},{"name":"sw","role":"scalar","elem":"I32"},{"name":"ph","role":"scalar","elem":"I32"},{"name":"pw","role":"scalar","elem":"I32"},{"name":"dh","role":"scalar","elem":"I32"},{"name":"dw","role":"scalar","elem":"I32"}],"launch":{"block":[256,1,1],"grid":"a CTA per input plane staged in dynamic shared memory (the plane's bytes, at most 96 KiB), else a CTA per output row; up to 16 per SM","cluster":null,"dynamic_shared_bytes":0},"launch_bounds":{"max_threads":256,"min_blocks":0},"cooperative":false,"requires":["sm_100a"],"fidelity_notes":[],"workspace":null})J";
    default: return nullptr;
  }
}

extern "C" int up_sm100_kernel_interface(int kernel_id, char* buf, size_t cap, size_t* len) {
  const char* body = interface_body(kernel_id);
  if (!body) return fail_with(UP_ERR_UNSUPPORTED, "kernel_interface: no such kernel id");
  std::string text(body);
  const size_t at = text.find("%SMEM%");  // the persistent kernels' dynamic shared memory, from their constants
  if (at != std::string::npos) {
    const size_t smem = kernel_id == UP_K_SCAN_I32 ? scan_persist_smem_bytes() : w4a16_smem_bytes();
    text.replace(at, 6, std::to_string(smem));
  }
  if (kernel_id == UP_K_REDUCE_F32 || kernel_id == UP_K_REDUCE_I32) {  // the flattened-geometry entry
    const size_t e = text.find("up_sm100_reduce2d_");
    if (e != std::string::npos) text.replace(e, 18, "up_sm100_reduce3d_");
  }
  char rev[64];
  std::snprintf(rev, sizeof(rev), ",\"revision_hash\":\"0x%016llx\"}",
                (unsigned long long)up_sm100_revision_hash(kernel_id));
  text.pop_back();  // the closing brace
  text += rev;
  if (len) *len = text.size();
  if (!buf) return UP_OK;  // a NULL buffer asks for the length
  if (cap < text.size() + 1) return UP_ERR_INVALID;
  std::memcpy(buf, text.c_str(), text.size() + 1);
  return UP_OK;
}

UP_DEFINE_REVISION(interface)
