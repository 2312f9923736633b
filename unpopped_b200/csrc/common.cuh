// common.cuh — shared host/device helpers of libunpopped_sm100 (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/up_sm100.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libunpopped_sm100 is built for sm_100a only"
#endif

namespace up {

// ---- host-side state shared by the entry points (defined in backend.cpp) ----
void note_launch(uint64_t kernels = 1);
int cuda_status(cudaError_t e);   // maps a CUDA error to UP_ERR_CUDA and records its text
int check_launch();               // cudaGetLastError after a launch
uint64_t wait_limit_ns();
int take_withhold_flag();         // returns and clears the scan test hook
int sm_count();                   // SMs of the current device (cached per device)
int fail_with(int status, const char* text);  // records `text` as the last error, returns `status`
// A number that identifies the current CUDA context for the life of the process (cuCtxGetId); 0 when the driver
// cannot say. A cudaDeviceReset ends the primary context, and the next one gets a new number, so host caches of
// per-context state (function attributes, symbol addresses, allocations) key on it instead of the device index.
uint64_t context_id();
// Raises `func`'s dynamic shared-memory limit to at least `bytes` in the current context. The attribute belongs to
// the context, so this runs the CUDA call once per context and kernel, and again after a device reset.
cudaError_t ensure_smem_attr(const void* func, int bytes);
int row_mean_f32_auto(const float* x, int64_t rows, int64_t cols, int64_t row_stride, int block, float* out,
                      void* stream);  // reduce.cu: the Auto row sum divided by cols

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- device helpers ----
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Streaming (evict-first) 16-byte store: output that is not re-read should not displace inputs in L2.
__device__ __forceinline__ void st_cs_v4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Read-only 16-byte load through the non-coherent path, no L1 allocation (streamed once).
__device__ __forceinline__ uint4 ld_nc_na_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float4 ld_nc_na_f4(const float* p) {
  uint4 u = ld_nc_na_v4(p);
  return make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
}

}  // namespace up

// The source revision of a translation unit: FNV-1a 64 over its .cu file's text, the reference's revision hash
// (crates/unpopped/src/revision.rs), passed in by the build as UP_SOURCE_REVISION.
#ifndef UP_SOURCE_REVISION
#define UP_SOURCE_REVISION 0ull
#endif
#define UP_DEFINE_REVISION(name) \
  namespace up {                 \
  uint64_t revision_##name() { return UP_SOURCE_REVISION; } \
  }

#define UP_CHECK_ARG(cond)         \
  do {                             \
    if (!(cond)) return UP_ERR_INVALID; \
  } while (0)
