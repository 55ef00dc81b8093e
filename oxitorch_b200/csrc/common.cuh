// common.cuh -- shared plumbing for the oxicuda kernels (sm_100a).
//
// Status/message handling for the C ABI, device-property caching for grid
// sizing, cache-hinted 128-bit loads/stores and deterministic block
// reductions.  Every reduction here combines values in a fixed order, so a
// kernel run twice on the same input gives bit-identical results.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "oxicuda.h"

namespace oxc {

// ---- errors ----------------------------------------------------------------
// Records `msg` as this thread's last error and returns `code`.
oxc_status fail(oxc_status code, const char* fmt, ...);
// Maps a CUDA error (launch or runtime) to OXC_ERR_OTHER with its name.
oxc_status cuda_fail(cudaError_t err, const char* what);
// Checks the last launch of this thread; OXC_OK when it went through.
oxc_status check_launch(const char* what);
void clear_error();

// ---- device-side error words -------------------------------------------------
// Each translation unit with bounded-wait kernels owns a device error word and
// registers a reader for it; oxc_kernel_error() ORs them all.
typedef cudaError_t (*kernel_error_reader)(unsigned int* value, int clear);
int register_kernel_error_reader(kernel_error_reader fn);

// ---- device properties -----------------------------------------------------
// Streaming-multiprocessor count of the current device (148 on B200), cached.
int sm_count();
// Resident CTAs of `kernel` per SM for a block size and dynamic smem size.
int occupancy(const void* kernel, int block, size_t smem);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- cache-hinted vector access ---------------------------------------------
// Streaming loads (evict-first): for data read once per kernel.
__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ float ld_stream(const float* p) { return __ldcs(p); }
// Normal loads through L1/L2 (data that another CTA or kernel re-reads soon).
__device__ __forceinline__ float4 ld_keep(const float4* p) { return __ldg(p); }
__device__ __forceinline__ float ld_keep(const float* p) { return __ldg(p); }
// Streaming stores (evict-first) for outputs nobody reads in this kernel.
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }
__device__ __forceinline__ void st_stream(float* p, float v) { __stcs(p, v); }

// ---- deterministic reductions ------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Max that ignores NaN like Rust's f32::max (crates/oxi-tensor/src/ops.rs:258).
__device__ __forceinline__ float nan_ignoring_max(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; every thread gets the result.  `scratch` holds >= 33 floats.
// The warp partials are combined by warp 0 in warp order.
template <typename T>
__device__ __forceinline__ T block_sum(T v, T* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();  // scratch may still be read by a previous call
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    T t = lane < nwarps ? scratch[lane] : T(0);
    t = warp_sum(t);
    if (lane == 0) scratch[32] = t;
  }
  __syncthreads();
  return scratch[32];
}

__device__ __forceinline__ float block_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < nwarps ? scratch[lane] : -INFINITY;
    t = warp_max(t);
    if (lane == 0) scratch[32] = t;
  }
  __syncthreads();
  return scratch[32];
}

// Programmatic dependent launch.  A kernel launched with the
// programmatic-stream-serialization attribute may be scheduled while the
// kernel before it in the stream is still running; pdl_wait() then blocks
// until that kernel has completed and its memory is visible, so it must come
// before any read of the predecessor's output.  pdl_launch_dependents() in the
// predecessor lets the dependent be scheduled once every CTA of the
// predecessor has issued it (or exited), so a dependent never takes resources
// that a predecessor CTA still waits for.  Both are no-ops without the
// attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launches `kernel` as a programmatic dependent of the previous kernel in the
// stream (the kernel must call pdl_wait() before it reads that kernel's
// output).  A launch error is left for check_launch().
template <typename... KArgs, typename... Args>
inline void launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t s,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Column sums of `parts` [nparts, cols] into out[cols] (f32), in a fixed
// order: warp w of a CTA sums parts w, w+32, ... for 32 columns, then warp
// partials are added in warp order.  Used to finish per-CTA weight-gradient
// partials deterministically.  With parts2/out2 a second set of the same
// shape is summed in the same launch.  Launched as a programmatic dependent
// of the VJP kernel that wrote the partials (that kernel calls
// pdl_launch_dependents()).
void launch_colsum_partials(const float* parts, int nparts, int64_t cols, float* out,
                            cudaStream_t stream, const float* parts2 = nullptr,
                            float* out2 = nullptr);

}  // namespace oxc
