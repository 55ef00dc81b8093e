// no_alloc.cu -- LayerNorm(+GELU) backward for callers that cannot allocate.
//
// oxc_layer_norm_bwd needs a workspace for its per-CTA dweight/dbias partials,
// which the caller normally allocates.  Some callers cannot: a host that owns
// all device memory through its own pool (where a cudaMalloc outside the pool
// fails or fragments the reservation), or a latency-critical step where
// cudaMalloc's implicit device synchronisation is not acceptable.  For them,
// oxc_layer_norm_bwd_noalloc takes its scratch from a fixed device array
// defined in this file, of OXC_NOALLOC_SCRATCH_BYTES (16 MiB).
//
// Properties a caller must know:
//   - every GPU that loads this library holds the 16 MiB array until the
//     process exits;
//   - the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current, once per device; make
//     that first call before any stream capture.  The address is cached per
//     device for the life of the process; cudaDeviceReset unloads the module
//     that holds the array, so a process that resets a device must not call
//     this entry point on it again (the cached address would be stale);
//   - all calls on a device share the one array: calls whose kernels overlap
//     on the GPU (different streams, or concurrent host threads) race on it
//     and must be serialised by the caller;
//   - the array keeps the last call's contents; nothing in it needs to start
//     at zero, because every partial is written in full before it is read;
//   - sizes whose scratch exceeds the array are rejected with
//     OXC_ERR_INVALID_ARGUMENT before anything is launched.
// It calls no cudaMalloc, cudaFree or allocating library routine.
#include <mutex>

#include "common.cuh"

namespace oxc {

static __device__ __align__(256) unsigned char g_ln_bwd_scratch[OXC_NOALLOC_SCRATCH_BYTES];

// Device address of g_ln_bwd_scratch per device (the host-side symbol is only
// a stand-in and must never be passed to a kernel).
static void* g_scratch_addr[64] = {nullptr};
static std::mutex g_scratch_mu;

static oxc_status scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "oxc_layer_norm_bwd_noalloc (cudaGetDevice)");
  if (dev < 0 || dev >= 64)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: device ordinal %d >= 64", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ln_bwd_scratch);
    if (e != cudaSuccess || !p)
      return cuda_fail(e == cudaSuccess ? cudaErrorInvalidSymbol : e,
                       "oxc_layer_norm_bwd_noalloc (cudaGetSymbolAddress)");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return OXC_OK;
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_layer_norm_bwd_noalloc(const float* x, const float* w, const float* b,
                                      const float* mean, const float* rstd, const float* dy,
                                      float* dx, float* dw, float* db, int64_t rows, int64_t cols,
                                      int32_t act, int32_t grad_mode, void* stream) {
  if (rows < 0 || cols < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: layer_norm backward (no-alloc): negative shape");
  const size_t need = oxc_layer_norm_bwd_workspace_size(rows, cols);
  if (need > (size_t)OXC_NOALLOC_SCRATCH_BYTES)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: layer_norm backward (no-alloc) for [%lld, %lld] needs %zu bytes "
                "of scratch, more than the fixed %zu-byte scratch; call oxc_layer_norm_bwd with a "
                "workspace instead",
                (long long)rows, (long long)cols, need, (size_t)OXC_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  oxc_status st = scratch_address(&scratch);
  if (st) return st;
  return oxc_layer_norm_bwd(x, w, b, mean, rstd, dy, dx, dw, db, rows, cols, act, grad_mode,
                            scratch, (size_t)OXC_NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
