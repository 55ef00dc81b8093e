// abi.cu -- library-level C ABI: errors, device queries, synchronisation,
// registry id tables and the shared column-sum finisher.
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "common.cuh"

namespace oxc {

static thread_local char g_last_error[512] = {0};

oxc_status fail(oxc_status code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

oxc_status cuda_fail(cudaError_t err, const char* what) {
  return fail(OXC_ERR_OTHER, "%s: CUDA error %s (%s)", what, cudaGetErrorName(err),
              cudaGetErrorString(err));
}

oxc_status check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(err, what);
  return OXC_OK;
}

void clear_error() { g_last_error[0] = 0; }

static std::vector<kernel_error_reader>& kernel_error_readers() {
  static std::vector<kernel_error_reader> readers;
  return readers;
}

int register_kernel_error_reader(kernel_error_reader fn) {
  kernel_error_readers().push_back(fn);
  return (int)kernel_error_readers().size();
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

int occupancy(const void* kernel, int block, size_t smem) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, block, smem) != cudaSuccess || n <= 0)
    n = 1;
  return n;
}

// Column sums of per-CTA partials.  CTA = 32 warps x 32 columns; warp w adds
// parts w, w+32, w+64, ... (4 loads in flight), then warp 0 adds the 32 warp
// results in warp order.  Fixed order => deterministic.
// blockIdx.y selects the column set: (parts1, out1) or (parts2, out2), so the
// dweight and dbias sums of a VJP finish in one launch.
__global__ void __launch_bounds__(1024) colsum_partials_kernel(const float* __restrict__ parts1,
                                                               int nparts, int64_t cols,
                                                               float* __restrict__ out1,
                                                               const float* __restrict__ parts2,
                                                               float* __restrict__ out2) {
  const float* __restrict__ parts = blockIdx.y ? parts2 : parts1;
  float* __restrict__ out = blockIdx.y ? out2 : out1;
  __shared__ float red[32][33];
  pdl_wait();  // the partials are the previous kernel's output
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.x * 32 + lane;
  float acc = 0.0f;
  if (col < cols) {
    int p = warp;
    for (; p + 96 < nparts; p += 128) {
      const float a = parts[(int64_t)p * cols + col];
      const float b = parts[(int64_t)(p + 32) * cols + col];
      const float c = parts[(int64_t)(p + 64) * cols + col];
      const float d = parts[(int64_t)(p + 96) * cols + col];
      acc = __fadd_rn(acc, a);
      acc = __fadd_rn(acc, b);
      acc = __fadd_rn(acc, c);
      acc = __fadd_rn(acc, d);
    }
    for (; p < nparts; p += 32) acc = __fadd_rn(acc, parts[(int64_t)p * cols + col]);
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && col < cols) {
    float s = red[0][lane];
    for (int w = 1; w < 32; ++w) s = __fadd_rn(s, red[w][lane]);
    out[col] = s;
  }
}

void launch_colsum_partials(const float* parts, int nparts, int64_t cols, float* out,
                            cudaStream_t stream, const float* parts2, float* out2) {
  launch_dependent(colsum_partials_kernel, dim3((unsigned)((cols + 31) / 32), parts2 ? 2u : 1u),
                   dim3(1024), stream, parts, nparts, cols, out, parts2, out2);
}

}  // namespace oxc

using namespace oxc;

static const char* const kBinary[] = {"add", "sub", "mul", "div", "pow", "min", "max"};
static const char* const kCmp[] = {"eq", "ne", "lt", "le", "gt", "ge"};
static const char* const kUnary[] = {"neg",  "abs",   "sqrt",    "rsqrt", "exp",   "log",   "log2",
                                     "log10", "sin",  "cos",     "tanh",  "relu",  "sigmoid",
                                     "floor", "ceil", "round",   "sign",  "square", "reciprocal"};
static const char* const kReduce[] = {"sum", "mean", "max", "min", "argmax", "argmin", "norm"};

template <size_t N>
static int32_t lookup(const char* const (&table)[N], const char* name) {
  if (!name) return -1;
  for (size_t i = 0; i < N; ++i)
    if (std::strcmp(table[i], name) == 0) return (int32_t)i;
  return -1;
}

extern "C" {

int32_t oxc_abi_version(void) { return 1; }

const char* oxc_last_error(void) { return g_last_error; }

int32_t oxc_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

oxc_status oxc_stream_sync(void* stream, int64_t timeout_ms) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (timeout_ms < 0) {
    cudaError_t e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? OXC_OK : cuda_fail(e, "oxc_stream_sync");
  }
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  for (;;) {
    cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return OXC_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, "oxc_stream_sync");
    if (std::chrono::steady_clock::now() >= deadline)
      return fail(OXC_ERR_TIMEOUT, "timeout: stream did not drain within %lld ms",
                  (long long)timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

oxc_status oxc_check_error_flag(int32_t* flag_dev, void* stream, int64_t timeout_ms) {
  if (!flag_dev) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: null error flag");
  oxc_status st = oxc_stream_sync(stream, timeout_ms);
  if (st != OXC_OK) return st;
  int32_t host[4] = {0, 0, 0, 0};
  cudaError_t e = cudaMemcpy(host, flag_dev, sizeof(host), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "oxc_check_error_flag");
  if (host[0] == 0) return OXC_OK;
  const int64_t idx = (int64_t)(((uint64_t)(uint32_t)host[2] << 32) | (uint32_t)host[1]);
  const int32_t zero[4] = {0, 0, 0, 0};
  e = cudaMemcpy(flag_dev, zero, sizeof(zero), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "oxc_check_error_flag");
  // flag[0] is 1 + the indexed dim (kernels indexing dim 0 store 1)
  return fail(OXC_ERR_OUT_OF_BOUNDS, "out of bounds: index %lld out of range for dim %d of size %d",
              (long long)idx, host[0] - 1, host[3]);
}

oxc_status oxc_kernel_error(uint32_t* bits, int32_t clear) {
  if (!bits) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: null bits pointer");
  *bits = 0;
  for (kernel_error_reader fn : kernel_error_readers()) {
    unsigned int v = 0;
    cudaError_t e = fn(&v, clear);
    if (e != cudaSuccess) return cuda_fail(e, "oxc_kernel_error");
    *bits |= v;
  }
  return OXC_OK;
}

int32_t oxc_binary_op_id(const char* name) { return lookup(kBinary, name); }
int32_t oxc_cmp_op_id(const char* name) { return lookup(kCmp, name); }
int32_t oxc_unary_op_id(const char* name) { return lookup(kUnary, name); }
int32_t oxc_reduce_kind_id(const char* name) { return lookup(kReduce, name); }

}  // extern "C"
