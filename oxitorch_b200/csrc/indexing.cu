// indexing.cu -- row selection for the dim-0 scatter and its VJP (sm_100a).
//
// The reference runs Tensor::scatter_dim0 (crates/oxi-tensor/src/lib.rs:895-933)
// and the VJP of ops::scatter_dim0 (crates/oxi-autograd/src/ops.rs:531-598) as
// host loops over to_vec() copies.  All three results are row selections:
//
//   forward      out[r]  = written(r) ? values[last writer of r] : base[r]
//   d/dbase      gb[r]   = written(r) ? 0 : g[r]
//   d/dvalues    gv[p]   = p is the last writer of its row ? g[row of p] : 0
//
// so one kernel serves them: out[i] = map[i] >= 0 ? a[map[i]] : (b ? b[i] : 0),
// rows of `inner` floats.  The host resolves the last-write-wins map from the
// index list (which the reference's API takes as a host slice), so the device
// work is one coalesced pass: read each selected row once, write each output
// row once.  HBM-bound; a warp per row with 128-bit accesses where the rows
// and pointers allow, grid-stride over rows.
#include <algorithm>

#include "common.cuh"

namespace oxc {

__device__ __forceinline__ void select_record_bad(int32_t* flag, int64_t value, int64_t size) {
  if (flag && atomicCAS(flag, 0, 1) == 0) {
    flag[1] = (int32_t)(uint32_t)((uint64_t)value & 0xffffffffu);
    flag[2] = (int32_t)(uint32_t)((uint64_t)value >> 32);
    flag[3] = (int32_t)size;
  }
}

// T = float4 (inner4 = inner / 4 vectors per row) or float (inner4 = inner).
template <typename T>
__global__ void __launch_bounds__(256) select_rows_kernel(const T* __restrict__ a, int64_t a_rows,
                                                          const int64_t* __restrict__ map, int64_t n,
                                                          const T* __restrict__ b, T* __restrict__ out,
                                                          int64_t vecs, int32_t* err) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t i = warp; i < n; i += nwarps) {
    const int64_t r = map[i];
    T* d = out + i * vecs;
    if (r >= a_rows) {
      if (lane == 0) select_record_bad(err, r, a_rows);
      continue;
    }
    if (r >= 0) {
      const T* s = a + r * vecs;
      for (int64_t k = lane; k < vecs; k += 32) d[k] = __ldg(s + k);
    } else if (b) {
      const T* s = b + i * vecs;
      for (int64_t k = lane; k < vecs; k += 32) d[k] = __ldg(s + k);
    } else {
      const T z{};
      for (int64_t k = lane; k < vecs; k += 32) d[k] = z;
    }
  }
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_select_rows(const float* a, int64_t a_rows, const int64_t* map, int64_t n,
                           const float* b, float* out, int64_t inner, int32_t* err_flag,
                           void* stream) {
  if (a_rows < 0 || n < 0 || inner < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: select_rows: negative size");
  if (n == 0 || inner == 0) return OXC_OK;
  if (!map || !out || (a_rows > 0 && !a))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: select_rows: null pointer");
  const bool v4 = inner % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(out);
  const int64_t vecs = v4 ? inner / 4 : inner;
  const int64_t cap = (int64_t)sm_count() * 8 * 4;  // 8 CTAs of 256 per SM, 4 waves
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, cap));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v4)
    select_rows_kernel<float4><<<grid, 256, 0, s>>>(reinterpret_cast<const float4*>(a), a_rows, map, n,
                                                    reinterpret_cast<const float4*>(b),
                                                    reinterpret_cast<float4*>(out), vecs, err_flag);
  else
    select_rows_kernel<float><<<grid, 256, 0, s>>>(a, a_rows, map, n, b, out, vecs, err_flag);
  return check_launch("oxc_select_rows");
}

}  // extern "C"
