// activation.cu -- F.gelu on its own, forward and VJP (python/oxitorch/nn/
// functional.py:194-199), for the GELU that does not follow a LayerNorm.
//
// The reference builds GELU from registry ops (x*x, *x, *0.044715, +x, *C,
// tanh, +1, x*0.5, *) and its graph sums the derivative of every node; here
// the forward is one elementwise kernel and the VJP another, both evaluating
// the tanh form through its logistic identity exactly as the fused
// LayerNorm+GELU kernels do (gelu.cuh): dx = dy * gelu'(x).
//
// Both are HBM-bound streaming passes over dense arrays: 128-bit loads and
// stores with a scalar tail, grid-stride over one wave of resident CTAs.
#include <algorithm>

#include "gelu.cuh"

namespace oxc {

template <int VW>
__global__ void __launch_bounds__(256) gelu_fwd_kernel(const float* __restrict__ x,
                                                       float* __restrict__ y, int64_t n,
                                                       GeluConst gc) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t nv = n / VW;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    if constexpr (VW == 4) {
      const float4 a = ld_stream(reinterpret_cast<const float4*>(x) + v);
      st_stream(reinterpret_cast<float4*>(y) + v,
                make_float4(gelu_fwd(a.x, gc), gelu_fwd(a.y, gc), gelu_fwd(a.z, gc),
                            gelu_fwd(a.w, gc)));
    } else {
      st_stream(y + v, gelu_fwd(ld_stream(x + v), gc));
    }
  }
  if constexpr (VW == 4)
    for (int64_t i = nv * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
      y[i] = gelu_fwd(x[i], gc);
}

template <int VW>
__global__ void __launch_bounds__(256) gelu_bwd_kernel(const float* __restrict__ x,
                                                       const float* __restrict__ dy,
                                                       float* __restrict__ dx, int64_t n,
                                                       GeluConst gc) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t nv = n / VW;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    if constexpr (VW == 4) {
      const float4 a = ld_stream(reinterpret_cast<const float4*>(x) + v);
      const float4 g = ld_stream(reinterpret_cast<const float4*>(dy) + v);
      st_stream(reinterpret_cast<float4*>(dx) + v,
                make_float4(gelu_grad(a.x, g.x, gc), gelu_grad(a.y, g.y, gc),
                            gelu_grad(a.z, g.z, gc), gelu_grad(a.w, g.w, gc)));
    } else {
      st_stream(dx + v, gelu_grad(ld_stream(x + v), ld_stream(dy + v), gc));
    }
  }
  if constexpr (VW == 4)
    for (int64_t i = nv * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
      dx[i] = gelu_grad(x[i], dy[i], gc);
}

template <typename K>
static unsigned wave_grid(K kernel, int64_t work) {
  const int64_t fit = (int64_t)sm_count() * std::max(1, occupancy((const void*)kernel, 256, 0));
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, fit));
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_gelu_fwd(const float* x, float* y, int64_t n, void* stream) {
  if (n < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: gelu: negative size");
  if (n == 0) return OXC_OK;
  if (!x || !y) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: gelu: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const GeluConst gc = gelu_const();
  if (aligned16(x) && aligned16(y))
    gelu_fwd_kernel<4><<<wave_grid(gelu_fwd_kernel<4>, n / 4), 256, 0, s>>>(x, y, n, gc);
  else
    gelu_fwd_kernel<1><<<wave_grid(gelu_fwd_kernel<1>, n), 256, 0, s>>>(x, y, n, gc);
  return check_launch("oxc_gelu_fwd");
}

oxc_status oxc_gelu_bwd(const float* x, const float* dy, float* dx, int64_t n, void* stream) {
  if (n < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: gelu backward: negative size");
  if (n == 0) return OXC_OK;
  if (!x || !dy || !dx)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: gelu backward: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const GeluConst gc = gelu_const();
  if (aligned16(x) && aligned16(dy) && aligned16(dx))
    gelu_bwd_kernel<4><<<wave_grid(gelu_bwd_kernel<4>, n / 4), 256, 0, s>>>(x, dy, dx, n, gc);
  else
    gelu_bwd_kernel<1><<<wave_grid(gelu_bwd_kernel<1>, n), 256, 0, s>>>(x, dy, dx, n, gc);
  return check_launch("oxc_gelu_bwd");
}

}  // extern "C"
