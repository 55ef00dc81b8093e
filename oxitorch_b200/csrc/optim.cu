// optim.cu -- the optimizer step on device: SGD (optionally Nesterov)
// momentum and Adam/AdamW over flat f32 parameters, updated in place.
//
// Reference (crates/oxi-autograd/src/optim.rs), per element, every operation
// an f32 operation rounded on its own (Rust does not contract a*b + c):
//   Sgd::step_param (104-138):
//     buf = momentum * buf + g
//     upd = nesterov ? g + momentum * buf : buf        (momentum == 0: upd = g)
//     p   = p - lr * upd
//   AdamW::step_param (223-261), t = the parameter's own step counter:
//     bc1 = 1 - beta1^t, bc2 = 1 - beta2^t             (f32 powf, once per step)
//     g'  = decoupled || wd == 0 ? g : g + wd * p
//     m   = beta1 * m + (1 - beta1) * g'
//     v   = beta2 * v + ((1 - beta2) * g') * g'
//     p'  = p - (lr * (m / bc1)) / (sqrt(v / bc2) + eps)
//     p'  = p' - (lr * wd) * p                         (decoupled and wd != 0)
// The kernels evaluate exactly that sequence with explicitly rounded
// intrinsics, so on the same inputs they give the reference's bits.  The
// host computes bc1/bc2 with the C library's powf, the function Rust's
// f32::powf calls.
//
// Both are streaming elementwise passes, HBM-bound: SGD with momentum moves
// 20 bytes per element (read p, g, buf; write p, buf), Adam 28 (read p, g,
// m, v; write p, m, v).  128-bit grid-stride loops when every pointer is
// 16-byte aligned, a scalar loop for the rest.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace oxc {

struct AdamConst {
  float lr, beta1, beta2, omb1, omb2, eps, wd, bc1, bc2;
  int decay_grad, decay_param;  // classic Adam: g' = g + wd*p; AdamW: p' -= (lr*wd)*p
};

__device__ __forceinline__ void adam_elem(float& p, float g, float& m, float& v,
                                          const AdamConst& c) {
  const float ge = c.decay_grad ? __fadd_rn(g, __fmul_rn(c.wd, p)) : g;
  m = __fadd_rn(__fmul_rn(c.beta1, m), __fmul_rn(c.omb1, ge));
  v = __fadd_rn(__fmul_rn(c.beta2, v), __fmul_rn(__fmul_rn(c.omb2, ge), ge));
  const float m_hat = __fdiv_rn(m, c.bc1);
  const float v_hat = __fdiv_rn(v, c.bc2);
  float next = __fsub_rn(p, __fdiv_rn(__fmul_rn(c.lr, m_hat), __fadd_rn(__fsqrt_rn(v_hat), c.eps)));
  if (c.decay_param) next = __fsub_rn(next, __fmul_rn(__fmul_rn(c.lr, c.wd), p));
  p = next;
}

template <bool V4>
__global__ void __launch_bounds__(256) adam_kernel(float* __restrict__ p,
                                                   const float* __restrict__ g,
                                                   float* __restrict__ m, float* __restrict__ v,
                                                   int64_t n, AdamConst c) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if constexpr (V4) {
    const int64_t nv = n / 4;
    float4* p4 = reinterpret_cast<float4*>(p);
    float4* m4 = reinterpret_cast<float4*>(m);
    float4* v4 = reinterpret_cast<float4*>(v);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    for (int64_t k = i; k < nv; k += stride) {
      float4 pp = ld_stream(p4 + k), mm = ld_stream(m4 + k), vv = ld_stream(v4 + k);
      const float4 gg = ld_stream(g4 + k);
      adam_elem(pp.x, gg.x, mm.x, vv.x, c);
      adam_elem(pp.y, gg.y, mm.y, vv.y, c);
      adam_elem(pp.z, gg.z, mm.z, vv.z, c);
      adam_elem(pp.w, gg.w, mm.w, vv.w, c);
      st_stream(p4 + k, pp);
      st_stream(m4 + k, mm);
      st_stream(v4 + k, vv);
    }
    i += nv * 4;  // the tail of n % 4 elements
  }
  for (; i < n; i += stride) {
    float pp = p[i], mm = m[i], vv = v[i];
    adam_elem(pp, g[i], mm, vv, c);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
  }
}

struct SgdConst {
  float lr, momentum;
  int use_buf, nesterov;
};

__device__ __forceinline__ void sgd_elem(float& p, float g, float& buf, const SgdConst& c) {
  float upd = g;
  if (c.use_buf) {
    buf = __fadd_rn(__fmul_rn(c.momentum, buf), g);
    upd = c.nesterov ? __fadd_rn(g, __fmul_rn(c.momentum, buf)) : buf;
  }
  p = __fsub_rn(p, __fmul_rn(c.lr, upd));
}

template <bool V4>
__global__ void __launch_bounds__(256) sgd_kernel(float* __restrict__ p,
                                                  const float* __restrict__ g,
                                                  float* __restrict__ buf, int64_t n, SgdConst c) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if constexpr (V4) {
    const int64_t nv = n / 4;
    float4* p4 = reinterpret_cast<float4*>(p);
    float4* b4 = reinterpret_cast<float4*>(buf);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    for (int64_t k = i; k < nv; k += stride) {
      float4 pp = ld_stream(p4 + k);
      const float4 gg = ld_stream(g4 + k);
      float4 bb = c.use_buf ? ld_stream(b4 + k) : make_float4(0, 0, 0, 0);
      sgd_elem(pp.x, gg.x, bb.x, c);
      sgd_elem(pp.y, gg.y, bb.y, c);
      sgd_elem(pp.z, gg.z, bb.z, c);
      sgd_elem(pp.w, gg.w, bb.w, c);
      st_stream(p4 + k, pp);
      if (c.use_buf) st_stream(b4 + k, bb);
    }
    i += nv * 4;
  }
  for (; i < n; i += stride) {
    float pp = p[i], bb = c.use_buf ? buf[i] : 0.0f;
    sgd_elem(pp, g[i], bb, c);
    p[i] = pp;
    if (c.use_buf) buf[i] = bb;
  }
}

// clip_grad_value_ (python/oxitorch/optim.py:266-272) clamps with np.clip:
// min(max(x, lo), hi), where max(a, b) = isnan(a) ? a : (a > b ? a : b) and
// min likewise, so NaN gradients stay NaN, -0.0 stays -0.0 and NaN bounds
// give NaN.
__device__ __forceinline__ float np_clip(float x, float lo, float hi) {
  const float m = isnan(x) ? x : (x > lo ? x : lo);
  return isnan(m) ? m : (m < hi ? m : hi);
}

template <bool V4>
__global__ void __launch_bounds__(256) clip_value_kernel(float* __restrict__ g, int64_t n, float lo,
                                                         float hi) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if constexpr (V4) {
    const int64_t nv = n / 4;
    float4* g4 = reinterpret_cast<float4*>(g);
    for (int64_t k = i; k < nv; k += stride) {
      float4 v = ld_stream(g4 + k);
      v.x = np_clip(v.x, lo, hi);
      v.y = np_clip(v.y, lo, hi);
      v.z = np_clip(v.z, lo, hi);
      v.w = np_clip(v.w, lo, hi);
      st_stream(g4 + k, v);
    }
    i += nv * 4;
  }
  for (; i < n; i += stride) g[i] = np_clip(g[i], lo, hi);
}

static unsigned elem_grid(int64_t work) {
  const int64_t cap = (int64_t)sm_count() * 8 * 4;  // 8 CTAs of 256 per SM, 4 waves
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, cap));
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_sgd_step(float* param, const float* grad, float* velocity, int64_t n, float lr,
                        float momentum, int32_t nesterov, void* stream) {
  if (n < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: sgd step: negative size");
  if (nesterov && !(momentum > 0.0f))
    return fail(OXC_ERR_INVALID_ARGUMENT, "nesterov momentum requires momentum > 0");
  if (n == 0) return OXC_OK;
  const bool use_buf = momentum > 0.0f;
  if (!param || !grad || (use_buf && !velocity))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: sgd step: null pointer");
  const SgdConst c{lr, momentum, use_buf ? 1 : 0, nesterov ? 1 : 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool v4 = aligned16(param) && aligned16(grad) && (!use_buf || aligned16(velocity));
  if (v4)
    sgd_kernel<true><<<elem_grid(n / 4 + 1), 256, 0, s>>>(param, grad, velocity, n, c);
  else
    sgd_kernel<false><<<elem_grid(n), 256, 0, s>>>(param, grad, velocity, n, c);
  return check_launch("oxc_sgd_step");
}

oxc_status oxc_adamw_step(float* param, const float* grad, float* m, float* v, int64_t n,
                          float lr, float beta1, float beta2, float eps, float weight_decay,
                          int32_t decoupled, int64_t step, void* stream) {
  if (n < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: adam step: negative size");
  if (step < 1)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: adam step counter %lld (from 1)",
                (long long)step);
  if (n == 0) return OXC_OK;
  if (!param || !grad || !m || !v)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: adam step: null pointer");
  AdamConst c;
  c.lr = lr;
  c.beta1 = beta1;
  c.beta2 = beta2;
  c.omb1 = 1.0f - beta1;
  c.omb2 = 1.0f - beta2;
  c.eps = eps;
  c.wd = weight_decay;
  // optim.rs:232-233: 1 - beta^(t as f32), f32 powf
  c.bc1 = 1.0f - powf(beta1, (float)step);
  c.bc2 = 1.0f - powf(beta2, (float)step);
  c.decay_grad = (!decoupled && weight_decay != 0.0f) ? 1 : 0;
  c.decay_param = (decoupled && weight_decay != 0.0f) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool v4 = aligned16(param) && aligned16(grad) && aligned16(m) && aligned16(v);
  if (v4)
    adam_kernel<true><<<elem_grid(n / 4 + 1), 256, 0, s>>>(param, grad, m, v, n, c);
  else
    adam_kernel<false><<<elem_grid(n), 256, 0, s>>>(param, grad, m, v, n, c);
  return check_launch("oxc_adamw_step");
}

oxc_status oxc_clip_grad_value(float* grad, int64_t n, float clip_value, void* stream) {
  // The reference checks the Python float (<= 0 raises) before NumPy rounds
  // it to f32; here only a negative f32 bound is refused, so a positive bound
  // that rounds to 0 clamps to +-0 as np.clip does, and a NaN bound gives NaN.
  if (clip_value < 0.0f) return fail(OXC_ERR_INVALID_ARGUMENT, "clip_value must be positive");
  if (n < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: clip_grad_value_: negative size");
  if (n == 0) return OXC_OK;
  if (!grad) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: clip_grad_value_: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (aligned16(grad))
    clip_value_kernel<true><<<elem_grid(n / 4 + 1), 256, 0, s>>>(grad, n, -clip_value, clip_value);
  else
    clip_value_kernel<false><<<elem_grid(n), 256, 0, s>>>(grad, n, -clip_value, clip_value);
  return check_launch("oxc_clip_grad_value");
}

}  // extern "C"
