// gelu.cuh -- the reference's tanh-form GELU and its derivative, shared by the
// fused LayerNorm+GELU kernels and the standalone activation kernels.
//
// Reference (python/oxitorch/nn/functional.py:194-199):
//   out = (x*0.5) * (tanh((x + x*x*x*0.044715) * C) + 1),  C = float(sqrt(2/pi))
#pragma once

#include <math.h>

#include "common.cuh"

namespace oxc {

struct GeluConst {
  float k;   // 0.044715 as f32
  float k3;  // 3 * k
  float c2;  // 2 * c, c = sqrt(2/pi) rounded to f32
  float e2;  // -2 * c * log2(e): e^(-2 c v) = 2^(v * e2)
};

// The reference's GELU, 0.5*y*(1 + tanh(c*v)) with v = y + k*y^3, evaluated
// through the logistic form of tanh:
//   (1 + tanh(c v)) / 2 = s = 1 / (1 + E),   E = e^(-2 c v),
// so gelu(y) = y * s and, with 1 - s = E * s and sech^2 = 4 s (1 - s),
//   gelu'(y) = s + 2 y s (1 - s) * c (1 + 3 k y^2).
// E comes from ex2.approx (relative error about 2^-22) and s from rcp.approx
// (1 ulp), so s carries a few ulp of relative error for every v.  The direct
// form loses relative accuracy where 1 + tanh and 1 - tanh^2 cancel (c v far
// below 0, and |c v| large for the derivative); this one has no cancellation,
// and it needs two MUFU operations where tanhf needs a longer sequence.
// Limits: v = +inf gives E = 0, s = 1; v = -inf gives E = inf, s = 0, and
// 1 - s is taken as min(E * s, 1) so inf * 0 does not make it NaN.
__device__ __forceinline__ float ex2_approx(float a) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}
__device__ __forceinline__ float rcp_approx(float a) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

__device__ __forceinline__ float gelu_fwd(float y, const GeluConst& gc) {
  const float v = fmaf(gc.k * (y * y), y, y);  // y + k*y^3
  return y * rcp_approx(1.0f + ex2_approx(v * gc.e2));
}

// g * d gelu / d y at y.
__device__ __forceinline__ float gelu_grad(float y, float g, const GeluConst& gc) {
  const float y2 = y * y;
  const float v = fmaf(gc.k * y2, y, y);
  const float E = ex2_approx(v * gc.e2);
  const float s = rcp_approx(1.0f + E);
  const float oms = fminf(E * s, 1.0f);                // 1 - s
  const float dv = gc.c2 * fmaf(gc.k3, y2, 1.0f);      // 2 * d(c v)/dy
  return g * fmaf(y * s * oms, dv, s);
}

// gelu_grad for two lanes at once on the packed f32x2 pipe of sm_100
// (__ffma2_rn / __fadd2_rn / __fmul2_rn round each lane exactly like the
// scalar fmaf / __fadd_rn / __fmul_rn).  The operations and their order are
// those of gelu_grad, which has no multiply-add pair the compiler could
// contract, so both forms give the same bits; this one issues half the FP
// instructions (the two MUFU operations and the clamp stay per lane).
__device__ __forceinline__ float2 bcast2(float a) { return make_float2(a, a); }

__device__ __forceinline__ float2 gelu_grad2(float2 y, float2 g, const GeluConst& gc) {
  const float2 y2 = __fmul2_rn(y, y);
  const float2 v = __ffma2_rn(__fmul2_rn(bcast2(gc.k), y2), y, y);
  const float2 t = __fmul2_rn(v, bcast2(gc.e2));
  const float2 E = make_float2(ex2_approx(t.x), ex2_approx(t.y));
  const float2 d = __fadd2_rn(bcast2(1.0f), E);
  const float2 s = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  const float2 es = __fmul2_rn(E, s);
  const float2 oms = make_float2(fminf(es.x, 1.0f), fminf(es.y, 1.0f));
  const float2 dv = __fmul2_rn(bcast2(gc.c2), __ffma2_rn(bcast2(gc.k3), y2, bcast2(1.0f)));
  const float2 q = __fmul2_rn(__fmul2_rn(y, s), oms);
  return __fmul2_rn(g, __ffma2_rn(q, dv, s));
}

// The constants as f32, computed on the host once per launch.
inline GeluConst gelu_const() {
  GeluConst gc;
  gc.k = (float)0.044715;
  gc.k3 = 3.0f * gc.k;
  const float c = (float)sqrt(2.0 / M_PI);
  gc.c2 = 2.0f * c;
  gc.e2 = (float)(-2.0 * (double)c * M_LOG2E);
  return gc;
}

}  // namespace oxc
