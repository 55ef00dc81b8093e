// layer_norm.cu -- F.layer_norm (+ F.gelu fused) forward and VJP.
//
// Reference (python/oxitorch/nn/functional.py:227-233, 194-199):
//   mu = x.mean(-1, True); c = x - mu; var = (c*c).mean(-1, True)
//   inv = (var + eps).apply("rsqrt")             -- detached (bindings lib.rs:682-697)
//   yln = c * inv * weight + bias
//   gelu: x32 = y*y; inner = (y + y*x32*0.044715) * C; out = (y*0.5) * (tanh(inner) + 1)
//   with C = float(sqrt(2/pi)) computed in f64 and rounded to f32 at the boundary.
// Every elementwise step below is the same f32 operation in the same order as
// that composition; only the two row sums use a fixed-order tree.
//
// VJP (OXC_GRAD_REF, the reference graph):
//   g    = dL/d(yln): the composed GELU VJP; its five contributions are added
//          in the order the reference's backward visits them (graph.rs:324-438):
//          (a-path, u, p, x32 first input, x32 second input)
//   dw  += g * (c*inv)     db += g            (unbroadcast sums, graph.rs:274-313)
//   gc   = (g*w) * inv
//   dx   = gc + (-(sum_row gc)) * (1/cols)    (sub and mean VJPs, autograd/ops.rs:49-56, 340-349)
// OXC_GRAD_EXACT: dx = inv * (gw - mean(gw) - xhat*mean(gw*xhat)), gw = g*w.
#include <math.h>

#include "rowvec.cuh"

namespace oxc {

struct GeluConst {
  float k;  // 0.044715 as f32
  float c;  // sqrt(2/pi) rounded to f32
};

__device__ __forceinline__ float gelu_fwd(float y, const GeluConst& gc) {
  const float x32 = __fmul_rn(y, y);
  const float p = __fmul_rn(y, x32);
  const float q = __fmul_rn(p, gc.k);
  const float u = __fadd_rn(y, q);
  const float inner = __fmul_rn(u, gc.c);
  const float th = tanhf(inner);
  const float a = __fmul_rn(y, 0.5f);
  const float bb = __fadd_rn(th, 1.0f);
  return __fmul_rn(a, bb);
}

// d out / d y times g, as the reference's graph computes it.
__device__ __forceinline__ float gelu_vjp(float y, float g, const GeluConst& gc) {
  const float x32 = __fmul_rn(y, y);
  const float p = __fmul_rn(y, x32);
  const float q = __fmul_rn(p, gc.k);
  const float u = __fadd_rn(y, q);
  const float inner = __fmul_rn(u, gc.c);
  const float th = tanhf(inner);
  const float a = __fmul_rn(y, 0.5f);
  const float bb = __fadd_rn(th, 1.0f);
  const float g_a = __fmul_rn(g, bb);
  const float g_bb = __fmul_rn(g, a);
  const float d = __fsub_rn(1.0f, __fmul_rn(th, th));
  const float g_inner = __fmul_rn(g_bb, d);
  const float g_u = __fmul_rn(g_inner, gc.c);
  const float g_p = __fmul_rn(g_u, gc.k);
  const float g_x32 = __fmul_rn(g_p, y);
  float r = __fmul_rn(g_a, 0.5f);
  r = __fadd_rn(r, g_u);
  r = __fadd_rn(r, __fmul_rn(g_p, x32));
  const float t = __fmul_rn(g_x32, y);
  r = __fadd_rn(r, t);
  r = __fadd_rn(r, t);
  return r;
}

template <int VW, int VPT, int MAXT, int ACT>
__global__ void __launch_bounds__(MAXT) ln_fwd_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
    float* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
    int64_t rows, int cols, float eps, GeluConst gc) {
  __shared__ float scratch[33];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * (int64_t)cols;
    float v[VPT][VW];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * blockDim.x + threadIdx.x) * VW;
      if (e < cols) {
        load_vec<VW>(v[i], xr + e, true);
      } else {
#pragma unroll
        for (int k = 0; k < VW; ++k) v[i][k] = 0.0f;
      }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int k = 0; k < VW; ++k) s = __fadd_rn(s, v[i][k]);
    s = block_sum(s, scratch);
    const float mu = __fdiv_rn(s, (float)cols);
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * blockDim.x + threadIdx.x) * VW;
#pragma unroll
      for (int k = 0; k < VW; ++k) {
        v[i][k] = __fsub_rn(v[i][k], mu);
        if (e < cols) ss = __fadd_rn(ss, __fmul_rn(v[i][k], v[i][k]));
      }
    }
    ss = block_sum(ss, scratch);
    const float var = __fdiv_rn(ss, (float)cols);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    float* yr = y + row * (int64_t)cols;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * blockDim.x + threadIdx.x) * VW;
      if (e < cols) {
        float wv[VW], bv[VW], o[VW];
        load_vec<VW>(wv, w + e, false);
        load_vec<VW>(bv, b + e, false);
#pragma unroll
        for (int k = 0; k < VW; ++k) {
          const float yl = __fadd_rn(__fmul_rn(__fmul_rn(v[i][k], inv), wv[k]), bv[k]);
          o[k] = ACT == OXC_ACT_GELU_TANH ? gelu_fwd(yl, gc) : yl;
        }
        store_vec<VW>(yr + e, o);
      }
    }
    if (threadIdx.x == 0) {
      mean_out[row] = mu;
      rstd_out[row] = inv;
    }
  }
}

// Persistent VJP; CTA b owns rows [b*chunk, ...) and writes dw/db partials to
// parts[b][cols] and parts[nctas + b][cols].
template <int VW, int VPT, int MAXT, int ACT, int MODE>
__global__ void __launch_bounds__(MAXT) ln_bwd_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
    const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
    const float* __restrict__ dy, float* __restrict__ dx, float* __restrict__ parts,
    int64_t rows, int cols, int64_t chunk, GeluConst gc) {
  __shared__ float scratch[33];
  const int64_t r0 = (int64_t)blockIdx.x * chunk;
  const int64_t r1 = min(rows, r0 + chunk);
  float wv[VPT][VW], bv[VPT][VW], adw[VPT][VW], adb[VPT][VW];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int e = (i * blockDim.x + threadIdx.x) * VW;
#pragma unroll
    for (int k = 0; k < VW; ++k) { adw[i][k] = 0.0f; adb[i][k] = 0.0f; }
    if (e < cols) {
      load_vec<VW>(wv[i], w + e, false);
      load_vec<VW>(bv[i], b + e, false);
    } else {
#pragma unroll
      for (int k = 0; k < VW; ++k) { wv[i][k] = 0.0f; bv[i][k] = 0.0f; }
    }
  }
  const float inv_n = __fdiv_rn(1.0f, (float)cols);
  for (int64_t row = r0; row < r1; ++row) {
    const float* xr = x + row * (int64_t)cols;
    const float* gr = dy + row * (int64_t)cols;
    float xv[VPT][VW], gv[VPT][VW];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * blockDim.x + threadIdx.x) * VW;
      if (e < cols) {
        load_vec<VW>(xv[i], xr + e, true);
        load_vec<VW>(gv[i], gr + e, true);
      } else {
#pragma unroll
        for (int k = 0; k < VW; ++k) { xv[i][k] = 0.0f; gv[i][k] = 0.0f; }
      }
    }
    const float mu = __ldg(mean_in + row);
    const float inv = __ldg(rstd_in + row);
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * blockDim.x + threadIdx.x) * VW;
#pragma unroll
      for (int k = 0; k < VW; ++k) {
        const float t1 = __fmul_rn(__fsub_rn(xv[i][k], mu), inv);  // c*inv
        float g = gv[i][k];
        if constexpr (ACT == OXC_ACT_GELU_TANH) {
          const float yl = __fadd_rn(__fmul_rn(t1, wv[i][k]), bv[i][k]);
          g = gelu_vjp(yl, g, gc);
        }
        if (e < cols) {
          adw[i][k] = __fadd_rn(adw[i][k], __fmul_rn(g, t1));
          adb[i][k] = __fadd_rn(adb[i][k], g);
        }
        const float gw = __fmul_rn(g, wv[i][k]);
        if constexpr (MODE == OXC_GRAD_REF) {
          const float gcv = __fmul_rn(gw, inv);
          gv[i][k] = gcv;
          if (e < cols) s1 = __fadd_rn(s1, gcv);
        } else {
          gv[i][k] = gw;
          xv[i][k] = t1;  // xhat
          if (e < cols) {
            s1 = __fadd_rn(s1, gw);
            s2 = __fadd_rn(s2, __fmul_rn(gw, t1));
          }
        }
      }
    }
    s1 = block_sum(s1, scratch);
    if constexpr (MODE == OXC_GRAD_EXACT) s2 = block_sum(s2, scratch);
    float* dxr = dx + row * (int64_t)cols;
    const float gmu = -s1;  // sum(-gc) == -(sum gc) exactly
    const float m1 = __fmul_rn(s1, inv_n), m2 = __fmul_rn(s2, inv_n);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * blockDim.x + threadIdx.x) * VW;
      if (e < cols) {
        float o[VW];
#pragma unroll
        for (int k = 0; k < VW; ++k) {
          if constexpr (MODE == OXC_GRAD_REF) {
            o[k] = __fadd_rn(gv[i][k], __fmul_rn(gmu, inv_n));
          } else {
            o[k] = __fmul_rn(inv, __fsub_rn(__fsub_rn(gv[i][k], m1), __fmul_rn(xv[i][k], m2)));
          }
        }
        store_vec<VW>(dxr + e, o);
      }
    }
  }
  float* pw = parts + (int64_t)blockIdx.x * cols;
  float* pb = parts + ((int64_t)gridDim.x + blockIdx.x) * cols;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int e = (i * blockDim.x + threadIdx.x) * VW;
    if (e < cols) {
#pragma unroll
      for (int k = 0; k < VW; ++k) { pw[e + k] = adw[i][k]; pb[e + k] = adb[i][k]; }
    }
  }
}

static int64_t ln_bwd_ctas(int64_t rows) {
  int64_t g = 2 * (int64_t)sm_count();
  const int64_t by_rows = (rows + 7) / 8;
  if (g > by_rows) g = by_rows;
  return g < 1 ? 1 : g;
}

static GeluConst gelu_const() {
  GeluConst gc;
  gc.k = (float)0.044715;
  gc.c = (float)sqrt(2.0 / M_PI);
  return gc;
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_layer_norm_fwd(const float* x, const float* w, const float* b, float* y,
                              float* mean, float* rstd, int64_t rows, int64_t cols, float eps,
                              int32_t act, void* stream) {
  if (rows < 0 || cols < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: layer_norm: negative shape");
  if (act != OXC_ACT_NONE && act != OXC_ACT_GELU_TANH)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown activation %d", act);
  if (cols > 32768)
    return fail(OXC_ERR_NOT_IMPLEMENTED,
                "not implemented: layer_norm: rows wider than 32768 elements are not supported");
  if (rows == 0) return OXC_OK;
  if (cols == 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: layer_norm over a zero-length dim");
  if (!x || !w || !b || !y || !mean || !rstd)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: layer_norm: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool v4 = cols % 4 == 0 && aligned16(x) && aligned16(w) && aligned16(b) && aligned16(y);
  RowGeom g = row_geom(cols, v4);
  const unsigned grid = (unsigned)(rows < 0x7fffffff ? rows : 0x7fffffff);
  const GeluConst gc = gelu_const();
#define LAUNCH(VW, VPT, MAXT)                                                            \
  do {                                                                                   \
    if (act == OXC_ACT_GELU_TANH)                                                        \
      ln_fwd_kernel<VW, VPT, MAXT, OXC_ACT_GELU_TANH>                                    \
          <<<grid, g.block, 0, s>>>(x, w, b, y, mean, rstd, rows, (int)cols, eps, gc);   \
    else                                                                                 \
      ln_fwd_kernel<VW, VPT, MAXT, OXC_ACT_NONE>                                         \
          <<<grid, g.block, 0, s>>>(x, w, b, y, mean, rstd, rows, (int)cols, eps, gc);   \
  } while (0)
  OXC_DISPATCH_ROW(g, LAUNCH);
#undef LAUNCH
  return check_launch("oxc_layer_norm_fwd");
}

size_t oxc_layer_norm_bwd_workspace_size(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return 2 * (size_t)ln_bwd_ctas(rows) * (size_t)cols * sizeof(float);
}

oxc_status oxc_layer_norm_bwd(const float* x, const float* w, const float* b, const float* mean,
                              const float* rstd, const float* dy, float* dx, float* dw, float* db,
                              int64_t rows, int64_t cols, int32_t act, int32_t grad_mode,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (rows < 0 || cols < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: layer_norm backward: negative shape");
  if (act != OXC_ACT_NONE && act != OXC_ACT_GELU_TANH)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown activation %d", act);
  if (grad_mode != OXC_GRAD_REF && grad_mode != OXC_GRAD_EXACT)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown grad mode %d", grad_mode);
  if (cols > 32768)
    return fail(OXC_ERR_NOT_IMPLEMENTED,
                "not implemented: layer_norm: rows wider than 32768 elements are not supported");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cols == 0) return OXC_OK;
  if (rows == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, (size_t)cols * sizeof(float), s);
    if (e == cudaSuccess) e = cudaMemsetAsync(db, 0, (size_t)cols * sizeof(float), s);
    return e == cudaSuccess ? OXC_OK : cuda_fail(e, "oxc_layer_norm_bwd");
  }
  const size_t need = oxc_layer_norm_bwd_workspace_size(rows, cols);
  if (!workspace || workspace_bytes < need)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: layer_norm backward needs a %zu-byte workspace, got %zu", need,
                workspace_bytes);
  if (!x || !w || !b || !mean || !rstd || !dy || !dx || !dw || !db)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: layer_norm backward: null pointer");
  const bool v4 = cols % 4 == 0 && aligned16(x) && aligned16(w) && aligned16(b) &&
                  aligned16(dy) && aligned16(dx) && aligned16(workspace);
  RowGeom g = row_geom(cols, v4, 512);
  const int64_t ctas = ln_bwd_ctas(rows);
  const int64_t chunk = (rows + ctas - 1) / ctas;
  float* parts = static_cast<float*>(workspace);
  const GeluConst gc = gelu_const();
#define LAUNCH_M(VW, VPT, MAXT, ACT, MODE)                                              \
  ln_bwd_kernel<VW, VPT, MAXT, ACT, MODE><<<(unsigned)ctas, g.block, 0, s>>>(           \
      x, w, b, mean, rstd, dy, dx, parts, rows, (int)cols, chunk, gc)
#define LAUNCH(VW, VPT, MAXT)                                                           \
  do {                                                                                  \
    if (act == OXC_ACT_GELU_TANH) {                                                     \
      if (grad_mode == OXC_GRAD_REF) LAUNCH_M(VW, VPT, MAXT, OXC_ACT_GELU_TANH, OXC_GRAD_REF); \
      else LAUNCH_M(VW, VPT, MAXT, OXC_ACT_GELU_TANH, OXC_GRAD_EXACT);                   \
    } else {                                                                            \
      if (grad_mode == OXC_GRAD_REF) LAUNCH_M(VW, VPT, MAXT, OXC_ACT_NONE, OXC_GRAD_REF); \
      else LAUNCH_M(VW, VPT, MAXT, OXC_ACT_NONE, OXC_GRAD_EXACT);                       \
    }                                                                                   \
  } while (0)
  OXC_DISPATCH_ROW(g, LAUNCH);
#undef LAUNCH
#undef LAUNCH_M
  oxc_status st = check_launch("oxc_layer_norm_bwd");
  if (st) return st;
  launch_colsum_partials(parts, (int)ctas, cols, dw, s);
  launch_colsum_partials(parts + ctas * cols, (int)ctas, cols, db, s);
  return check_launch("oxc_layer_norm_bwd (dw, db)");
}

}  // extern "C"
