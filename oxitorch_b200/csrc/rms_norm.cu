// rms_norm.cu -- F.rms_norm forward and its VJP (python/oxitorch/nn/functional.py:236-240).
//
// Reference composition: ms = (x*x).mean(-1, keepdim); inv = (ms + eps).apply("rsqrt");
// y = x * inv * weight.  The forward reproduces that rounding sequence
// (x*x, sum, /cols, +eps, 1/sqrt, *inv, *w) with a fixed-order tree for the
// row sum instead of the reference's left-to-right fold.
//
// VJP (OXC_GRAD_REF): "rsqrt" is outside the differentiable apply whitelist
// (crates/oxi-bindings/src/lib.rs:682-697), so inv is a constant and
//   dx = (dy * w) * inv                         (autograd/ops.rs:62-73, twice)
//   dw = sum_rows dy * (x * inv)                (unbroadcast, graph.rs:274-313)
// OXC_GRAD_EXACT adds the derivative through inv:
//   dx = inv*g - x * inv^3 * mean_row(g*x),  g = dy*w.
//
// Bytes per row (fp32): fwd reads x, writes y (+4 B rstd); VJP reads x, dy,
// writes dx.  Both are HBM-bound; the VJP keeps the column accumulators for
// dw in registers across the rows of a persistent CTA and finishes them with
// one deterministic column sum over the per-CTA partials.
#include <algorithm>

#include "rowvec.cuh"

namespace oxc {

template <int VW, int VPT, int MAXT>
__global__ void __launch_bounds__(MAXT) rms_fwd_kernel(const float* __restrict__ x,
                                                       const float* __restrict__ w,
                                                       float* __restrict__ y,
                                                       float* __restrict__ rstd, int64_t rows,
                                                       int cols, float eps) {
  __shared__ float scratch[33];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * (int64_t)cols;
    float v[VPT][VW];
    float ss = 0.0f;
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
      for (int k = 0; k < VW; ++k) ss = __fadd_rn(ss, __fmul_rn(v[i][k], v[i][k]));
    ss = block_sum(ss, scratch);
    const float ms = __fdiv_rn(ss, (float)cols);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    float* yr = y + row * (int64_t)cols;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * blockDim.x + threadIdx.x) * VW;
      if (e < cols) {
        float wv[VW], o[VW];
        load_vec<VW>(wv, w + e, false);
#pragma unroll
        for (int k = 0; k < VW; ++k) o[k] = __fmul_rn(__fmul_rn(v[i][k], inv), wv[k]);
        store_vec<VW>(yr + e, o);
      }
    }
    if (threadIdx.x == 0) rstd[row] = inv;
  }
}

// Persistent VJP: CTA b handles rows [b*chunk, min((b+1)*chunk, rows)) and
// writes its dw partial to parts[b][cols].
template <int VW, int VPT, int MAXT, int MODE>
__global__ void __launch_bounds__(MAXT) rms_bwd_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ rstd,
    const float* __restrict__ dy, float* __restrict__ dx, float* __restrict__ parts, int64_t rows,
    int cols, int64_t chunk) {
  pdl_launch_dependents();  // the dweight finisher waits for this grid
  __shared__ float scratch[33];
  const int64_t r0 = (int64_t)blockIdx.x * chunk;
  const int64_t r1 = min(rows, r0 + chunk);
  float wv[VPT][VW], acc[VPT][VW];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int e = (i * blockDim.x + threadIdx.x) * VW;
#pragma unroll
    for (int k = 0; k < VW; ++k) acc[i][k] = 0.0f;
    if (e < cols) {
      load_vec<VW>(wv[i], w + e, false);
    } else {
#pragma unroll
      for (int k = 0; k < VW; ++k) wv[i][k] = 0.0f;
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
    const float inv = __ldg(rstd + row);
    // dw partial: acc += dy * (x*inv)
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int k = 0; k < VW; ++k)
        acc[i][k] = __fadd_rn(acc[i][k], __fmul_rn(gv[i][k], __fmul_rn(xv[i][k], inv)));
    float corr = 0.0f;
    if constexpr (MODE == OXC_GRAD_EXACT) {
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
#pragma unroll
        for (int k = 0; k < VW; ++k)
          s = __fadd_rn(s, __fmul_rn(__fmul_rn(gv[i][k], wv[i][k]), xv[i][k]));
      s = block_sum(s, scratch);
      // inv^3 * mean(g*x)
      corr = __fmul_rn(__fmul_rn(__fmul_rn(inv, inv), inv), __fmul_rn(s, inv_n));
    }
    float* dxr = dx + row * (int64_t)cols;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * blockDim.x + threadIdx.x) * VW;
      if (e < cols) {
        float o[VW];
#pragma unroll
        for (int k = 0; k < VW; ++k) {
          o[k] = __fmul_rn(__fmul_rn(gv[i][k], wv[i][k]), inv);
          if constexpr (MODE == OXC_GRAD_EXACT) o[k] = __fsub_rn(o[k], __fmul_rn(xv[i][k], corr));
        }
        store_vec<VW>(dxr + e, o);
      }
    }
  }
  float* pr = parts + (int64_t)blockIdx.x * cols;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int e = (i * blockDim.x + threadIdx.x) * VW;
    if (e < cols) {
#pragma unroll
      for (int k = 0; k < VW; ++k) pr[e + k] = acc[i][k];
    }
  }
}

// The REF-mode VJP as a streaming tile kernel.  With the rsqrt factor
// detached, dx = (dy*w)*inv needs no row reduction, so a CTA takes a stripe of
// blockDim.x float4 columns (blockIdx.x) over a block of rows (blockIdx.y):
// every thread keeps U rows of x and dy loads in flight, streams dx out and
// carries the dw partial of its four columns in registers; parts[blockIdx.y]
// holds the stripe's partial, summed by the column finisher.  The same
// per-element operations as rms_bwd_kernel; only the grouping of the dw sums
// differs.
template <int U>
__global__ void __launch_bounds__(256) rms_bwd_stream_kernel(
    const float4* __restrict__ x, const float4* __restrict__ w, const float* __restrict__ rstd,
    const float4* __restrict__ dy, float4* __restrict__ dx, float4* __restrict__ parts,
    int64_t rows, int64_t cols4, int64_t rows_per_cta) {
  pdl_launch_dependents();  // the dweight finisher waits for this grid
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols4) return;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_cta;
  const int64_t r1 = min(rows, r0 + rows_per_cta);
  const float4 wv = __ldg(w + c);
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int64_t r = r0; r < r1; r += U) {
    float4 xv[U], gv[U];
    float inv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (r + u < r1) {
        xv[u] = ld_stream(x + (r + u) * cols4 + c);
        gv[u] = ld_stream(dy + (r + u) * cols4 + c);
        inv[u] = __ldg(rstd + r + u);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (r + u < r1) {
        const float i = inv[u];
        acc.x = __fadd_rn(acc.x, __fmul_rn(gv[u].x, __fmul_rn(xv[u].x, i)));
        acc.y = __fadd_rn(acc.y, __fmul_rn(gv[u].y, __fmul_rn(xv[u].y, i)));
        acc.z = __fadd_rn(acc.z, __fmul_rn(gv[u].z, __fmul_rn(xv[u].z, i)));
        acc.w = __fadd_rn(acc.w, __fmul_rn(gv[u].w, __fmul_rn(xv[u].w, i)));
        float4 o;
        o.x = __fmul_rn(__fmul_rn(gv[u].x, wv.x), i);
        o.y = __fmul_rn(__fmul_rn(gv[u].y, wv.y), i);
        o.z = __fmul_rn(__fmul_rn(gv[u].z, wv.z), i);
        o.w = __fmul_rn(__fmul_rn(gv[u].w, wv.w), i);
        st_stream(dx + (r + u) * cols4 + c, o);
      }
    }
  }
  parts[(int64_t)blockIdx.y * cols4 + c] = acc;
}

constexpr int kRmsStreamThreads = 256;
constexpr int kRmsStreamU = 4;

// Number of persistent CTAs of the VJP: two per SM, at least 8 rows each.
static int64_t rms_bwd_ctas(int64_t rows) {
  int64_t g = 2 * (int64_t)sm_count();
  const int64_t by_rows = (rows + 7) / 8;
  if (g > by_rows) g = by_rows;
  return g < 1 ? 1 : g;
}

static oxc_status check_rows(const char* fn, int64_t rows, int64_t cols) {
  if (rows < 0 || cols < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative shape [%lld, %lld]", fn,
                (long long)rows, (long long)cols);
  if (cols > 32768)
    return fail(OXC_ERR_NOT_IMPLEMENTED,
                "not implemented: %s: rows wider than 32768 elements are not supported", fn);
  return OXC_OK;
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_rms_norm_fwd(const float* x, const float* w, float* y, float* rstd, int64_t rows,
                            int64_t cols, float eps, void* stream) {
  oxc_status st = check_rows("rms_norm", rows, cols);
  if (st) return st;
  if (rows == 0) return OXC_OK;
  if (cols == 0) {
    // mean over an empty dim is NaN (0/0); y is empty.
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: rms_norm over a zero-length dim");
  }
  if (!x || !w || !y || !rstd)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: rms_norm: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool v4 = cols % 4 == 0 && aligned16(x) && aligned16(w) && aligned16(y);
  // float4 rows: 8 vectors per thread where the row allows (on B200, 3% over
  // 256 threads x 4 vectors at [16384, 4096])
  RowGeom g = row_geom(cols, v4);
  if (v4) {
    const RowGeom d = row_geom_deep(cols);
    if (d.ok && d.block <= 512) g = d;
  }
  const unsigned grid = (unsigned)(rows < 0x7fffffff ? rows : 0x7fffffff);
#define LAUNCH(VW, VPT, MAXT) \
  rms_fwd_kernel<VW, VPT, MAXT><<<grid, g.block, 0, s>>>(x, w, y, rstd, rows, (int)cols, eps)
  OXC_DISPATCH_ROW(g, LAUNCH);
#undef LAUNCH
  return check_launch("oxc_rms_norm_fwd");
}

size_t oxc_rms_norm_bwd_workspace_size(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return (size_t)rms_bwd_ctas(rows) * (size_t)cols * sizeof(float);
}

oxc_status oxc_rms_norm_bwd(const float* x, const float* w, const float* rstd, const float* dy,
                            float* dx, float* dw, int64_t rows, int64_t cols, int32_t grad_mode,
                            void* workspace, size_t workspace_bytes, void* stream) {
  oxc_status st = check_rows("rms_norm backward", rows, cols);
  if (st) return st;
  if (grad_mode != OXC_GRAD_REF && grad_mode != OXC_GRAD_EXACT)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown grad mode %d", grad_mode);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cols == 0) return OXC_OK;
  if (rows == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, (size_t)cols * sizeof(float), s);
    return e == cudaSuccess ? OXC_OK : cuda_fail(e, "oxc_rms_norm_bwd");
  }
  const size_t need = oxc_rms_norm_bwd_workspace_size(rows, cols);
  if (!workspace || workspace_bytes < need)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: rms_norm backward needs a %zu-byte workspace, got %zu", need,
                workspace_bytes);
  if (!x || !w || !rstd || !dy || !dx || !dw)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: rms_norm backward: null pointer");
  const bool v4 = cols % 4 == 0 && aligned16(x) && aligned16(w) && aligned16(dy) &&
                  aligned16(dx) && aligned16(workspace);
  float* parts = static_cast<float*>(workspace);
  if (v4 && grad_mode == OXC_GRAD_REF) {
    // streaming tile kernel: one wave of resident CTAs, the row blocks no more
    // than the workspace's partial slots (rms_bwd_ctas)
    const int64_t cols4 = cols / 4;
    const int64_t gx = (cols4 + kRmsStreamThreads - 1) / kRmsStreamThreads;
    const int block = (int)std::min<int64_t>(kRmsStreamThreads, ((cols4 + 31) / 32) * 32);
    const int64_t resident =
        (int64_t)sm_count() * occupancy((const void*)rms_bwd_stream_kernel<kRmsStreamU>, block, 0);
    int64_t gy = std::max<int64_t>(1, resident / gx);
    gy = std::min<int64_t>(gy, rms_bwd_ctas(rows));
    const int64_t per = (rows + gy - 1) / gy;
    gy = (rows + per - 1) / per;
    if (gy > 65535 || (size_t)gy * cols * sizeof(float) > workspace_bytes)
      return fail(OXC_ERR_OTHER, "internal: rms_norm backward partials exceed the workspace");
    rms_bwd_stream_kernel<kRmsStreamU><<<dim3((unsigned)gx, (unsigned)gy), block, 0, s>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<const float4*>(w), rstd,
        reinterpret_cast<const float4*>(dy), reinterpret_cast<float4*>(dx),
        reinterpret_cast<float4*>(parts), rows, cols4, per);
    st = check_launch("oxc_rms_norm_bwd");
    if (st) return st;
    launch_colsum_partials(parts, (int)gy, cols, dw, s);
    return check_launch("oxc_rms_norm_bwd (dw)");
  }
  RowGeom g = row_geom(cols, v4, 512);
  const int64_t ctas = rms_bwd_ctas(rows);
  const int64_t chunk = (rows + ctas - 1) / ctas;
#define LAUNCH(VW, VPT, MAXT)                                                                \
  do {                                                                                       \
    if (grad_mode == OXC_GRAD_REF)                                                           \
      rms_bwd_kernel<VW, VPT, MAXT, OXC_GRAD_REF><<<(unsigned)ctas, g.block, 0, s>>>(        \
          x, w, rstd, dy, dx, parts, rows, (int)cols, chunk);                                \
    else                                                                                     \
      rms_bwd_kernel<VW, VPT, MAXT, OXC_GRAD_EXACT><<<(unsigned)ctas, g.block, 0, s>>>(      \
          x, w, rstd, dy, dx, parts, rows, (int)cols, chunk);                                \
  } while (0)
  OXC_DISPATCH_ROW(g, LAUNCH);
#undef LAUNCH
  st = check_launch("oxc_rms_norm_bwd");
  if (st) return st;
  launch_colsum_partials(parts, (int)ctas, cols, dw, s);
  return check_launch("oxc_rms_norm_bwd (dw)");
}

}  // extern "C"
