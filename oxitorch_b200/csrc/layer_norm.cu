// layer_norm.cu -- F.layer_norm (+ F.gelu fused) forward and VJP.
//
// Reference (python/oxitorch/nn/functional.py:227-233, 194-199):
//   mu = x.mean(-1, True); c = x - mu; var = (c*c).mean(-1, True)
//   inv = (var + eps).apply("rsqrt")             -- detached (bindings lib.rs:682-697)
//   yln = c * inv * weight + bias
//   gelu: out = (y*0.5) * (tanh((y + y*y*y*0.044715) * C) + 1),  C = float(sqrt(2/pi))
//
// VJP (OXC_GRAD_REF, the reference graph, autograd/ops.rs):
//   g    = dL/d(yln) = dy * gelu'(yln)   (the reference accumulates the same
//          derivative from five graph contributions; here it is one FMA chain)
//   dw  += g * (c*inv)     db += g            (unbroadcast sums, graph.rs:274-313)
//   gc   = (g*w) * inv
//   dx   = gc - (sum_row gc) / cols            (sub and mean VJPs, ops.rs:49-56, 340-349)
// OXC_GRAD_EXACT: dx = inv * (gw - mean(gw) - xhat*mean(gw*xhat)), gw = g*w.
//
// Kernels:
//   ln_fwd_kernel: any width up to 32768, register-resident rows, plain loads;
//     mean and variance from one block reduction (a shifted one-pass sum,
//     corrected by a second pass when the shift was poor).  Aligned float4
//     rows of up to 16384 columns run it persistent with the next row
//     prefetched and 8 vectors per thread where the row allows (row_geom_deep).
//   ln_bwd_pipe_kernel: the VJP for rows with cols % 4 == 0 and 16-byte
//     aligned tensors.  One persistent CTA per SM; a producer warp streams
//     whole rows into a shared-memory ring with bulk copies (pipeline.cuh)
//     while 16 consumer warps compute, so HBM stays busy during the arithmetic.
//   ln_bwd_kernel: the VJP for other rows, register-resident.
#include <math.h>

#include <algorithm>

#include "gelu.cuh"
#include "pipeline.cuh"
#include "rowvec.cuh"

namespace oxc {

// Block-wide sums of two values; every thread gets both.  Fixed order: the
// warp butterfly, then each thread adds the per-warp partials in warp order.
// scratch: >= 64 floats.
__device__ __forceinline__ float2 block_sum2(float a, float b, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  __syncthreads();  // earlier readers of scratch are done
  if (lane == 0) {
    scratch[warp] = a;
    scratch[32 + warp] = b;
  }
  __syncthreads();
  float2 t = make_float2(0.0f, 0.0f);
  for (int w = 0; w < nw; ++w) {
    t.x += scratch[w];
    t.y += scratch[32 + w];
  }
  return t;
}

// Forward, register-resident rows.  PF: persistent CTAs that load their next
// row into registers before working on the current one, so a row's loads are
// in flight while the previous row is reduced and stored.  !PF: one row per
// CTA and fewer registers (LayerNorm+GELU on rows the prefetching geometry
// does not cover: unaligned, or wider than 16384 columns).
//
// Statistics in one block reduction: sums around a pilot K (the mean of the
// row's first min(cols, 32) elements, which every warp computes on its own
// with the same butterfly, so all get the same K):
//   S1 = sum(x - K), S2 = sum((x - K)^2);  mean = K + S1/n;  var = S2/n - (S1/n)^2.
// The rounding of S1 and the cancellation in var grow with |S1/n| / sigma;
// when (S1/n)^2 > var (a pilot more than one standard deviation off the mean)
// a second reduction takes the same two sums around the first estimate, which
// is then within a tiny fraction of sigma of the mean, and corrects both mean
// and variance.  Every row ends up as accurate as the reference's two-pass
// formula.  x - mean is rounded once, as in the reference, except on rows
// that take the second pass: there the centred value is corrected by c1, one
// more rounding (at most half an ulp of the centred value).
template <int VW, int VPT, int MAXT, int ACT, bool PF>
__global__ void __launch_bounds__(MAXT) ln_fwd_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
    float* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
    int64_t rows, int cols, float eps, GeluConst gc) {
  __shared__ float scratch[64];
  const int lane = threadIdx.x & 31;
  const int npilot = cols < 32 ? cols : 32;
  const float n = (float)cols;
  float nv[VPT][VW], np = 0.0f;
  auto load_row = [&](int64_t row) {
    const float* xr = x + row * (int64_t)cols;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * blockDim.x + threadIdx.x) * VW;
      if (e < cols) {
        load_vec<VW>(nv[i], xr + e, true);
      } else {
#pragma unroll
        for (int k = 0; k < VW; ++k) nv[i][k] = 0.0f;
      }
    }
    np = lane < npilot ? __ldg(xr + lane) : 0.0f;
  };
  int64_t row = blockIdx.x;
  if (row < rows) load_row(row);
  for (; row < rows; row += gridDim.x) {
    float v[VPT][VW];
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int k = 0; k < VW; ++k) v[i][k] = nv[i][k];
    // K needs no particular rounding: the sums are taken around whatever
    // value it has, and only |mean - K| affects the accuracy
    const float K = warp_sum(np) / (float)npilot;
    if (PF && row + gridDim.x < rows) load_row(row + gridDim.x);
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * blockDim.x + threadIdx.x) * VW;
#pragma unroll
      for (int k = 0; k < VW; ++k) {
        const float d = e < cols ? v[i][k] - K : 0.0f;
        s1 += d;
        s2 = fmaf(d, d, s2);
      }
    }
    float2 r = block_sum2(s1, s2, scratch);
    const float m1 = __fdiv_rn(r.x, n);
    float mu = K + m1;
    float var = __fdiv_rn(r.y, n) - m1 * m1;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int k = 0; k < VW; ++k) v[i][k] = __fsub_rn(v[i][k], mu);
    if (m1 * m1 > var) {  // uniform: every thread holds the same sums
      // pilot far from the mean: the same sums over the values centred on the
      // first estimate give the mean correction c1 and the variance
      float t1 = 0.0f, t2 = 0.0f;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int e = (i * blockDim.x + threadIdx.x) * VW;
#pragma unroll
        for (int k = 0; k < VW; ++k) {
          const float d = e < cols ? v[i][k] : 0.0f;
          t1 += d;
          t2 = fmaf(d, d, t2);
        }
      }
      r = block_sum2(t1, t2, scratch);
      const float c1 = __fdiv_rn(r.x, n);
      mu += c1;
      var = __fdiv_rn(r.y, n) - c1 * c1;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
#pragma unroll
        for (int k = 0; k < VW; ++k) v[i][k] = __fsub_rn(v[i][k], c1);
    }
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(fmaxf(var, 0.0f), eps)));
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
          const float yl = fmaf(v[i][k] * inv, wv[k], bv[k]);
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
  pdl_launch_dependents();  // the dweight/dbias finisher waits for this grid
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
        const float t1 = (xv[i][k] - mu) * inv;  // c*inv
        float g = gv[i][k];
        if constexpr (ACT == OXC_ACT_GELU_TANH) g = gelu_grad(fmaf(t1, wv[i][k], bv[i][k]), g, gc);
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


// ---- bulk-copy pipelined kernels (cols % 4 == 0, aligned) -------------------
//
// NG consumer groups of NWG warps each + 1 producer warp.  Group g processes
// the CTA's rows i = g, g + NG, ... so NG rows are in their arithmetic at the
// same time (each group's reductions use its own named barrier), while the
// producer keeps the next rows streaming in.  weight/bias live in shared
// memory (read once per CTA), leaving registers for the row slices.

// Loads w (and b) into shared memory with every thread of the CTA.
__device__ __forceinline__ void stage_params(float* ws, const float* w, float* bs, const float* b,
                                             int cols) {
  const int nvec = cols >> 2;
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    reinterpret_cast<float4*>(ws)[v] = ld_keep(reinterpret_cast<const float4*>(w) + v);
    if (bs) reinterpret_cast<float4*>(bs)[v] = ld_keep(reinterpret_cast<const float4*>(b) + v);
  }
}

// SACC: the per-group dweight/dbias accumulators live in shared memory
// (2 * cols floats per group after w and b) instead of registers.
template <int NG, int NWG, int VPT, int ACT, int MODE, bool SACC>
__global__ void __launch_bounds__((NG * NWG + 1) * 32, 1) ln_bwd_pipe_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
    const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
    const float* __restrict__ dy, float* __restrict__ dx, float* __restrict__ parts,
    int64_t rows, int cols, int64_t chunk, int stages, GeluConst gc) {
  pdl_launch_dependents();  // the dweight/dbias finisher waits for this grid
  extern __shared__ unsigned char smem[];
  float* red;
  const RowRing<2> ring = make_ring<2, NWG>(smem, stages, cols, &red);
  float* ws = red + 64;
  float* bs = ws + cols;
  float* sacc = bs + cols;  // [NG][2][cols] when SACC
  stage_params(ws, w, bs, b, cols);
  if constexpr (SACC) {
    for (int v = threadIdx.x; v < NG * 2 * cols; v += blockDim.x) sacc[v] = 0.0f;
  }
  __syncthreads();
  const int64_t r0 = (int64_t)blockIdx.x * chunk;
  const int64_t r1 = min(rows, r0 + chunk);
  const int warp = threadIdx.x >> 5;
  if (warp == NG * NWG) {
    if ((threadIdx.x & 31) == 0 && r0 < r1) {
      const float* src[2] = {x, dy};
      produce_rows<2>(ring, src, r0, r1);
    }
    return;
  }
  constexpr int T = NWG * 32;
  const int g = warp / NWG, gt = threadIdx.x - g * T, bar = 1 + g;
  float* gred = red + g * (NWG + 1);
  const int nvec = cols >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(ws);
  const float4* b4 = reinterpret_cast<const float4*>(bs);
  float4 adw[SACC ? 1 : VPT], adb[SACC ? 1 : VPT];
  if constexpr (!SACC) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      adw[k] = make_float4(0, 0, 0, 0);
      adb[k] = make_float4(0, 0, 0, 0);
    }
  }
  float4* gdw = reinterpret_cast<float4*>(sacc + (size_t)g * 2 * cols);
  float4* gdb = gdw + nvec;
  const float inv_n = __fdiv_rn(1.0f, (float)cols);
  // Row statistics are prefetched one group-iteration ahead so their global
  // load latency is not on each row's critical path.
  float mu_next = 0.0f, inv_next = 0.0f;
  if (g < r1 - r0) {
    mu_next = __ldg(mean_in + r0 + g);
    inv_next = __ldg(rstd_in + r0 + g);
  }
  for (int64_t i = g; i < r1 - r0; i += NG) {
    const int64_t row = r0 + i;
    const float mu = mu_next, inv = inv_next;
    if (i + NG < r1 - r0) {
      mu_next = __ldg(mean_in + row + NG);
      inv_next = __ldg(rstd_in + row + NG);
    }
    const bool ok = consumer_acquire<2>(ring, i);
    const int stage = (int)(i % ring.stages);
    const float4* xs = reinterpret_cast<const float4*>(ring.row(stage, 0));
    const float4* gs = reinterpret_cast<const float4*>(ring.row(stage, 1));
    float4 xv[VPT], gv[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int slot = k * T + gt;
      const bool valid = ok && slot < nvec;
      xv[k] = valid ? xs[slot] : make_float4(0, 0, 0, 0);
      gv[k] = valid ? gs[slot] : make_float4(0, 0, 0, 0);
    }
    consumer_release<2>(ring, i);
    // Element pairs on the packed f32x2 pipe: every lane rounds as the scalar
    // operations would, and the row sums run as two interleaved partials.
    const float2 nmu2 = bcast2(-mu), inv2 = bcast2(inv);
    float2 s1p = make_float2(0.0f, 0.0f), s2p = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int slot = k * T + gt;
      float4 wv = make_float4(0, 0, 0, 0), bv = make_float4(0, 0, 0, 0);
      if (slot < nvec) {
        wv = w4[slot];
        bv = b4[slot];
      }
      float2* xe = reinterpret_cast<float2*>(&xv[k]);
      float2* ge = reinterpret_cast<float2*>(&gv[k]);
      const float2* we = reinterpret_cast<const float2*>(&wv);
      const float2* be = reinterpret_cast<const float2*>(&bv);
      float4 dw4, db4;
      if constexpr (SACC) {
        dw4 = slot < nvec ? gdw[slot] : make_float4(0, 0, 0, 0);
        db4 = slot < nvec ? gdb[slot] : make_float4(0, 0, 0, 0);
      }
      float2* dwe = SACC ? reinterpret_cast<float2*>(&dw4) : reinterpret_cast<float2*>(&adw[SACC ? 0 : k]);
      float2* dbe = SACC ? reinterpret_cast<float2*>(&db4) : reinterpret_cast<float2*>(&adb[SACC ? 0 : k]);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float2 t1 = __fmul2_rn(__fadd2_rn(xe[e], nmu2), inv2);  // (x - mu) * inv
        float2 gg = ge[e];
        if constexpr (ACT == OXC_ACT_GELU_TANH) gg = gelu_grad2(__ffma2_rn(t1, we[e], be[e]), gg, gc);
        dwe[e] = __ffma2_rn(gg, t1, dwe[e]);
        dbe[e] = __fadd2_rn(dbe[e], gg);
        const float2 gw = __fmul2_rn(gg, we[e]);
        if constexpr (MODE == OXC_GRAD_REF) {
          ge[e] = __fmul2_rn(gw, inv2);
          s1p = __fadd2_rn(s1p, ge[e]);
        } else {
          ge[e] = gw;
          xe[e] = t1;
          s1p = __fadd2_rn(s1p, gw);
          s2p = __ffma2_rn(gw, t1, s2p);
        }
      }
      if constexpr (SACC) {
        if (slot < nvec) {
          gdw[slot] = dw4;
          gdb[slot] = db4;
        }
      }
    }
    float s1 = s1p.x + s1p.y, s2 = s2p.x + s2p.y;
    s1 = group_sum<NWG>(s1, gred, bar);
    if constexpr (MODE == OXC_GRAD_EXACT) s2 = group_sum<NWG>(s2, gred, bar);
    float4* dxr = reinterpret_cast<float4*>(dx + row * (int64_t)cols);
    const float shift = -s1 * inv_n;
    const float m1 = s1 * inv_n, m2 = s2 * inv_n;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int slot = k * T + gt;
      if (ok && slot < nvec) {
        float4 o;
        float2* oe = reinterpret_cast<float2*>(&o);
        const float2* xe = reinterpret_cast<const float2*>(&xv[k]);
        const float2* ge = reinterpret_cast<const float2*>(&gv[k]);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if constexpr (MODE == OXC_GRAD_REF) {
            oe[e] = __fadd2_rn(ge[e], bcast2(shift));
          } else {  // inv * ((g - m1) - x * m2), the last two as one fused step
            oe[e] = __fmul2_rn(inv2, __ffma2_rn(xe[e], bcast2(-m2), __fadd2_rn(ge[e], bcast2(-m1))));
          }
        }
        st_stream(dxr + slot, o);
      }
    }
  }
  // Combine the groups' column partials in group order.
  all_consumers_sync<NG * NWG * 32>();
  if constexpr (SACC) {
    float4* pw = reinterpret_cast<float4*>(parts + (int64_t)blockIdx.x * cols);
    float4* pb = reinterpret_cast<float4*>(parts + ((int64_t)gridDim.x + blockIdx.x) * cols);
    const float4* s4 = reinterpret_cast<const float4*>(sacc);
    for (int v = threadIdx.x; v < nvec; v += NG * NWG * 32) {
      float4 a = s4[v], c = s4[nvec + v];
      for (int h = 1; h < NG; ++h) {
        const float4 p = s4[(size_t)2 * h * nvec + v];
        const float4 q = s4[(size_t)(2 * h + 1) * nvec + v];
        a.x += p.x; a.y += p.y; a.z += p.z; a.w += p.w;
        c.x += q.x; c.y += q.y; c.z += q.z; c.w += q.w;
      }
      pw[v] = a;
      pb[v] = c;
    }
    return;
  } else {
  float4* comb = reinterpret_cast<float4*>(ring.buf);  // (NG-1) x 2 x cols floats
  if (g > 0) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int slot = k * T + gt;
      if (slot < nvec) {
        comb[(size_t)(2 * (g - 1)) * nvec + slot] = adw[k];
        comb[(size_t)(2 * (g - 1) + 1) * nvec + slot] = adb[k];
      }
    }
  }
  all_consumers_sync<NG * NWG * 32>();
  if (g == 0) {
    float4* pw = reinterpret_cast<float4*>(parts + (int64_t)blockIdx.x * cols);
    float4* pb = reinterpret_cast<float4*>(parts + ((int64_t)gridDim.x + blockIdx.x) * cols);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int slot = k * T + gt;
      if (slot < nvec) {
        float4 a = adw[k], c = adb[k];
        for (int h = 1; h < NG; ++h) {
          const float4 p = comb[(size_t)(2 * (h - 1)) * nvec + slot];
          const float4 q = comb[(size_t)(2 * (h - 1) + 1) * nvec + slot];
          a.x += p.x; a.y += p.y; a.z += p.z; a.w += p.w;
          c.x += q.x; c.y += q.y; c.z += q.z; c.w += q.w;
        }
        pw[slot] = a;
        pb[slot] = c;
      }
    }
  }
  }
}

// Pipeline geometry: NG groups x NWG warps.
constexpr int kBwdNG = 2, kBwdNWG = 8;   // 2 rows in flight, 256 threads per row

// Max dynamic shared memory per block (opt-in) of the current device.
static size_t max_smem_optin() {
  static size_t cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 48 * 1024;
  if (!cached[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
      v = 48 * 1024;
    cached[dev] = (size_t)v;
  }
  return cached[dev];
}

// Stages of the ring for `nin` inputs of `cols` floats plus the staged
// weight/bias (0 = pipeline unusable: fewer than `min_stages` fit).
static int pipe_stages(int nin, int64_t cols, int max_stages, int min_stages,
                       int64_t extra_floats = 0) {
  const size_t avail = max_smem_optin();
  int st = max_stages;
  while (st >= min_stages && ring_smem_bytes(nin, cols, st, 2 * cols + extra_floats) > avail) --st;
  return st >= min_stages ? st : 0;
}

// VPT (float4 slots per consumer thread, threads = nwg * 32), or 0.
static int pipe_vpt(int64_t cols, int nwg, int max_vpt) {
  const int64_t nvec = cols / 4, T = (int64_t)nwg * 32;
  for (int v : {1, 2, 3, 4, 8})
    if (v <= max_vpt && nvec <= v * T) return v;
  return 0;
}

template <typename K>
static void allow_smem(K kernel, size_t bytes) {
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

static int64_t ln_bwd_ctas(int64_t rows) {
  int64_t g = 2 * (int64_t)sm_count();
  const int64_t by_rows = (rows + 7) / 8;
  if (g > by_rows) g = by_rows;
  return g < 1 ? 1 : g;
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
  const GeluConst gc = gelu_const();
  // float4 rows that fit 8 vectors per thread on at most 512 threads (up to
  // 16384 columns): the persistent register kernel, next row prefetched, with
  // the deep geometry -- for plain LayerNorm and LayerNorm+GELU alike
  const RowGeom deep = v4 ? row_geom_deep(cols) : RowGeom{};
  if (deep.ok && deep.block <= 512) {
    auto ctas = [&](const void* k) {
      const int64_t fit = (int64_t)sm_count() * std::max(1, occupancy(k, deep.block, 0));
      return (unsigned)std::min<int64_t>(rows, fit);
    };
#define LAUNCH_D(VW, VPT, MAXT)                                                            \
  do {                                                                                     \
    if (act == OXC_ACT_GELU_TANH) {                                                        \
      auto k = ln_fwd_kernel<VW, VPT, MAXT, OXC_ACT_GELU_TANH, true>;                      \
      k<<<ctas((const void*)k), deep.block, 0, s>>>(x, w, b, y, mean, rstd, rows,          \
                                                    (int)cols, eps, gc);                   \
    } else {                                                                               \
      auto k = ln_fwd_kernel<VW, VPT, MAXT, OXC_ACT_NONE, true>;                           \
      k<<<ctas((const void*)k), deep.block, 0, s>>>(x, w, b, y, mean, rstd, rows,          \
                                                    (int)cols, eps, gc);                   \
    }                                                                                      \
  } while (0)
    OXC_DISPATCH_ROW(deep, LAUNCH_D);
#undef LAUNCH_D
    return check_launch("oxc_layer_norm_fwd");
  }
  // wider or unaligned rows: one row per CTA for LayerNorm+GELU, persistent
  // for plain LayerNorm
  RowGeom g = row_geom(cols, v4);
  const unsigned grid = (unsigned)(rows < 0x7fffffff ? rows : 0x7fffffff);
  // persistent: as many CTAs as fit on the GPU at once, each looping over rows
  auto ctas_for = [&](const void* k) {
    const int64_t fit = (int64_t)sm_count() * std::max(1, occupancy(k, g.block, 0));
    return (unsigned)std::min<int64_t>(rows, fit);
  };
#define LAUNCH(VW, VPT, MAXT)                                                              \
  do {                                                                                     \
    if (act == OXC_ACT_GELU_TANH) {                                                        \
      ln_fwd_kernel<VW, VPT, MAXT, OXC_ACT_GELU_TANH, false>                               \
          <<<grid, g.block, 0, s>>>(x, w, b, y, mean, rstd, rows, (int)cols, eps, gc);     \
    } else {                                                                               \
      auto k = ln_fwd_kernel<VW, VPT, MAXT, OXC_ACT_NONE, true>;                           \
      k<<<ctas_for((const void*)k), g.block, 0, s>>>(x, w, b, y, mean, rstd, rows,         \
                                                     (int)cols, eps, gc);                  \
    }                                                                                      \
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
  float* parts = static_cast<float*>(workspace);
  const GeluConst gc = gelu_const();
  // shared-memory accumulators (2 * NG * cols floats) when the ring keeps
  // NG + 2 stages alongside them; else register accumulators
  const int stages_sacc = v4 ? pipe_stages(2, cols, 6, kBwdNG + 2, 2 * kBwdNG * cols) : 0;
  const bool sacc = stages_sacc > 0;
  const int stages = sacc ? stages_sacc : (v4 ? pipe_stages(2, cols, 6, kBwdNG + 1) : 0);
  const int vpt = v4 ? pipe_vpt(cols, kBwdNWG, 4) : 0;
  if (stages && vpt) {
    // At most ln_bwd_ctas(rows) CTAs, the partial slots the workspace holds.
    const int64_t ctas = std::min<int64_t>(sm_count(), ln_bwd_ctas(rows));
    if ((size_t)2 * ctas * cols * sizeof(float) > workspace_bytes)
      return fail(OXC_ERR_OTHER, "internal: layer_norm backward partials exceed the workspace");
    const int64_t chunk = (rows + ctas - 1) / ctas;
    const size_t smem = ring_smem_bytes(2, cols, stages, 2 * cols + (sacc ? 2 * kBwdNG * cols : 0));
    const int block = (kBwdNG * kBwdNWG + 1) * 32;
#define LAUNCH_P(VPT, ACT, MODE)                                                              \
  do {                                                                                        \
    if (sacc) {                                                                               \
      auto k = ln_bwd_pipe_kernel<kBwdNG, kBwdNWG, VPT, ACT, MODE, true>;                     \
      allow_smem(k, smem);                                                                    \
      k<<<(unsigned)ctas, block, smem, s>>>(x, w, b, mean, rstd, dy, dx, parts, rows,         \
                                            (int)cols, chunk, stages, gc);                    \
    } else {                                                                                  \
      auto k = ln_bwd_pipe_kernel<kBwdNG, kBwdNWG, VPT, ACT, MODE, false>;                    \
      allow_smem(k, smem);                                                                    \
      k<<<(unsigned)ctas, block, smem, s>>>(x, w, b, mean, rstd, dy, dx, parts, rows,         \
                                            (int)cols, chunk, stages, gc);                    \
    }                                                                                         \
  } while (0)
#define LAUNCH_A(VPT)                                                                         \
  do {                                                                                        \
    if (act == OXC_ACT_GELU_TANH) {                                                           \
      if (grad_mode == OXC_GRAD_REF) LAUNCH_P(VPT, OXC_ACT_GELU_TANH, OXC_GRAD_REF);          \
      else LAUNCH_P(VPT, OXC_ACT_GELU_TANH, OXC_GRAD_EXACT);                                  \
    } else {                                                                                  \
      if (grad_mode == OXC_GRAD_REF) LAUNCH_P(VPT, OXC_ACT_NONE, OXC_GRAD_REF);               \
      else LAUNCH_P(VPT, OXC_ACT_NONE, OXC_GRAD_EXACT);                                       \
    }                                                                                         \
  } while (0)
    switch (vpt) {
      case 1: LAUNCH_A(1); break;
      case 2: LAUNCH_A(2); break;
      case 3: LAUNCH_A(3); break;
      default: LAUNCH_A(4); break;
    }
#undef LAUNCH_A
#undef LAUNCH_P
    oxc_status st = check_launch("oxc_layer_norm_bwd");
    if (st) return st;
    launch_colsum_partials(parts, (int)ctas, cols, dw, s, parts + ctas * cols, db);
    return check_launch("oxc_layer_norm_bwd (dw, db)");
  }
  RowGeom g = row_geom(cols, v4, 512);
  const int64_t ctas = ln_bwd_ctas(rows);
  const int64_t chunk = (rows + ctas - 1) / ctas;
  if ((size_t)2 * ctas * cols * sizeof(float) > workspace_bytes)
    return fail(OXC_ERR_OTHER, "internal: layer_norm backward partials exceed the workspace");
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
  launch_colsum_partials(parts, (int)ctas, cols, dw, s, parts + ctas * cols, db);
  return check_launch("oxc_layer_norm_bwd (dw, db)");
}

}  // extern "C"
