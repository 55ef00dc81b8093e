// swiglu.cu -- F.silu and the SwiGLU gate silu(g) * u, forward and VJP.
//
// Reference (python/oxitorch/nn/functional.py:202-204; registry ops.rs:176):
//   s = sigmoid(g) = 1 / (1 + exp(-g));  silu = g * s;  h = silu * u
// VJP of that graph (crates/oxi-autograd/src/ops.rs:62-73 mul, 236-247 sigmoid):
//   du = dh * silu
//   t  = dh * u                       (grad of silu)
//   dg = t * s + (t * g) * (s * (1 - s))
// Each step is the same f32 operation in the same order (the two terms of dg
// are the two graph contributions; their sum is order-free); exp is CUDA's.
// F.silu is the same kernel with u = 1 (the multiplications by 1 are exact).
//
// Layout: g and u are 2-D views [rows, cols] with any strides -- BASELINE
// config 5 passes g as a transposed view (strides [1, rows]).  Rows are tokens,
// columns features.  A CTA owns strips of 32 tokens and walks all features of a
// strip, so the forward finishes the dim-1 sum / max / argmax of h in registers
// (no second pass over h) and the VJP accumulates sum(dg^2) + sum(du^2)
// (clip_grad_norm_'s total) per CTA.  Three kernel families, picked per call:
//  * tile kernels (the fast path: 16-byte aligned rows, gate row- or
//    column-major, u and dh dense): a warp-specialised bulk-copy/TMA pipeline
//    with 192-feature tiles; the long contiguous row segments (768 bytes) are
//    what keeps HBM near its copy bandwidth;
//  * streaming kernels (any row stride, gate row- or column-major): gate
//    staged in shared memory per 256-feature chunk, other operands streamed;
//  * 32x32 tile kernels for anything else (every operand any strides).
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "tilepipe.cuh"

namespace oxc {

// 1 / (1 + e^-g) as the reference rounds it: the sum rounded, then the
// correctly rounded quotient.  __frcp_rn is the correctly rounded reciprocal,
// the same value as __fdiv_rn(1.0f, x) for every x, in fewer instructions.
__device__ __forceinline__ float sigmoid_ref(float g) {
  return __frcp_rn(__fadd_rn(1.0f, expf(-g)));
}

// Stages a 32x32 tile of v (rows r0.., cols c0..) into t[c][r].
__device__ __forceinline__ void load_tile(float (*t)[33], const View2& v, int64_t r0, int64_t c0,
                                          int64_t R, int64_t C) {
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  if (v.sr == 1 && v.sc != 1) {  // column-major: lanes walk r
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
      const int64_t r = r0 + tx, c = c0 + j;
      t[j][tx] = (r < R && c < C) ? __ldg(v.p + r + c * v.sc) : 0.0f;
    }
  } else {  // row-major (or anything else): lanes walk c
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
      const int64_t r = r0 + j, c = c0 + tx;
      t[tx][j] = (r < R && c < C) ? __ldg(v.p + r * v.sr + c * v.sc) : 0.0f;
    }
  }
}

// Forward.  u.p == nullptr: silu only.  Row outputs optional.
__global__ void __launch_bounds__(256) swiglu_fwd_kernel(View2 g, View2 u, float* __restrict__ h,
                                                         int64_t R, int64_t C,
                                                         float* __restrict__ row_sum,
                                                         float* __restrict__ row_max,
                                                         float* __restrict__ row_argmax) {
  __shared__ float tg[32][33];
  __shared__ float tu[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const bool rows_out = row_sum || row_max || row_argmax;
  for (int64_t r0 = (int64_t)blockIdx.x * 32; r0 < R; r0 += (int64_t)gridDim.x * 32) {
    float sum[4], mx[4];
    int64_t am[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) { sum[k] = 0.0f; mx[k] = 0.0f; am[k] = -1; }
    for (int64_t c0 = 0; c0 < C; c0 += 32) {
      load_tile(tg, g, r0, c0, R, C);
      if (u.p) load_tile(tu, u, r0, c0, R, C);
      __syncthreads();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = ty + 8 * k;
        const int64_t r = r0 + j, c = c0 + tx;
        if (r < R && c < C) {
          const float gv = tg[tx][j];
          const float s1 = __fmul_rn(gv, sigmoid_ref(gv));
          const float hv = u.p ? __fmul_rn(s1, tu[tx][j]) : s1;
          st_stream(h + r * C + c, hv);
          if (rows_out) {
            sum[k] = __fadd_rn(sum[k], hv);
            if (!isnan(hv) && (am[k] < 0 || hv > mx[k])) { mx[k] = hv; am[k] = c; }
          }
        }
      }
      __syncthreads();
    }
    if (rows_out) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float s = sum[k], m = mx[k];
        long long a = am[k];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
          const float om = __shfl_xor_sync(0xffffffffu, m, off);
          const long long oa = __shfl_xor_sync(0xffffffffu, a, off);
          if (oa >= 0 && (a < 0 || om > m || (om == m && oa < a))) { m = om; a = oa; }
        }
        const int64_t r = r0 + ty + 8 * k;
        if (tx == 0 && r < R) {
          if (row_sum) row_sum[r] = s;
          // f32::max fold from -inf ignores NaN; all-NaN rows give -inf
          if (row_max) row_max[r] = a < 0 ? -INFINITY : m;
          if (row_argmax) {
            // the reference's argmax starts at element 0: a NaN there wins
            const float h0 = h[r * C];
            row_argmax[r] = (C > 0 && isnan(h0)) ? 0.0f : (float)(a < 0 ? 0 : a);
          }
        }
      }
    }
  }
}

// VJP.  u.p == nullptr: silu only (du not written).  sumsq_parts (optional):
// per-CTA f64 sum of dg^2 + du^2.
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(View2 g, View2 u, View2 dh,
                                                         float* __restrict__ dg,
                                                         float* __restrict__ du, int64_t R,
                                                         int64_t C,
                                                         double* __restrict__ sumsq_parts) {
  __shared__ float tg[32][33];
  __shared__ float tu[32][33];
  __shared__ float td[32][33];
  __shared__ double red[33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  double sq = 0.0;
  for (int64_t r0 = (int64_t)blockIdx.x * 32; r0 < R; r0 += (int64_t)gridDim.x * 32) {
    for (int64_t c0 = 0; c0 < C; c0 += 32) {
      load_tile(tg, g, r0, c0, R, C);
      if (u.p) load_tile(tu, u, r0, c0, R, C);
      load_tile(td, dh, r0, c0, R, C);
      __syncthreads();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = ty + 8 * k;
        const int64_t r = r0 + j, c = c0 + tx;
        if (r < R && c < C) {
          const float gv = tg[tx][j], dv = td[tx][j];
          const float s = sigmoid_ref(gv);
          const float s1 = __fmul_rn(gv, s);
          float t = dv;
          if (u.p) {
            const float uv = tu[tx][j];
            const float duv = __fmul_rn(dv, s1);
            st_stream(du + r * C + c, duv);
            sq += (double)duv * (double)duv;
            t = __fmul_rn(dv, uv);
          }
          const float term1 = __fmul_rn(t, s);
          const float dsig = __fmul_rn(s, __fsub_rn(1.0f, s));
          const float term2 = __fmul_rn(__fmul_rn(t, gv), dsig);
          const float dgv = __fadd_rn(term1, term2);
          st_stream(dg + r * C + c, dgv);
          sq += (double)dgv * (double)dgv;
        }
      }
      __syncthreads();
    }
  }
  if (sumsq_parts) {
    const double tot = block_sum(sq, red);
    if (threadIdx.x == 0) sumsq_parts[blockIdx.x] = tot;
  }
}

// Fixed-order block reduction of the per-CTA partials (thread t adds parts
// t, t+256, ... in order; then the warp/block tree of block_sum).
__global__ void __launch_bounds__(256) sumsq_parts_finish(const double* __restrict__ parts, int n,
                                                          double* __restrict__ out) {
  __shared__ double red[33];
  double a = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) a += parts[i];
  const double t = block_sum(a, red);
  if (threadIdx.x == 0) out[0] = t;
}

// ---- streaming kernels: row-major u/dh/outputs, gate row- or column-major ----
//
// A CTA owns 32 tokens (rows) and walks the features in chunks of 256.  The
// gate chunk [32 x 256] is staged in shared memory as st[token][feature]
// (row pitch 257 floats): a column-major gate is read 128 bytes per feature
// (lanes over tokens), a row-major one 128 bytes per token; writes and reads of
// the tile are bank-conflict free.  Every row-major operand (u, dh, h, dg, du)
// is streamed straight between HBM and registers in 1 KB row segments: warp w
// handles tokens w, w+8, w+16, w+24 and lane l features l + 32k of the chunk.
constexpr int kSwTok = 32, kSwChunk = 256, kSwPitch = kSwChunk + 1;

__device__ __forceinline__ void stage_gate(float* st, const View2& g, int64_t r0, int64_t c0,
                                           int64_t R, int64_t C) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (g.sr == 1) {  // column-major: lanes over tokens, one feature row per step
#pragma unroll 8
    for (int f = warp; f < kSwChunk; f += 8) {
      const int64_t r = r0 + lane, c = c0 + f;
      st[lane * kSwPitch + f] = (r < R && c < C) ? __ldg(g.p + r + c * g.sc) : 0.0f;
    }
  } else {  // row-major (or any): lanes over features
#pragma unroll 4
    for (int t = warp; t < kSwTok; t += 8) {
      const int64_t r = r0 + t;
#pragma unroll
      for (int k = 0; k < kSwChunk / 32; ++k) {
        const int64_t c = c0 + lane + 32 * k;
        st[t * kSwPitch + lane + 32 * k] = (r < R && c < C) ? __ldg(g.p + r * g.sr + c * g.sc) : 0.0f;
      }
    }
  }
}

__global__ void __launch_bounds__(256, 3) swiglu_fwd_stream_kernel(
    View2 g, const float* __restrict__ u, float* __restrict__ h, int64_t R, int64_t C,
    float* __restrict__ row_sum, float* __restrict__ row_max, float* __restrict__ row_argmax) {
  __shared__ float st[kSwTok * kSwPitch];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool rows_out = row_sum || row_max || row_argmax;
  for (int64_t r0 = (int64_t)blockIdx.x * kSwTok; r0 < R; r0 += (int64_t)gridDim.x * kSwTok) {
    float sum[4], mx[4];
    int am[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) { sum[i] = 0.0f; mx[i] = 0.0f; am[i] = -1; }
    for (int64_t c0 = 0; c0 < C; c0 += kSwChunk) {
      __syncthreads();  // previous chunk's tile fully read
      stage_gate(st, g, r0, c0, R, C);
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = warp + 8 * i;
        const int64_t r = r0 + t;
        if (r >= R) continue;
        float uv[kSwChunk / 32];
#pragma unroll
        for (int k = 0; k < kSwChunk / 32; ++k) {
          const int64_t c = c0 + lane + 32 * k;
          uv[k] = (u && c < C) ? ld_stream(u + r * C + c) : 1.0f;
        }
#pragma unroll
        for (int k = 0; k < kSwChunk / 32; ++k) {
          const int64_t c = c0 + lane + 32 * k;
          if (c < C) {
            const float gv = st[t * kSwPitch + lane + 32 * k];
            const float s1 = __fmul_rn(gv, sigmoid_ref(gv));
            const float hv = u ? __fmul_rn(s1, uv[k]) : s1;
            st_stream(h + r * C + c, hv);
            if (rows_out) {
              sum[i] = __fadd_rn(sum[i], hv);
              if (!isnan(hv) && (am[i] < 0 || hv > mx[i])) { mx[i] = hv; am[i] = (int)c; }
            }
          }
        }
      }
    }
    if (rows_out) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float s = sum[i], m = mx[i];
        int a = am[i];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
          const float om = __shfl_xor_sync(0xffffffffu, m, off);
          const int oa = __shfl_xor_sync(0xffffffffu, a, off);
          if (oa >= 0 && (a < 0 || om > m || (om == m && oa < a))) { m = om; a = oa; }
        }
        const int64_t r = r0 + warp + 8 * i;
        if (lane == 0 && r < R) {
          if (row_sum) row_sum[r] = s;
          if (row_max) row_max[r] = a < 0 ? -INFINITY : m;
          if (row_argmax) {
            const float h0 = h[r * C];  // written by this lane (feature 0, k = 0)
            row_argmax[r] = (C > 0 && isnan(h0)) ? 0.0f : (float)(a < 0 ? 0 : a);
          }
        }
      }
    }
  }
}

__global__ void __launch_bounds__(256) swiglu_bwd_stream_kernel(
    View2 g, const float* __restrict__ u, const float* __restrict__ dh, float* __restrict__ dg,
    float* __restrict__ du, int64_t R, int64_t C, double* __restrict__ sumsq_parts) {
  __shared__ float st[kSwTok * kSwPitch];
  __shared__ double red[33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double sq = 0.0;
  for (int64_t r0 = (int64_t)blockIdx.x * kSwTok; r0 < R; r0 += (int64_t)gridDim.x * kSwTok) {
    for (int64_t c0 = 0; c0 < C; c0 += kSwChunk) {
      __syncthreads();
      stage_gate(st, g, r0, c0, R, C);
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = warp + 8 * i;
        const int64_t r = r0 + t;
        if (r >= R) continue;
        float uv[kSwChunk / 32], dv[kSwChunk / 32];
#pragma unroll
        for (int k = 0; k < kSwChunk / 32; ++k) {
          const int64_t c = c0 + lane + 32 * k;
          uv[k] = (u && c < C) ? ld_stream(u + r * C + c) : 1.0f;
          dv[k] = c < C ? ld_stream(dh + r * C + c) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < kSwChunk / 32; ++k) {
          const int64_t c = c0 + lane + 32 * k;
          if (c < C) {
            const float gv = st[t * kSwPitch + lane + 32 * k];
            const float s = sigmoid_ref(gv);
            const float s1 = __fmul_rn(gv, s);
            float tt = dv[k];
            if (u) {
              const float duv = __fmul_rn(dv[k], s1);
              st_stream(du + r * C + c, duv);
              sq += (double)duv * (double)duv;
              tt = __fmul_rn(dv[k], uv[k]);
            }
            const float term1 = __fmul_rn(tt, s);
            const float dsig = __fmul_rn(s, __fsub_rn(1.0f, s));
            const float dgv = __fadd_rn(term1, __fmul_rn(__fmul_rn(tt, gv), dsig));
            st_stream(dg + r * C + c, dgv);
            sq += (double)dgv * (double)dgv;
          }
        }
      }
    }
  }
  if (sumsq_parts) {
    const double tot = block_sum(sq, red);
    if (threadIdx.x == 0) sumsq_parts[blockIdx.x] = tot;
  }
}

// Row statistics of one lane: sum (in the lane's feature order), the max with
// its first index (a < 0: no value above -inf seen; NaN never compares
// greater, which is f32::max's NaN-ignoring fold), and whether h[r, 0] is NaN
// (the reference's argmax starts at element 0, so a NaN there is the answer).
struct RowStat {
  float s, m;
  int a;
  int nan0;
};

__device__ __forceinline__ void stat_merge(RowStat& x, float os, float om, int oa, int on) {
  x.s = __fadd_rn(x.s, os);
  if (oa >= 0 && (x.a < 0 || om > x.m || (om == x.m && oa < x.a))) { x.m = om; x.a = oa; }
  x.nan0 |= on;
}

template <bool GT, bool HAS_U>
__global__ void __launch_bounds__(kTThreads, 1) swiglu_fwd_tile_kernel(
    const __grid_constant__ CUtensorMap gmap, View2 g, const float* __restrict__ u,
    float* __restrict__ h, int64_t R, int64_t C, float* __restrict__ row_sum,
    float* __restrict__ row_max, float* __restrict__ row_argmax) {
  constexpr int NSLOT = HAS_U ? 2 : 1;
  extern __shared__ unsigned char smem_raw[];
  const TileRing<NSLOT, GT> ring = make_tile_ring<NSLOT, GT>(smem_raw, kStageFwd);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == kTCW) {
    const float* const src[2] = {u, nullptr};
    tile_producer<GT, NSLOT>(ring, &gmap, g, src, HAS_U ? 1 : 0, R, C);
    return;
  }
  const bool rows_out = row_sum || row_max || row_argmax;
  const int part = warp >> 3;
  const int t = 4 * (warp & 7) + (lane & 3);
  const int fl = part * (kTF / kTParts) + (lane >> 2);
  const int goff = gate_off<GT>(t, fl), uoff = t * kTP + fl;
  const int64_t nstrips = (R + kTT - 1) / kTT;
  int64_t i = 0;
  int parity = 0;
  for (int64_t strip = blockIdx.x; strip < nstrips; strip += gridDim.x, parity ^= 1) {
    const int64_t r = strip * kTT + t;
    float* hrow = h + r * C + fl;
    RowStat st{0.0f, -INFINITY, -1, 0};
    for (int64_t c0 = 0; c0 < C; c0 += kTF, ++i) {
      if (!tile_acquire(ring, i)) continue;
      const int stage = (int)(i % ring.stages);
      const float* gs = ring.slot(stage, 0) + goff;
      const float* us = ring.slot(stage, NSLOT - 1) + uoff;
      float gv[kTK], uv[kTK];
#pragma unroll
      for (int k = 0; k < kTK; ++k) {
        gv[k] = gs[k * kGateStep<GT>];
        uv[k] = HAS_U ? us[8 * k] : 1.0f;
      }
      tile_release(ring, i);
      if (r >= R) continue;
      const bool full = c0 + kTF <= C;
#pragma unroll
      for (int k = 0; k < kTK; ++k) {
        const int64_t c = c0 + fl + 8 * k;
        if (full || c < C) {
          const float s1 = __fmul_rn(gv[k], sigmoid_ref(gv[k]));
          const float hv = HAS_U ? __fmul_rn(s1, uv[k]) : s1;
          st_stream(hrow + c0 + 8 * k, hv);
          if (rows_out) {
            st.s = __fadd_rn(st.s, hv);
            if (hv > st.m) { st.m = hv; st.a = (int)c; }
            if (k == 0 && c == 0) st.nan0 = isnan(hv);
          }
        }
      }
    }
    if (!rows_out) continue;
    // the 8 lanes of a token (lane % 4 equal), then the feature parts in order
#pragma unroll
    for (int off = 4; off < 32; off <<= 1)
      stat_merge(st, __shfl_xor_sync(0xffffffffu, st.s, off),
                 __shfl_xor_sync(0xffffffffu, st.m, off), __shfl_xor_sync(0xffffffffu, st.a, off),
                 __shfl_xor_sync(0xffffffffu, st.nan0, off));
    float* xs = ring.stat + parity * kTParts * kTT * 4;
    if (part > 0 && lane < 4) {
      float* e = xs + (part * kTT + t) * 4;
      e[0] = st.s;
      e[1] = st.m;
      e[2] = __int_as_float(st.a);
      e[3] = __int_as_float(st.nan0);
    }
    consumer_sync<kTCW>();
    if (part == 0 && lane < 4 && r < R) {
#pragma unroll
      for (int p = 1; p < kTParts; ++p) {
        const float* e = xs + (p * kTT + t) * 4;
        stat_merge(st, e[0], e[1], __float_as_int(e[2]), __float_as_int(e[3]));
      }
      if (row_sum) row_sum[r] = st.s;
      if (row_max) row_max[r] = st.a < 0 ? -INFINITY : st.m;
      if (row_argmax) row_argmax[r] = st.nan0 ? 0.0f : (float)(st.a < 0 ? 0 : st.a);
    }
  }
}

template <bool GT, bool HAS_U>
__global__ void __launch_bounds__(kTThreads, 1) swiglu_bwd_tile_kernel(
    const __grid_constant__ CUtensorMap gmap, View2 g, const float* __restrict__ u,
    const float* __restrict__ dh, float* __restrict__ dg, float* __restrict__ du, int64_t R,
    int64_t C, double* __restrict__ sumsq_parts) {
  constexpr int NSLOT = HAS_U ? 3 : 2;
  extern __shared__ unsigned char smem_raw[];
  const TileRing<NSLOT, GT> ring = make_tile_ring<NSLOT, GT>(smem_raw, kStageBwd);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == kTCW) {
    const float* const src[2] = {HAS_U ? u : dh, dh};
    tile_producer<GT, NSLOT>(ring, &gmap, g, src, HAS_U ? 2 : 1, R, C);
    return;
  }
  const int t = 4 * (warp & 7) + (lane & 3);
  const int fl = (warp >> 3) * (kTF / kTParts) + (lane >> 2);
  const int goff = gate_off<GT>(t, fl), roff = t * kTP + fl;
  const int64_t nstrips = (R + kTT - 1) / kTT;
  double sq = 0.0;
  int64_t i = 0;
  for (int64_t strip = blockIdx.x; strip < nstrips; strip += gridDim.x) {
    const int64_t r = strip * kTT + t;
    float* dgrow = dg + r * C + fl;
    float* durow = HAS_U ? du + r * C + fl : nullptr;
    for (int64_t c0 = 0; c0 < C; c0 += kTF, ++i) {
      if (!tile_acquire(ring, i)) continue;
      const int stage = (int)(i % ring.stages);
      const float* gs = ring.slot(stage, 0) + goff;
      const float* us = ring.slot(stage, 1) + roff;
      const float* ds = ring.slot(stage, NSLOT - 1) + roff;
      float gv[kTK], uv[kTK], dv[kTK];
#pragma unroll
      for (int k = 0; k < kTK; ++k) {
        gv[k] = gs[k * kGateStep<GT>];
        uv[k] = HAS_U ? us[8 * k] : 1.0f;
        dv[k] = ds[8 * k];
      }
      tile_release(ring, i);
      if (r >= R) continue;
      const bool full = c0 + kTF <= C;
#pragma unroll
      for (int k = 0; k < kTK; ++k) {
        if (full || c0 + fl + 8 * k < C) {
          const float s = sigmoid_ref(gv[k]);
          const float s1 = __fmul_rn(gv[k], s);
          float tt = dv[k];
          if (HAS_U) {
            const float duv = __fmul_rn(dv[k], s1);
            st_stream(durow + c0 + 8 * k, duv);
            sq += (double)duv * (double)duv;
            tt = __fmul_rn(dv[k], uv[k]);
          }
          const float term1 = __fmul_rn(tt, s);
          const float dsig = __fmul_rn(s, __fsub_rn(1.0f, s));
          const float dgv = __fadd_rn(term1, __fmul_rn(__fmul_rn(tt, gv[k]), dsig));
          st_stream(dgrow + c0 + 8 * k, dgv);
          sq += (double)dgv * (double)dgv;
        }
      }
    }
  }
  if (sumsq_parts) {
    sq = warp_sum(sq);
    if (lane == 0) ring.red[warp] = sq;
    consumer_sync<kTCW>();
    if (warp == 0) {
      double v = lane < kTCW ? ring.red[lane] : 0.0;
      v = warp_sum(v);
      if (lane == 0) sumsq_parts[blockIdx.x] = v;
    }
  }
}

// The tile kernels need 16-byte aligned rows: C % 4 == 0, row-major u / dh
// dense with aligned bases, and the gate row-major (row stride % 4 == 0) or
// column-major (feature stride % 4 == 0, >= R) with an aligned base.
static int tile_gate_kind(const View2& g, const View2& u, const View2* d, int64_t R, int64_t C) {
  if (C % 4 != 0 || R > INT32_MAX || C > INT32_MAX || !aligned16(g.p)) return 0;
  if (u.p && !(u.sc == 1 && u.sr == C && aligned16(u.p))) return 0;
  if (d && !(d->sc == 1 && d->sr == C && aligned16(d->p))) return 0;
  if (g.sc == 1 && g.sr % 4 == 0 && g.sr >= C) return 1;               // row-major
  if (g.sr == 1 && g.sc % 4 == 0 && g.sc >= R && C > 1) return 2;      // column-major
  return 0;
}

static oxc_status view2(const oxc_view* v, const char* name, int64_t* R, int64_t* C, View2* out,
                        bool required) {
  if (!v) {
    if (required) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s is required", name);
    out->p = nullptr;
    out->sr = out->sc = 0;
    return OXC_OK;
  }
  if (v->ndim != 2)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s must be 2-D, got %d-D", name, v->ndim);
  if (*R < 0) { *R = v->shape[0]; *C = v->shape[1]; }
  if (v->shape[0] != *R || v->shape[1] != *C)
    return fail(OXC_ERR_SHAPE_MISMATCH, "shape mismatch: %s is [%lld, %lld], expected [%lld, %lld]",
                name, (long long)v->shape[0], (long long)v->shape[1], (long long)*R, (long long)*C);
  out->p = v->data;
  out->sr = v->strides[0];
  out->sc = v->strides[1];
  return OXC_OK;
}

static int64_t swiglu_ctas(int64_t R) {
  const int64_t tiles = (R + 31) / 32;
  return std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)sm_count() * 8));
}

// The streaming kernels need u (if any) dense row-major and the gate row- or
// column-major.
static bool stream_ok(const View2& g, const View2& u, int64_t C) {
  const bool g_ok = g.sc == 1 || g.sr == 1;
  const bool u_ok = !u.p || (u.sc == 1 && u.sr == C);
  return g_ok && u_ok;
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_swiglu_fwd(const oxc_view* gate, const oxc_view* up, float* h, float* row_sum,
                          float* row_max, float* row_argmax, void* stream) {
  int64_t R = -1, C = -1;
  View2 g, u;
  oxc_status st = view2(gate, "gate", &R, &C, &g, true);
  if (st || (st = view2(up, "up", &R, &C, &u, false))) return st;
  if (R == 0 || C == 0) return OXC_OK;
  if (!h || !g.p) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: swiglu: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int kind = tile_gate_kind(g, u, nullptr, R, C);
  CUtensorMap map{};
  if (kind == 2 && !gate_tensor_map(&map, g, R, C))
    return fail(OXC_ERR_OTHER, "oxc_swiglu_fwd: cuTensorMapEncodeTiled failed for the gate");
  if (kind) {
    const size_t smem = kind == 2 ? tile_smem_bytes<2, true>(kStageFwd, true)
                                  : tile_smem_bytes<2, false>(kStageFwd, true);
    const char* what = "oxc_swiglu_fwd";
    if (kind == 2 && u.p)
      return launch_tile(swiglu_fwd_tile_kernel<true, true>, smem, R, s, what, nullptr, map, g,
                         u.p, h, R, C, row_sum, row_max, row_argmax);
    if (kind == 2)
      return launch_tile(swiglu_fwd_tile_kernel<true, false>, smem, R, s, what, nullptr, map, g,
                         u.p, h, R, C, row_sum, row_max, row_argmax);
    if (u.p)
      return launch_tile(swiglu_fwd_tile_kernel<false, true>, smem, R, s, what, nullptr, map, g,
                         u.p, h, R, C, row_sum, row_max, row_argmax);
    return launch_tile(swiglu_fwd_tile_kernel<false, false>, smem, R, s, what, nullptr, map, g,
                       u.p, h, R, C, row_sum, row_max, row_argmax);
  }
  if (stream_ok(g, u, C)) {
    swiglu_fwd_stream_kernel<<<(unsigned)swiglu_ctas(R), 256, 0, s>>>(g, u.p, h, R, C, row_sum,
                                                                      row_max, row_argmax);
  } else {
    swiglu_fwd_kernel<<<(unsigned)swiglu_ctas(R), 256, 0, s>>>(g, u, h, R, C, row_sum, row_max,
                                                               row_argmax);
  }
  return check_launch("oxc_swiglu_fwd");
}

size_t oxc_swiglu_bwd_workspace_size(int64_t rows, int64_t cols) {
  (void)cols;
  return (size_t)swiglu_ctas(std::max<int64_t>(rows, 1)) * sizeof(double) + 256;
}

oxc_status oxc_swiglu_bwd(const oxc_view* gate, const oxc_view* up, const oxc_view* dh,
                          float* dgate, float* dup, double* sumsq, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int64_t R = -1, C = -1;
  View2 g, u, d;
  oxc_status st = view2(gate, "gate", &R, &C, &g, true);
  if (st || (st = view2(up, "up", &R, &C, &u, false)) || (st = view2(dh, "dh", &R, &C, &d, true)))
    return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (R == 0 || C == 0) {
    if (sumsq) {
      cudaError_t e = cudaMemsetAsync(sumsq, 0, sizeof(double), s);
      if (e != cudaSuccess) return cuda_fail(e, "oxc_swiglu_bwd");
    }
    return OXC_OK;
  }
  if (!dgate || (u.p && !dup))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: swiglu backward: null pointer");
  const int64_t ctas = swiglu_ctas(R);
  double* parts = nullptr;
  if (sumsq) {
    if (!workspace || workspace_bytes < oxc_swiglu_bwd_workspace_size(R, C))
      return fail(OXC_ERR_INVALID_ARGUMENT,
                  "invalid argument: swiglu backward needs a %zu-byte workspace for sumsq, got %zu",
                  oxc_swiglu_bwd_workspace_size(R, C), workspace_bytes);
    parts = reinterpret_cast<double*>((reinterpret_cast<uintptr_t>(workspace) + 15) & ~uintptr_t(15));
  }
  int64_t nparts = ctas;
  const int kind = tile_gate_kind(g, u, &d, R, C);
  if (kind) {
    CUtensorMap map{};
    if (kind == 2 && !gate_tensor_map(&map, g, R, C))
      return fail(OXC_ERR_OTHER, "oxc_swiglu_bwd: cuTensorMapEncodeTiled failed for the gate");
    const size_t smem = kind == 2 ? tile_smem_bytes<3, true>(kStageBwd, false)
                                  : tile_smem_bytes<3, false>(kStageBwd, false);
    const char* what = "oxc_swiglu_bwd";
    if (kind == 2 && u.p)
      st = launch_tile(swiglu_bwd_tile_kernel<true, true>, smem, R, s, what, &nparts, map, g, u.p,
                       d.p, dgate, dup, R, C, parts);
    else if (kind == 2)
      st = launch_tile(swiglu_bwd_tile_kernel<true, false>, smem, R, s, what, &nparts, map, g,
                       u.p, d.p, dgate, dup, R, C, parts);
    else if (u.p)
      st = launch_tile(swiglu_bwd_tile_kernel<false, true>, smem, R, s, what, &nparts, map, g,
                       u.p, d.p, dgate, dup, R, C, parts);
    else
      st = launch_tile(swiglu_bwd_tile_kernel<false, false>, smem, R, s, what, &nparts, map, g,
                       u.p, d.p, dgate, dup, R, C, parts);
  } else {
    if (stream_ok(g, u, C) && d.sc == 1 && d.sr == C)
      swiglu_bwd_stream_kernel<<<(unsigned)ctas, 256, 0, s>>>(g, u.p, d.p, dgate, dup, R, C,
                                                              parts);
    else
      swiglu_bwd_kernel<<<(unsigned)ctas, 256, 0, s>>>(g, u, d, dgate, dup, R, C, parts);
    st = check_launch("oxc_swiglu_bwd");
  }
  if (st || !sumsq) return st;
  sumsq_parts_finish<<<1, 256, 0, s>>>(parts, (int)nparts, sumsq);
  return check_launch("oxc_swiglu_bwd (sumsq)");
}

}  // extern "C"
