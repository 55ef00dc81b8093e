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
// config 5 passes g as a transposed view (strides [1, rows]).  A CTA owns 32
// rows and walks the columns in 32x32 tiles staged through shared memory, so
// every operand is read along its contiguous dim and every output written
// row-major, all coalesced.  Owning whole rows lets the forward finish the
// dim-1 sum / max / argmax of h in registers (no second pass over h) and the
// VJP accumulate sum(dg^2) + sum(du^2) (clip_grad_norm_'s total) per CTA.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace oxc {

struct View2 {
  const float* p;
  int64_t sr, sc;  // strides in elements
};

__device__ __forceinline__ float sigmoid_ref(float g) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
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
  if (stream_ok(g, u, C) && d.sc == 1 && d.sr == C)
    swiglu_bwd_stream_kernel<<<(unsigned)ctas, 256, 0, s>>>(g, u.p, d.p, dgate, dup, R, C, parts);
  else
    swiglu_bwd_kernel<<<(unsigned)ctas, 256, 0, s>>>(g, u, d, dgate, dup, R, C, parts);
  st = check_launch("oxc_swiglu_bwd");
  if (st || !sumsq) return st;
  sumsq_parts_finish<<<1, 256, 0, s>>>(parts, (int)ctas, sumsq);
  return check_launch("oxc_swiglu_bwd (sumsq)");
}

}  // extern "C"
