// softmax.cu -- F.softmax / F.log_softmax forward and VJP, and F.cross_entropy
// (mean reduction) forward and VJP.
//
// Reference (python/oxitorch/nn/functional.py):
//   softmax      (211-215): m = x.max(-1, True); e = (x - m).exp(); y = e / e.sum(-1, True)
//   log_softmax  (218-222): z = x - m; y = z - z.exp().sum(-1, True).log()
//   cross_entropy(277-293): ls = log_softmax(x); picked = (onehot * ls).sum(-1);
//                           loss = -(picked.mean())
// VJPs are the ones the reference graph builds (crates/oxi-autograd/src/ops.rs):
//   softmax:      dx = y * (g - sum_row(g*y))
//   log_softmax:  dx = g - exp(y) * sum_row(g)
//   cross_entropy: d[r,c] = exp(x - m) * ((g/M) * (1/s)) - (c == t_r ? g/M : 0)
//     (log VJP 1/s, exp VJP, sub VJP, the one-hot pick; the mean over M rows)
// The max node's VJP additionally scatters -sum_row(dz) to the argmax column;
// that sum is zero in exact arithmetic and only the row's rounding noise in
// the reference, so the kernels leave it out.
//
// Kernels, all HBM-bound (no contraction):
//   softmax_fwd/bwd: one CTA per row, two passes; pass 1 reads the row with
//     L2-allocating 128-bit loads (online max + rescaled sum over 16-value
//     chunks, the sum's terms from ex2.approx -- exp_rel -- or plain sums),
//     pass 2 re-reads it from L2 and writes -- DRAM sees one read + one write.
//   ce_fwd: one CTA of at most 256 threads per row, one online pass; writes
//     per-row (max, sum of exp, -log p_target) and never materialises a
//     full-size tensor.
//   ce_loss: deterministic f64 tree over the per-row values.
//   ce_bwd: grid-stride elementwise over [rows, cols] (128-bit when cols % 4
//     == 0), per-row (max, 1/s, target) read through L1; rows of >= 2048
//     classes go to ce_bwd_rows (one CTA per row, same per-element expression).
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace oxc {

struct MaxSum {
  float m;
  float s;
};

__device__ __forceinline__ MaxSum ms_merge(MaxSum a, MaxSum b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, a.s + b.s};
  const float sa = a.m == m ? a.s : a.s * expf(a.m - m);
  const float sb = b.m == m ? b.s : b.s * expf(b.m - m);
  return {m, sa + sb};
}

// Block-wide merge; every thread gets the result.  scratch: 2 x 33 floats.
__device__ __forceinline__ MaxSum block_maxsum(MaxSum v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MaxSum w{__shfl_xor_sync(0xffffffffu, v.m, o), __shfl_xor_sync(0xffffffffu, v.s, o)};
    v = ms_merge(v, w);
  }
  __syncthreads();
  if (lane == 0) {
    scratch[warp] = v.m;
    scratch[33 + warp] = v.s;
  }
  __syncthreads();
  if (warp == 0) {
    MaxSum t = lane < nwarps ? MaxSum{scratch[lane], scratch[33 + lane]} : MaxSum{-INFINITY, 0.0f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      MaxSum w{__shfl_xor_sync(0xffffffffu, t.m, o), __shfl_xor_sync(0xffffffffu, t.s, o)};
      t = ms_merge(t, w);
    }
    if (lane == 0) {
      scratch[32] = t.m;
      scratch[65] = t.s;
    }
  }
  __syncthreads();
  return {scratch[32], scratch[65]};
}

// e^d for d = x - m <= 0 as 2^(d * log2 e) with the ex2.approx instruction
// (flush-to-zero: results below 2^-126 of the row maximum's term are 0).  The
// subtraction comes first, so the terms near the maximum -- the ones that make
// up the sum -- see only ex2's own error; farther terms carry an extra
// |d| * 2^-23 relative error from the rounded argument, on values at most
// e^d of the largest term.  Used only for the row sums of exp; outputs that are
// themselves exponentials use expf.
__device__ __forceinline__ float exp_rel(float d) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d * 1.44269504088896341f));
  return r;
}

// Folds n values into the running (max, sum): the NaN-ignoring max of the
// values first, one rescale of the sum when the max grows, then n terms.
// While the max is still -inf the base is 0, so a -inf value adds 0 and a NaN
// adds NaN; a row whose final max is -inf gets the reference's NaN sum at the
// end (row_maxsum).
// With MIN the running minimum is folded into *mn as well (NaN-ignoring).
template <int N, bool MIN = false>
__device__ __forceinline__ void ms_fold(MaxSum& a, const float (&v)[N], float* mn = nullptr) {
  float mm = a.m;
#pragma unroll
  for (int i = 0; i < N; ++i) mm = fmaxf(mm, v[i]);
  if constexpr (MIN) {
#pragma unroll
    for (int i = 0; i < N; ++i) *mn = fminf(*mn, v[i]);
  }
  if (mm > a.m) {
    a.s *= exp_rel(a.m - mm);
    a.m = mm;
  }
  const float base = mm == -INFINITY ? 0.0f : mm;
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < N; ++i) t += exp_rel(v[i] - base);
  a.s += t;
}

// Row statistics (max, sum exp(x - max)) with 128-bit (VW = 4) or scalar
// loads; `keep` loads allocate in L2 so a second pass hits it.  A row whose
// max is -inf (all -inf and/or NaN) has sum NaN, as exp(-inf - -inf) is NaN.
// With MIN, *row_min (every thread) gets the row's NaN-ignoring minimum.
template <int VW, bool MIN = false>
__device__ __forceinline__ MaxSum row_maxsum(const float* xr, int cols, float* scratch,
                                             float* row_min = nullptr) {
  MaxSum a{-INFINITY, 0.0f};
  float mn = INFINITY;
  if constexpr (VW == 4) {
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    const int nvec = cols >> 2;
    int v = threadIdx.x;
    for (; v + 3 * (int)blockDim.x < nvec; v += 4 * blockDim.x) {
      float q[16];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 t = ld_keep(x4 + v + u * blockDim.x);
        q[4 * u] = t.x; q[4 * u + 1] = t.y; q[4 * u + 2] = t.z; q[4 * u + 3] = t.w;
      }
      ms_fold<16, MIN>(a, q, &mn);
    }
    for (; v < nvec; v += blockDim.x) {
      const float4 t = ld_keep(x4 + v);
      const float q[4] = {t.x, t.y, t.z, t.w};
      ms_fold<4, MIN>(a, q, &mn);
    }
  } else {
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      const float q[1] = {ld_keep(xr + c)};
      ms_fold<1, MIN>(a, q, &mn);
    }
  }
  MaxSum r = block_maxsum(a, scratch);
  if (r.m == -INFINITY) r.s = NAN;
  if constexpr (MIN) {
    // scratch[66..98]: per-warp minima (block_maxsum's last barrier orders
    // this after its reads)
    mn = warp_min(mn);
    if ((threadIdx.x & 31) == 0) scratch[66 + (threadIdx.x >> 5)] = mn;
    __syncthreads();
    const int nw = (blockDim.x + 31) >> 5;
    float t = INFINITY;
    for (int w = 0; w < nw; ++w) t = fminf(t, scratch[66 + w]);
    *row_min = t;
    __syncthreads();
  }
  return r;
}

template <int VW, bool LOG>
__global__ void __launch_bounds__(512) softmax_fwd_kernel(const float* __restrict__ x,
                                                          float* __restrict__ y, int64_t rows,
                                                          int cols) {
  __shared__ float scratch[66];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * (int64_t)cols;
    float* yr = y + row * (int64_t)cols;
    const MaxSum st = row_maxsum<VW>(xr, cols, scratch);
    const float logs = LOG ? logf(st.s) : 0.0f;
    // exp(x - m) / s as exp(x - m) * (1/s): within one ulp of the quotient,
    // one multiply per element instead of a division
    const float inv = LOG ? 0.0f : __frcp_rn(st.s);
    if constexpr (VW == 4) {
      const float4* x4 = reinterpret_cast<const float4*>(xr);
      float4* y4 = reinterpret_cast<float4*>(yr);
      // one vector per iteration: four in flight measured slower here
      for (int v = threadIdx.x; v < (cols >> 2); v += blockDim.x) {
        const float4 q = ld_stream(x4 + v);
        float4 o;
        if constexpr (LOG) {
          o.x = (q.x - st.m) - logs; o.y = (q.y - st.m) - logs;
          o.z = (q.z - st.m) - logs; o.w = (q.w - st.m) - logs;
        } else {
          o.x = expf(q.x - st.m) * inv; o.y = expf(q.y - st.m) * inv;
          o.z = expf(q.z - st.m) * inv; o.w = expf(q.w - st.m) * inv;
        }
        st_stream(y4 + v, o);
      }
    } else {
      for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float q = ld_stream(xr + c);
        st_stream(yr + c, LOG ? (q - st.m) - logs : expf(q - st.m) * inv);
      }
    }
  }
}

template <int VW, bool LOG>
__global__ void __launch_bounds__(512) softmax_bwd_kernel(const float* __restrict__ y,
                                                          const float* __restrict__ dy,
                                                          float* __restrict__ dx, int64_t rows,
                                                          int cols) {
  __shared__ float scratch[33];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* yr = y + row * (int64_t)cols;
    const float* gr = dy + row * (int64_t)cols;
    float* dr = dx + row * (int64_t)cols;
    float acc = 0.0f;
    if constexpr (VW == 4) {
      const float4* y4 = reinterpret_cast<const float4*>(yr);
      const float4* g4 = reinterpret_cast<const float4*>(gr);
      auto add = [&](const float4& g, const float4& q) {
        if constexpr (LOG) acc += (g.x + g.y) + (g.z + g.w);
        else acc += (g.x * q.x + g.y * q.y) + (g.z * q.z + g.w * q.w);
      };
      const int nv = cols >> 2;
      int v = threadIdx.x;
      for (; v + 3 * (int)blockDim.x < nv; v += 4 * blockDim.x) {  // four vectors in flight
        float4 g[4], q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          g[u] = ld_keep(g4 + v + u * blockDim.x);
          q[u] = LOG ? g[u] : ld_keep(y4 + v + u * blockDim.x);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) add(g[u], q[u]);
      }
      for (; v < nv; v += blockDim.x) {
        const float4 g = ld_keep(g4 + v);
        add(g, LOG ? g : ld_keep(y4 + v));
      }
    } else {
      for (int c = threadIdx.x; c < cols; c += blockDim.x)
        acc += LOG ? ld_keep(gr + c) : ld_keep(gr + c) * ld_keep(yr + c);
    }
    const float sum = block_sum(acc, scratch);
    if constexpr (VW == 4) {
      const float4* y4 = reinterpret_cast<const float4*>(yr);
      const float4* g4 = reinterpret_cast<const float4*>(gr);
      float4* d4 = reinterpret_cast<float4*>(dr);
      auto out = [&](const float4& g, const float4& q) {
        float4 o;
        if constexpr (LOG) {
          o.x = g.x - expf(q.x) * sum; o.y = g.y - expf(q.y) * sum;
          o.z = g.z - expf(q.z) * sum; o.w = g.w - expf(q.w) * sum;
        } else {
          o.x = q.x * (g.x - sum); o.y = q.y * (g.y - sum);
          o.z = q.z * (g.z - sum); o.w = q.w * (g.w - sum);
        }
        return o;
      };
      const int nv = cols >> 2;
      int v = threadIdx.x;
      for (; v + 3 * (int)blockDim.x < nv; v += 4 * blockDim.x) {  // four vectors in flight
        float4 g[4], q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          g[u] = ld_stream(g4 + v + u * blockDim.x);
          q[u] = ld_stream(y4 + v + u * blockDim.x);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) st_stream(d4 + v + u * blockDim.x, out(g[u], q[u]));
      }
      for (; v < nv; v += blockDim.x) st_stream(d4 + v, out(ld_stream(g4 + v), ld_stream(y4 + v)));
    } else {
      for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float g = ld_stream(gr + c), q = ld_stream(yr + c);
        st_stream(dr + c, LOG ? g - expf(q) * sum : q * (g - sum));
      }
    }
  }
}

// Records the first bad target: flag[0] = 1, flag[1..2] = value, flag[3] = cols.
__device__ __forceinline__ void record_bad_index(int32_t* flag, int64_t value, int64_t size) {
  if (flag && atomicCAS(flag, 0, 1) == 0) {
    flag[1] = (int32_t)(uint32_t)((uint64_t)value & 0xffffffffu);
    flag[2] = (int32_t)(uint32_t)((uint64_t)value >> 32);
    flag[3] = (int32_t)size;
  }
}

// Resolves a target like numpy fancy indexing does for onehot[i, t]
// (negative values count from the end); -1 if out of range.
__device__ __forceinline__ int64_t resolve_target(int64_t t, int64_t cols) {
  const int64_t r = t < 0 ? t + cols : t;
  return (r >= 0 && r < cols) ? r : -1;
}

template <int VW>
__global__ void __launch_bounds__(512) ce_fwd_kernel(const float* __restrict__ x,
                                                     const int64_t* __restrict__ targets,
                                                     float* __restrict__ row_max,
                                                     float* __restrict__ row_sum,
                                                     float* __restrict__ row_nll, int64_t rows,
                                                     int cols, int32_t* err) {
  __shared__ float scratch[66 + 33];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * (int64_t)cols;
    float mn;
    const MaxSum st = row_maxsum<VW, true>(xr, cols, scratch, &mn);
    const int64_t t = resolve_target(targets[row], cols);
    // The reference picks ls_t through a one-hot product summed over the row,
    // and 0 * -inf is NaN: a -inf logit anywhere but the target makes the
    // picked value NaN.  Rows without -inf skip the check (mn, t are uniform).
    int other_ninf = 0;
    if (mn == -INFINITY && t >= 0) {
      int f = 0;
      for (int c = threadIdx.x; c < cols; c += blockDim.x) f |= (c != t && xr[c] == -INFINITY);
      other_ninf = __syncthreads_or(f);
    }
    if (threadIdx.x == 0) {
      float nll = NAN;
      if (t < 0) {
        record_bad_index(err, targets[row], cols);
      } else if (!other_ninf) {
        // ls_t = (x_t - m) - log(s); the picked value is -ls_t
        nll = -((xr[t] - st.m) - logf(st.s));
      }
      row_max[row] = st.m;
      row_sum[row] = st.s;
      row_nll[row] = nll;
    }
  }
}

// loss = -(sum_rows ls) / total_rows, folded in f64 by one CTA in a fixed order.
__global__ void __launch_bounds__(1024) ce_loss_kernel(const float* __restrict__ row_nll,
                                                       int64_t rows, int64_t total_rows,
                                                       float* __restrict__ loss) {
  __shared__ double scratch[33];
  double acc = 0.0;
  for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) acc += (double)row_nll[r];
  const double sum = block_sum(acc, scratch);
  if (threadIdx.x == 0) {
    // reference: mean = sum / M in f32, then neg (of the mean of ls = -nll)
    const float mean_ls = __fdiv_rn((float)(-sum), (float)total_rows);
    loss[0] = -mean_ls;
  }
}

template <int VW>
__global__ void __launch_bounds__(256) ce_bwd_kernel(const float* __restrict__ x,
                                                     const int64_t* __restrict__ targets,
                                                     const float* __restrict__ row_max,
                                                     const float* __restrict__ row_sum,
                                                     const float* __restrict__ grad_loss,
                                                     float* __restrict__ dx, int64_t rows,
                                                     int cols, float inv_total) {
  const float g = grad_loss ? __ldg(grad_loss) : 1.0f;
  const float gm = g * inv_total;  // mean VJP: g * (1/M)
  const int64_t nvec = (int64_t)rows * (cols / VW);
  const int vpr = cols / VW;  // vectors per row
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = v / vpr;
    const int c0 = (int)(v - row * vpr) * VW;
    const float m = __ldg(row_max + row);
    const float scale = gm * __fdiv_rn(1.0f, __ldg(row_sum + row));  // (g/M) * (1/s)
    const int64_t t = resolve_target(__ldg(targets + row), cols);
    if constexpr (VW == 4) {
      const float4 q = ld_stream(reinterpret_cast<const float4*>(x) + v);
      float4 o;
      o.x = scale * expf(q.x - m) + (c0 + 0 == t ? -gm : -0.0f);
      o.y = scale * expf(q.y - m) + (c0 + 1 == t ? -gm : -0.0f);
      o.z = scale * expf(q.z - m) + (c0 + 2 == t ? -gm : -0.0f);
      o.w = scale * expf(q.w - m) + (c0 + 3 == t ? -gm : -0.0f);
      st_stream(reinterpret_cast<float4*>(dx) + v, o);
    } else {
      const float q = ld_stream(x + v);
      st_stream(dx + v, scale * expf(q - m) + (c0 == t ? -gm : -0.0f));
    }
  }
}

// The same VJP for rows of at least kCeRowCols classes, laid out like the
// softmax kernels: one CTA per row at a time, so the row's max, 1/sum scale and
// target are loaded once per row instead of once per vector, and four float4
// vectors in flight per thread.  Each element's expression is the one
// ce_bwd_kernel evaluates, so the two give identical bits.
constexpr int kCeRowCols = 2048;

__global__ void __launch_bounds__(512) ce_bwd_rows_kernel(const float* __restrict__ x,
                                                          const int64_t* __restrict__ targets,
                                                          const float* __restrict__ row_max,
                                                          const float* __restrict__ row_sum,
                                                          const float* __restrict__ grad_loss,
                                                          float* __restrict__ dx, int64_t rows,
                                                          int cols, float inv_total) {
  const float g = grad_loss ? __ldg(grad_loss) : 1.0f;
  const float gm = g * inv_total;
  const int nv = cols >> 2;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float m = __ldg(row_max + row);
    const float scale = gm * __fdiv_rn(1.0f, __ldg(row_sum + row));
    const int64_t t = resolve_target(__ldg(targets + row), cols);
    const float4* x4 = reinterpret_cast<const float4*>(x + row * (int64_t)cols);
    float4* d4 = reinterpret_cast<float4*>(dx + row * (int64_t)cols);
    auto out = [&](const float4& q, int v) {
      const int c0 = 4 * v;
      float4 o;
      o.x = scale * expf(q.x - m) + (c0 + 0 == t ? -gm : -0.0f);
      o.y = scale * expf(q.y - m) + (c0 + 1 == t ? -gm : -0.0f);
      o.z = scale * expf(q.z - m) + (c0 + 2 == t ? -gm : -0.0f);
      o.w = scale * expf(q.w - m) + (c0 + 3 == t ? -gm : -0.0f);
      return o;
    };
    int v = threadIdx.x;
    for (; v + 3 * (int)blockDim.x < nv; v += 4 * blockDim.x) {
      float4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = ld_stream(x4 + v + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < 4; ++u) st_stream(d4 + v + u * blockDim.x, out(q[u], v + u * blockDim.x));
    }
    for (; v < nv; v += blockDim.x) st_stream(d4 + v, out(ld_stream(x4 + v), v));
  }
}

// ---- softmax / log_softmax over any dim of a strided view ---------------------
//
// The reference composes both over any `dim` (functional.py:211-222): max and
// sum along `dim` are Tensor::reduce strips (lib.rs:519-576), so every
// logical row -- one index of every other dim -- is reduced on its own.  Here
// a logical row r (r in [0, outer * inner), other dims in logical order) has
// its elements at x + row_off(r) + j * xs, j < len; the output y is dense in
// x's logical shape, so row r's element j lands at
// (r / inner) * len * inner + r % inner + j * inner.
//   inner == 1 (the reduced dim is the last logical dim, x not dense):
//     softmax_dim_rows_*: one CTA per row, as the contiguous row kernels;
//   inner > 1: softmax_dim_cols_*: a CTA takes 32 consecutive logical rows
//     (one per lane, so loads and stores of a warp are consecutive in memory
//     whenever the innermost other dim is) and its warps split `len`; the
//     per-warp (max, sum) partials are merged in warp order.
struct DimRows {
  int nd;                      // the other dims, collapsed, outermost first
  int64_t n[OXC_MAX_DIMS];     // their sizes
  int64_t st[OXC_MAX_DIMS];    // their strides in x (forward) or dy (backward)
  int64_t len, xs;             // length of the reduced dim, its stride in x / dy
  int64_t inner;               // product of the logical dims after the reduced one
};

__device__ __forceinline__ int64_t dim_row_off(const DimRows& g, int64_t r) {
  int64_t off = 0;
  for (int d = g.nd - 1; d >= 0; --d) {
    const int64_t q = r / g.n[d];
    off += (r - q * g.n[d]) * g.st[d];
    r = q;
  }
  return off;
}

__device__ __forceinline__ int64_t dim_out_off(const DimRows& g, int64_t r) {
  const int64_t o = r / g.inner;
  return o * g.len * g.inner + (r - o * g.inner);
}

template <bool LOG>
__global__ void __launch_bounds__(512) softmax_dim_rows_fwd_kernel(const float* __restrict__ x,
                                                                   float* __restrict__ y,
                                                                   DimRows g, int64_t rows) {
  __shared__ float scratch[66];
  const int64_t len = g.len, xs = g.xs;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + dim_row_off(g, row);
    float* yr = y + row * len;
    MaxSum a{-INFINITY, 0.0f};
    int64_t c = threadIdx.x;
    for (; c + 3 * (int64_t)blockDim.x < len; c += 4 * blockDim.x) {
      float q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = ld_keep(xr + (c + u * blockDim.x) * xs);
      ms_fold<4>(a, q);
    }
    for (; c < len; c += blockDim.x) {
      const float q[1] = {ld_keep(xr + c * xs)};
      ms_fold<1>(a, q);
    }
    MaxSum st = block_maxsum(a, scratch);
    if (st.m == -INFINITY) st.s = NAN;
    const float logs = LOG ? logf(st.s) : 0.0f;
    const float inv = LOG ? 0.0f : __frcp_rn(st.s);
    for (c = threadIdx.x; c < len; c += blockDim.x) {
      const float q = ld_keep(xr + c * xs);
      st_stream(yr + c, LOG ? (q - st.m) - logs : expf(q - st.m) * inv);
    }
  }
}

template <bool LOG>
__global__ void __launch_bounds__(512) softmax_dim_rows_bwd_kernel(const float* __restrict__ y,
                                                                   const float* __restrict__ dy,
                                                                   float* __restrict__ dx,
                                                                   DimRows g, int64_t rows) {
  __shared__ float scratch[33];
  const int64_t len = g.len, gs = g.xs;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* yr = y + row * len;
    const float* gr = dy + dim_row_off(g, row);
    float* dr = dx + row * len;
    float acc = 0.0f;
    for (int64_t c = threadIdx.x; c < len; c += blockDim.x)
      acc += LOG ? ld_keep(gr + c * gs) : ld_keep(gr + c * gs) * ld_keep(yr + c);
    const float sum = block_sum(acc, scratch);
    for (int64_t c = threadIdx.x; c < len; c += blockDim.x) {
      const float gv = ld_keep(gr + c * gs), q = ld_keep(yr + c);
      st_stream(dr + c, LOG ? gv - expf(q) * sum : q * (gv - sum));
    }
  }
}

constexpr int kDimMaxWarps = 32;

template <bool LOG>
__global__ void __launch_bounds__(1024) softmax_dim_cols_fwd_kernel(const float* __restrict__ x,
                                                                    float* __restrict__ y,
                                                                    DimRows g, int64_t rows) {
  __shared__ float pm[kDimMaxWarps][33], ps[kDimMaxWarps][33];
  const int lane = threadIdx.x, w = threadIdx.y, nw = blockDim.y;
  const int64_t len = g.len, xs = g.xs, inner = g.inner;
  for (int64_t r0 = (int64_t)blockIdx.x * 32; r0 < rows; r0 += (int64_t)gridDim.x * 32) {
    const int64_t r = r0 + lane;
    const bool live = r < rows;
    const float* xr = x + (live ? dim_row_off(g, r) : 0);
    MaxSum a{-INFINITY, 0.0f};
    if (live) {
      int64_t j = w;
      for (; j + 3 * nw < len; j += 4 * nw) {
        float q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) q[u] = ld_keep(xr + (j + u * nw) * xs);
        ms_fold<4>(a, q);
      }
      for (; j < len; j += nw) {
        const float q[1] = {ld_keep(xr + j * xs)};
        ms_fold<1>(a, q);
      }
    }
    pm[w][lane] = a.m;
    ps[w][lane] = a.s;
    __syncthreads();
    MaxSum t{-INFINITY, 0.0f};
    for (int k = 0; k < nw; ++k) t = ms_merge(t, MaxSum{pm[k][lane], ps[k][lane]});
    if (t.m == -INFINITY) t.s = NAN;
    __syncthreads();  // the partials are read; the next tile may overwrite them
    if (!live) continue;
    const float logs = LOG ? logf(t.s) : 0.0f;
    const float inv = LOG ? 0.0f : __frcp_rn(t.s);
    float* yr = y + dim_out_off(g, r);
    for (int64_t j = w; j < len; j += nw) {
      const float q = ld_keep(xr + j * xs);
      st_stream(yr + j * inner, LOG ? (q - t.m) - logs : expf(q - t.m) * inv);
    }
  }
}

template <bool LOG>
__global__ void __launch_bounds__(1024) softmax_dim_cols_bwd_kernel(const float* __restrict__ y,
                                                                    const float* __restrict__ dy,
                                                                    float* __restrict__ dx,
                                                                    DimRows g, int64_t rows) {
  __shared__ float ps[kDimMaxWarps][33];
  const int lane = threadIdx.x, w = threadIdx.y, nw = blockDim.y;
  const int64_t len = g.len, gs = g.xs, inner = g.inner;
  for (int64_t r0 = (int64_t)blockIdx.x * 32; r0 < rows; r0 += (int64_t)gridDim.x * 32) {
    const int64_t r = r0 + lane;
    const bool live = r < rows;
    const float* gr = dy + (live ? dim_row_off(g, r) : 0);
    const int64_t oo = live ? dim_out_off(g, r) : 0;
    const float* yr = y + oo;
    float acc = 0.0f;
    if (live)
      for (int64_t j = w; j < len; j += nw)
        acc += LOG ? ld_keep(gr + j * gs) : ld_keep(gr + j * gs) * ld_keep(yr + j * inner);
    ps[w][lane] = acc;
    __syncthreads();
    float sum = 0.0f;
    for (int k = 0; k < nw; ++k) sum += ps[k][lane];
    __syncthreads();
    if (!live) continue;
    float* dr = dx + oo;
    for (int64_t j = w; j < len; j += nw) {
      const float gv = ld_keep(gr + j * gs), q = ld_keep(yr + j * inner);
      st_stream(dr + j * inner, LOG ? gv - expf(q) * sum : q * (gv - sum));
    }
  }
}

// Fills g for a softmax over `dim` of `v` (shape/strides), the other dims
// collapsed where their strides chain.  Returns the logical row count.
static int64_t dim_rows(const oxc_view* v, int d, DimRows* g) {
  int64_t n[OXC_MAX_DIMS], st[OXC_MAX_DIMS];
  int k = 0;
  int64_t rows = 1;
  g->inner = 1;
  for (int i = 0; i < v->ndim; ++i) {
    if (i == d) continue;
    rows *= v->shape[i];
    if (i > d) g->inner *= v->shape[i];
    if (v->shape[i] == 1) continue;
    if (k > 0 && st[k - 1] == v->strides[i] * v->shape[i]) {
      n[k - 1] *= v->shape[i];
      st[k - 1] = v->strides[i];
      continue;
    }
    n[k] = v->shape[i];
    st[k] = v->strides[i];
    ++k;
  }
  if (k == 0) {  // a single logical row
    n[0] = 1;
    st[0] = 0;
    k = 1;
  }
  g->nd = k;
  for (int i = 0; i < k; ++i) {
    g->n[i] = n[i];
    g->st[i] = st[i];
  }
  g->len = v->shape[d];
  g->xs = v->strides[d];
  return rows;
}

static void dim_cols_launch_geometry(int64_t rows, int64_t len, dim3* grid, dim3* block) {
  const int64_t tiles = (rows + 31) / 32;
  const int64_t want_warps = (int64_t)sm_count() * 48;  // warps to keep HBM busy
  int64_t nw = (want_warps + tiles - 1) / tiles;
  nw = std::max<int64_t>(4, std::min<int64_t>(nw, kDimMaxWarps));
  nw = std::max<int64_t>(1, std::min<int64_t>(nw, len));
  *block = dim3(32, (unsigned)nw);
  const int64_t per_sm = std::max<int64_t>(1, 64 / nw);
  *grid = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)sm_count() * per_sm)));
}

static unsigned row_grid(int64_t rows) {
  const int64_t cap = (int64_t)sm_count() * 64;
  return (unsigned)(rows < cap ? rows : cap);
}

static int row_block(int64_t cols) { return cols >= 8192 ? 512 : cols >= 1024 ? 256 : 128; }

static oxc_status check_shape(const char* fn, int64_t rows, int64_t cols) {
  if (rows < 0 || cols < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative shape", fn);
  if (cols > 0x7fffffff)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: %s: rows wider than 2^31", fn);
  return OXC_OK;
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_softmax_fwd(const float* x, float* y, int64_t rows, int64_t cols, int32_t log,
                           void* stream) {
  oxc_status st = check_shape(log ? "log_softmax" : "softmax", rows, cols);
  if (st) return st;
  if (rows == 0 || cols == 0) return OXC_OK;
  if (!x || !y) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: softmax: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool v4 = cols % 4 == 0 && aligned16(x) && aligned16(y);
  const unsigned grid = row_grid(rows);
  const int block = row_block(cols);
  if (v4) {
    if (log) softmax_fwd_kernel<4, true><<<grid, block, 0, s>>>(x, y, rows, (int)cols);
    else softmax_fwd_kernel<4, false><<<grid, block, 0, s>>>(x, y, rows, (int)cols);
  } else {
    if (log) softmax_fwd_kernel<1, true><<<grid, block, 0, s>>>(x, y, rows, (int)cols);
    else softmax_fwd_kernel<1, false><<<grid, block, 0, s>>>(x, y, rows, (int)cols);
  }
  return check_launch("oxc_softmax_fwd");
}

oxc_status oxc_softmax_bwd(const float* y, const float* dy, float* dx, int64_t rows, int64_t cols,
                           int32_t log, void* stream) {
  oxc_status st = check_shape(log ? "log_softmax backward" : "softmax backward", rows, cols);
  if (st) return st;
  if (rows == 0 || cols == 0) return OXC_OK;
  if (!y || !dy || !dx)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: softmax backward: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool v4 = cols % 4 == 0 && aligned16(y) && aligned16(dy) && aligned16(dx);
  const unsigned grid = row_grid(rows);
  const int block = row_block(cols);
  if (v4) {
    if (log) softmax_bwd_kernel<4, true><<<grid, block, 0, s>>>(y, dy, dx, rows, (int)cols);
    else softmax_bwd_kernel<4, false><<<grid, block, 0, s>>>(y, dy, dx, rows, (int)cols);
  } else {
    if (log) softmax_bwd_kernel<1, true><<<grid, block, 0, s>>>(y, dy, dx, rows, (int)cols);
    else softmax_bwd_kernel<1, false><<<grid, block, 0, s>>>(y, dy, dx, rows, (int)cols);
  }
  return check_launch("oxc_softmax_bwd");
}

static oxc_status dim_check(const char* fn, const oxc_view* v, int64_t dim, int* d) {
  if (!v) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null view", fn);
  if (v->ndim < 0 || v->ndim > OXC_MAX_DIMS)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: %s: rank %d > %d", fn, v->ndim,
                OXC_MAX_DIMS);
  if (v->ndim == 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: dim %lld out of range for 0-D tensor",
                (long long)dim);
  const int64_t dd = dim < 0 ? dim + v->ndim : dim;
  if (dd < 0 || dd >= v->ndim)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: dim %lld out of range for %d-D tensor",
                (long long)dim, v->ndim);
  for (int i = 0; i < v->ndim; ++i)
    if (v->shape[i] < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative dim", fn);
  if (v->shape[dd] == 0)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: cannot compute max/min over a zero-length dim");
  *d = (int)dd;
  return OXC_OK;
}

oxc_status oxc_softmax_dim_fwd(const oxc_view* x, int64_t dim, int32_t log, float* y,
                               void* stream) {
  const char* fn = log ? "log_softmax" : "softmax";
  int d = 0;
  oxc_status st = dim_check(fn, x, dim, &d);
  if (st) return st;
  DimRows g;
  const int64_t rows = dim_rows(x, d, &g);
  if (rows == 0) return OXC_OK;
  if (!x->data || !y) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // dense rows along the last dim: the contiguous row kernels
  if (g.inner == 1 && g.xs == 1 && g.nd == 1 && (g.st[0] == g.len || rows == 1))
    return oxc_softmax_fwd(x->data, y, rows, g.len, log, stream);
  if (g.inner == 1) {
    const unsigned grid = row_grid(rows);
    const int block = row_block(g.len);
    if (log) softmax_dim_rows_fwd_kernel<true><<<grid, block, 0, s>>>(x->data, y, g, rows);
    else softmax_dim_rows_fwd_kernel<false><<<grid, block, 0, s>>>(x->data, y, g, rows);
    return check_launch("oxc_softmax_dim_fwd");
  }
  dim3 grid, block;
  dim_cols_launch_geometry(rows, g.len, &grid, &block);
  if (log) softmax_dim_cols_fwd_kernel<true><<<grid, block, 0, s>>>(x->data, y, g, rows);
  else softmax_dim_cols_fwd_kernel<false><<<grid, block, 0, s>>>(x->data, y, g, rows);
  return check_launch("oxc_softmax_dim_fwd");
}

oxc_status oxc_softmax_dim_bwd(const float* y, const oxc_view* dy, int64_t dim, int32_t log,
                               float* dx, void* stream) {
  const char* fn = log ? "log_softmax backward" : "softmax backward";
  int d = 0;
  oxc_status st = dim_check(fn, dy, dim, &d);
  if (st) return st;
  DimRows g;
  const int64_t rows = dim_rows(dy, d, &g);
  if (rows == 0) return OXC_OK;
  if (!y || !dy->data || !dx)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (g.inner == 1 && g.xs == 1 && g.nd == 1 && (g.st[0] == g.len || rows == 1))
    return oxc_softmax_bwd(y, dy->data, dx, rows, g.len, log, stream);
  if (g.inner == 1) {
    const unsigned grid = row_grid(rows);
    const int block = row_block(g.len);
    if (log) softmax_dim_rows_bwd_kernel<true><<<grid, block, 0, s>>>(y, dy->data, dx, g, rows);
    else softmax_dim_rows_bwd_kernel<false><<<grid, block, 0, s>>>(y, dy->data, dx, g, rows);
    return check_launch("oxc_softmax_dim_bwd");
  }
  dim3 grid, block;
  dim_cols_launch_geometry(rows, g.len, &grid, &block);
  if (log) softmax_dim_cols_bwd_kernel<true><<<grid, block, 0, s>>>(y, dy->data, dx, g, rows);
  else softmax_dim_cols_bwd_kernel<false><<<grid, block, 0, s>>>(y, dy->data, dx, g, rows);
  return check_launch("oxc_softmax_dim_bwd");
}

oxc_status oxc_cross_entropy_fwd(const float* logits, const int64_t* targets, float* loss,
                                 float* row_max, float* row_sum, float* row_nll, int64_t rows,
                                 int64_t cols, int64_t total_rows, int32_t* err_flag,
                                 void* stream) {
  oxc_status st = check_shape("cross_entropy", rows, cols);
  if (st) return st;
  if (total_rows < rows || total_rows <= 0)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: cross_entropy: total_rows %lld must cover the %lld local rows",
                (long long)total_rows, (long long)rows);
  if (cols == 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: cross_entropy over zero classes");
  if (!logits || !targets || !loss || !row_max || !row_sum || !row_nll)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: cross_entropy: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows > 0) {
    const bool v4 = cols % 4 == 0 && aligned16(logits);
    const unsigned grid = row_grid(rows);
    // at most 256 threads per row: this single read-only pass gains from more
    // rows in flight per SM (B200, [32768, 32000]: 5.8 TB/s at 512 threads,
    // 6.8 at 128, 6.9 at 256); the two-pass softmax kernels keep 512, whose
    // second pass needs its rows to stay in L2
    const int block = std::min(row_block(cols), 256);
    if (v4)
      ce_fwd_kernel<4><<<grid, block, 0, s>>>(logits, targets, row_max, row_sum, row_nll, rows,
                                              (int)cols, err_flag);
    else
      ce_fwd_kernel<1><<<grid, block, 0, s>>>(logits, targets, row_max, row_sum, row_nll, rows,
                                              (int)cols, err_flag);
    st = check_launch("oxc_cross_entropy_fwd");
    if (st) return st;
  }
  ce_loss_kernel<<<1, 1024, 0, s>>>(row_nll, rows, total_rows, loss);
  return check_launch("oxc_cross_entropy_fwd (loss)");
}

oxc_status oxc_cross_entropy_bwd(const float* logits, const int64_t* targets,
                                 const float* row_max, const float* row_sum,
                                 const float* grad_loss, float* dlogits, int64_t rows,
                                 int64_t cols, int64_t total_rows, void* stream) {
  oxc_status st = check_shape("cross_entropy backward", rows, cols);
  if (st) return st;
  if (total_rows < rows || total_rows <= 0)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: cross_entropy backward: total_rows must cover the local rows");
  if (rows == 0 || cols == 0) return OXC_OK;
  if (!logits || !targets || !row_max || !row_sum || !dlogits)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: cross_entropy backward: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool v4 = cols % 4 == 0 && aligned16(logits) && aligned16(dlogits);
  const float inv_total = 1.0f / (float)total_rows;  // the mean VJP's 1/M (f32)
  if (v4 && cols >= kCeRowCols) {
    ce_bwd_rows_kernel<<<row_grid(rows), row_block(cols), 0, s>>>(
        logits, targets, row_max, row_sum, grad_loss, dlogits, rows, (int)cols, inv_total);
    return check_launch("oxc_cross_entropy_bwd");
  }
  const int block = 256;
  const int64_t work = rows * (v4 ? cols / 4 : cols);
  const int64_t cap = (int64_t)sm_count() * 8 * 4;  // 8 CTAs of 256 per SM, 4 waves of ILP
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + block - 1) / block, cap));
  if (v4)
    ce_bwd_kernel<4><<<grid, block, 0, s>>>(logits, targets, row_max, row_sum, grad_loss, dlogits,
                                            rows, (int)cols, inv_total);
  else
    ce_bwd_kernel<1><<<grid, block, 0, s>>>(logits, targets, row_max, row_sum, grad_loss, dlogits,
                                            rows, (int)cols, inv_total);
  return check_launch("oxc_cross_entropy_bwd");
}

}  // extern "C"
