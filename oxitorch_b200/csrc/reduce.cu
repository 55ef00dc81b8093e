// reduce.cu -- Tensor::reduce (dim / keepdim) and whole-tensor reductions.
//
// Reference: crates/oxi-tensor/src/lib.rs:519-576 (reduce), 582-604 (sum_all,
// mean_all, norm), ReduceKind::reduce_strip (ops.rs:246-285):
//   sum   left-to-right f32 fold;           mean = sum / len (f32)
//   max   fold(-inf, f32::max)  (NaN ignored; all-NaN -> -inf), min likewise
//   argmax first index of the maximum (`v > best` from data[0]: NaN never wins,
//          and a NaN at index 0 keeps index 0); argmin likewise
//   norm  sqrt(sum(v*v))
// Results are f32; argmax/argmin indices are returned as f32 values, the
// reference's carrier (lib.rs:568-572).  Empty strips: sum/mean/norm give 0,
// max/min/arg* are rejected on the host (InvalidArgument), as in the reference.
//
// Kernels (HBM-bound):
//   row:    the reduced dim has stride 1 -- a CTA (long strips) or a warp per
//           output, 128-bit loads when aligned, fixed-order tree combine;
//   column: otherwise -- one thread per output, walking the strip in index
//           order (for sum/mean/norm that is the reference's own left-to-right
//           fold, bit for bit); threads of a warp own neighbouring outputs so
//           the loads coalesce; long strips over few outputs are cut into
//           segments whose partials a finisher combines in segment order;
//   all:    whole-tensor, two stages with f64 partials for sum/mean/norm;
//   VJPs:   broadcast / scale / scatter / norm-ratio kernels writing dx dense.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace oxc {

enum RKind { RK_SUM = 0, RK_MEAN, RK_MAX, RK_MIN, RK_ARGMAX, RK_ARGMIN, RK_NORM };

// Partial result of a reduction: value (f32 or f64 sum) and index.
struct RAcc {
  double s;    // sum / sum of squares (f64 for whole-tensor), or unused
  float v;     // max/min/arg value; sum for the f32 paths
  int64_t i;   // arg index; -1 = nothing seen
};

__device__ __forceinline__ bool better(int kind, float v, int64_t i, float bv, int64_t bi) {
  if (isnan(v)) return false;
  if (bi < 0) return true;
  if (kind == RK_ARGMAX || kind == RK_MAX) return v > bv || (v == bv && i < bi);
  return v < bv || (v == bv && i < bi);
}

// ---- row mode ---------------------------------------------------------------------

struct Layout {
  int nd;                      // non-reduced dims (collapsed)
  int64_t n[OXC_MAX_DIMS];
  int64_t st[OXC_MAX_DIMS];
  int64_t len;                 // strip length
  int64_t sd;                  // strip stride
};

__device__ __forceinline__ int64_t base_offset(const Layout& L, int64_t o) {
  int64_t off = 0;
  for (int d = L.nd - 1; d >= 0; --d) {
    const int64_t q = o / L.n[d];
    off += (o - q * L.n[d]) * L.st[d];
    o = q;
  }
  return off;
}

__device__ __forceinline__ float finish(int kind, float sum_or_v, int64_t idx, int64_t len) {
  switch (kind) {
    case RK_SUM: return sum_or_v;
    case RK_MEAN: return len ? __fdiv_rn(sum_or_v, (float)len) : 0.0f;
    case RK_NORM: return __fsqrt_rn(sum_or_v);
    case RK_ARGMAX: case RK_ARGMIN: return (float)(idx < 0 ? 0 : idx);
    default: return sum_or_v;
  }
}

// Per-element step of a row reduction, specialised on the kind.  A thread
// scans its elements in increasing index order, so for argmax/argmin a strict
// compare keeps the first occurrence; NaN never compares and is skipped unless
// nothing else has been seen (f32::max's NaN-ignoring fold).
template <int KIND>
__device__ __forceinline__ void rpush(float& acc, float& bv, int64_t& bi, float x, int64_t j) {
  if constexpr (KIND == RK_NORM) {
    acc = __fadd_rn(acc, __fmul_rn(x, x));
  } else if constexpr (KIND == RK_SUM || KIND == RK_MEAN) {
    acc = __fadd_rn(acc, x);
  } else if constexpr (KIND == RK_MAX) {
    acc = fmaxf(acc, x);
  } else if constexpr (KIND == RK_MIN) {
    acc = fminf(acc, x);
  } else {
    const bool take = KIND == RK_ARGMAX ? x > bv : x < bv;
    if (take || (bi < 0 && !isnan(x))) { bv = x; bi = j; }
  }
}

template <int KIND>
__device__ __forceinline__ void rcombine(float& acc, float& bv, int64_t& bi, float oa, float ov,
                                         int64_t oi) {
  if constexpr (KIND == RK_SUM || KIND == RK_MEAN || KIND == RK_NORM) acc = __fadd_rn(acc, oa);
  else if constexpr (KIND == RK_MAX) acc = fmaxf(acc, oa);
  else if constexpr (KIND == RK_MIN) acc = fminf(acc, oa);
  else if (oi >= 0 && better(KIND, ov, oi, bv, bi)) { bv = ov; bi = oi; }
}

// One CTA (WARPS = blockDim/32 warps) or one warp per output; strip contiguous
// (or any stride, scalar loads).  128-bit loads, four in flight per thread.
template <int KIND, bool PER_WARP>
__global__ void __launch_bounds__(256) reduce_row_kernel(const float* __restrict__ in, Layout L,
                                                         int64_t nout, float* __restrict__ out) {
  __shared__ float sv[33];
  __shared__ long long si[33];
  constexpr bool kArg = KIND == RK_ARGMAX || KIND == RK_ARGMIN;
  constexpr bool kSum = KIND == RK_SUM || KIND == RK_MEAN || KIND == RK_NORM;
  constexpr float kInit = kSum ? 0.0f : (KIND == RK_MAX || KIND == RK_ARGMAX ? -INFINITY : INFINITY);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int lanes = PER_WARP ? 32 : blockDim.x;
  const int tid = PER_WARP ? lane : threadIdx.x;
  const int64_t per_block = PER_WARP ? blockDim.x / 32 : 1;
  for (int64_t o0 = (int64_t)blockIdx.x * per_block; o0 < nout; o0 += (int64_t)gridDim.x * per_block) {
    const int64_t o = o0 + (PER_WARP ? warp : 0);
    float acc = kInit, bv = kInit;
    int64_t bi = -1;
    if (o < nout) {
      const float* p = in + base_offset(L, o);
      const bool v4 = L.sd == 1 && (reinterpret_cast<uintptr_t>(p) & 15) == 0;
      int64_t j0 = 0;
      if (v4) {
        const float4* p4 = reinterpret_cast<const float4*>(p);
        const int64_t nv = L.len / 4;
        int64_t v = tid;
        for (; v + 3 * lanes < nv; v += 4 * lanes) {
          float4 q[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) q[u] = ld_stream(p4 + v + u * lanes);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int64_t j = 4 * (v + u * lanes);
            rpush<KIND>(acc, bv, bi, q[u].x, j);
            rpush<KIND>(acc, bv, bi, q[u].y, j + 1);
            rpush<KIND>(acc, bv, bi, q[u].z, j + 2);
            rpush<KIND>(acc, bv, bi, q[u].w, j + 3);
          }
        }
        for (; v < nv; v += lanes) {
          const float4 q = ld_stream(p4 + v);
          rpush<KIND>(acc, bv, bi, q.x, 4 * v);
          rpush<KIND>(acc, bv, bi, q.y, 4 * v + 1);
          rpush<KIND>(acc, bv, bi, q.z, 4 * v + 2);
          rpush<KIND>(acc, bv, bi, q.w, 4 * v + 3);
        }
        j0 = nv * 4;
      }
      for (int64_t j = j0 + tid; j < L.len; j += lanes) rpush<KIND>(acc, bv, bi, ld_stream(p + j * L.sd), j);
    }
    // warp combine (fixed order)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float oa = __shfl_xor_sync(0xffffffffu, acc, off);
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const long long oi = __shfl_xor_sync(0xffffffffu, (long long)bi, off);
      rcombine<KIND>(acc, bv, bi, oa, ov, oi);
    }
    if (!PER_WARP) {
      __syncthreads();
      if (lane == 0) { sv[warp] = kArg ? bv : acc; si[warp] = bi; }
      __syncthreads();
      if (warp == 0) {
        const int nw = blockDim.x / 32;
        float a2 = lane < nw ? sv[lane] : kInit;
        int64_t i2 = lane < nw ? si[lane] : -1;
        float b2 = a2;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          const float oa = __shfl_xor_sync(0xffffffffu, kArg ? b2 : a2, off);
          const long long oi = __shfl_xor_sync(0xffffffffu, (long long)i2, off);
          rcombine<KIND>(a2, b2, i2, oa, oa, oi);
        }
        acc = a2;
        bi = i2;
      }
    }
    if ((PER_WARP ? lane == 0 : threadIdx.x == 0) && o < nout) {
      if (kArg) {
        // a NaN at index 0 keeps index 0 (the reference starts from data[0])
        const float first = in[base_offset(L, o)];
        out[o] = isnan(first) ? 0.0f : finish(KIND, 0.0f, bi, L.len);
      } else {
        out[o] = finish(KIND, acc, -1, L.len);
      }
    }
    if (!PER_WARP) __syncthreads();
  }
}

template <bool PER_WARP>
static void launch_reduce_row(int kind, unsigned grid, cudaStream_t s, const float* in,
                              const Layout& L, int64_t nout, float* out) {
  switch (kind) {
    case RK_SUM: reduce_row_kernel<RK_SUM, PER_WARP><<<grid, 256, 0, s>>>(in, L, nout, out); break;
    case RK_MEAN: reduce_row_kernel<RK_MEAN, PER_WARP><<<grid, 256, 0, s>>>(in, L, nout, out); break;
    case RK_MAX: reduce_row_kernel<RK_MAX, PER_WARP><<<grid, 256, 0, s>>>(in, L, nout, out); break;
    case RK_MIN: reduce_row_kernel<RK_MIN, PER_WARP><<<grid, 256, 0, s>>>(in, L, nout, out); break;
    case RK_ARGMAX: reduce_row_kernel<RK_ARGMAX, PER_WARP><<<grid, 256, 0, s>>>(in, L, nout, out); break;
    case RK_ARGMIN: reduce_row_kernel<RK_ARGMIN, PER_WARP><<<grid, 256, 0, s>>>(in, L, nout, out); break;
    default: reduce_row_kernel<RK_NORM, PER_WARP><<<grid, 256, 0, s>>>(in, L, nout, out); break;
  }
}

// ---- column mode ------------------------------------------------------------------

// Thread per (output, segment): folds strip elements [seg*seglen, ...) in
// index order.  nseg == 1 writes the result; else writes partials.
__global__ void __launch_bounds__(256) reduce_col_kernel(int kind, const float* __restrict__ in,
                                                         Layout L, int64_t nout, int64_t nseg,
                                                         int64_t seglen, float* __restrict__ out,
                                                         float* __restrict__ pv,
                                                         long long* __restrict__ pi) {
  const int64_t total = nout * nseg;
  const bool sumlike = kind == RK_SUM || kind == RK_MEAN || kind == RK_NORM;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t seg = t / nout, o = t - seg * nout;
    const float* p = in + base_offset(L, o);
    const int64_t j0 = seg * seglen, j1 = min(L.len, j0 + seglen);
    float acc = sumlike ? -0.0f : (kind == RK_MAX || kind == RK_ARGMAX ? -INFINITY : INFINITY);
    float bv = 0.0f;
    int64_t bi = -1;
    int64_t j = j0;
    for (; j + 3 < j1; j += 4) {
      float x[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) x[k] = __ldg(p + (j + k) * L.sd);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (kind == RK_NORM) acc = __fadd_rn(acc, __fmul_rn(x[k], x[k]));
        else if (sumlike) acc = __fadd_rn(acc, x[k]);
        else if (kind == RK_MAX) acc = fmaxf(acc, x[k]);
        else if (kind == RK_MIN) acc = fminf(acc, x[k]);
        else if (better(kind, x[k], j + k, bv, bi)) { bv = x[k]; bi = j + k; }
      }
    }
    for (; j < j1; ++j) {
      const float x = __ldg(p + j * L.sd);
      if (kind == RK_NORM) acc = __fadd_rn(acc, __fmul_rn(x, x));
      else if (sumlike) acc = __fadd_rn(acc, x);
      else if (kind == RK_MAX) acc = fmaxf(acc, x);
      else if (kind == RK_MIN) acc = fminf(acc, x);
      else if (better(kind, x, j, bv, bi)) { bv = x; bi = j; }
    }
    if (nseg == 1) {
      if (kind == RK_ARGMAX || kind == RK_ARGMIN)
        out[o] = (L.len > 0 && isnan(p[0])) ? 0.0f : finish(kind, 0.0f, bi, L.len);
      else
        out[o] = finish(kind, acc, -1, L.len);
    } else {
      pv[t] = (kind == RK_ARGMAX || kind == RK_ARGMIN) ? bv : acc;
      pi[t] = bi;
    }
  }
}

__global__ void __launch_bounds__(256) reduce_col_finish_kernel(int kind, const float* __restrict__ in,
                                                                Layout L, int64_t nout, int64_t nseg,
                                                                const float* __restrict__ pv,
                                                                const long long* __restrict__ pi,
                                                                float* __restrict__ out) {
  const bool sumlike = kind == RK_SUM || kind == RK_MEAN || kind == RK_NORM;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < nout;
       o += (int64_t)gridDim.x * blockDim.x) {
    float acc = sumlike ? -0.0f : (kind == RK_MAX || kind == RK_ARGMAX ? -INFINITY : INFINITY);
    float bv = 0.0f;
    int64_t bi = -1;
    for (int64_t seg = 0; seg < nseg; ++seg) {
      const float v = pv[seg * nout + o];
      const int64_t i = pi[seg * nout + o];
      if (sumlike) acc = __fadd_rn(acc, v);
      else if (kind == RK_MAX) acc = fmaxf(acc, v);
      else if (kind == RK_MIN) acc = fminf(acc, v);
      else if (i >= 0 && better(kind, v, i, bv, bi)) { bv = v; bi = i; }
    }
    if (kind == RK_ARGMAX || kind == RK_ARGMIN)
      out[o] = (L.len > 0 && isnan(in[base_offset(L, o)])) ? 0.0f : finish(kind, 0.0f, bi, L.len);
    else
      out[o] = finish(kind, acc, -1, L.len);
  }
}

// ---- whole tensor ------------------------------------------------------------------

struct Flat {
  int nd;
  int64_t n[OXC_MAX_DIMS];
  int64_t st[OXC_MAX_DIMS];
};

__device__ __forceinline__ int64_t flat_offset(const Flat& f, int64_t i) {
  int64_t off = 0;
  for (int d = f.nd - 1; d >= 0; --d) {
    const int64_t q = i / f.n[d];
    off += (i - q * f.n[d]) * f.st[d];
    i = q;
  }
  return off;
}

// Stage 1: CTA b reduces logical indices [b*chunk, ...) into part[b].
__global__ void __launch_bounds__(256) reduce_all_stage1(int kind, const float* __restrict__ in,
                                                         Flat f, int64_t n, int64_t chunk,
                                                         double* __restrict__ ps,
                                                         float* __restrict__ pv,
                                                         long long* __restrict__ pi) {
  __shared__ double sd[33];
  __shared__ float sv[33];
  __shared__ long long si[33];
  const int64_t i0 = (int64_t)blockIdx.x * chunk, i1 = min(n, i0 + chunk);
  const bool dense = f.nd == 1 && f.st[0] == 1;
  const bool sumlike = kind == RK_SUM || kind == RK_MEAN || kind == RK_NORM;
  double acc = 0.0;
  float bv = (kind == RK_MAX || kind == RK_ARGMAX) ? -INFINITY : INFINITY;
  int64_t bi = -1;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const float x = dense ? ld_stream(in + i) : __ldg(in + flat_offset(f, i));
    if (kind == RK_NORM) acc += (double)x * (double)x;
    else if (sumlike) acc += (double)x;
    else if (kind == RK_MAX) bv = fmaxf(bv, x);
    else if (kind == RK_MIN) bv = fminf(bv, x);
    else if (better(kind, x, i, bv, bi)) { bv = x; bi = i; }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const double oa = __shfl_xor_sync(0xffffffffu, acc, off);
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const long long oi = __shfl_xor_sync(0xffffffffu, (long long)bi, off);
    acc += oa;
    if (kind == RK_MAX) bv = fmaxf(bv, ov);
    else if (kind == RK_MIN) bv = fminf(bv, ov);
    else if ((kind == RK_ARGMAX || kind == RK_ARGMIN) && oi >= 0 && better(kind, ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { sd[warp] = acc; sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0;
    float v = (kind == RK_MAX || kind == RK_ARGMAX) ? -INFINITY : INFINITY;
    long long b = -1;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) {
      a += sd[w];
      if (kind == RK_MAX) v = fmaxf(v, sv[w]);
      else if (kind == RK_MIN) v = fminf(v, sv[w]);
      else if ((kind == RK_ARGMAX || kind == RK_ARGMIN) && si[w] >= 0 && better(kind, sv[w], si[w], v, b)) { v = sv[w]; b = si[w]; }
    }
    ps[blockIdx.x] = a;
    pv[blockIdx.x] = v;
    pi[blockIdx.x] = b;
  }
}

__global__ void reduce_all_stage2(int kind, const float* __restrict__ in, Flat f, int64_t n,
                                  int64_t nparts, const double* __restrict__ ps,
                                  const float* __restrict__ pv, const long long* __restrict__ pi,
                                  float* __restrict__ out, double* __restrict__ out64) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double a = 0.0;
  float v = (kind == RK_MAX || kind == RK_ARGMAX) ? -INFINITY : INFINITY;
  long long b = -1;
  for (int64_t p = 0; p < nparts; ++p) {
    a += ps[p];
    if (kind == RK_MAX) v = fmaxf(v, pv[p]);
    else if (kind == RK_MIN) v = fminf(v, pv[p]);
    else if ((kind == RK_ARGMAX || kind == RK_ARGMIN) && pi[p] >= 0 && better(kind, pv[p], pi[p], v, b)) { v = pv[p]; b = pi[p]; }
  }
  double r64 = a;
  float r;
  switch (kind) {
    case RK_SUM: r = (float)a; break;
    case RK_MEAN: r64 = n ? a / (double)n : 0.0; r = n ? __fdiv_rn((float)a, (float)n) : 0.0f; break;
    case RK_NORM: r64 = sqrt(a); r = __fsqrt_rn((float)a); break;
    case RK_ARGMAX: case RK_ARGMIN:
      r = (n > 0 && isnan(in[flat_offset(f, 0)])) ? 0.0f : (float)(b < 0 ? 0 : b);
      r64 = r;
      break;
    default: r = v; r64 = v; break;
  }
  out[0] = r;
  if (out64) out64[0] = r64;
}

// Sum of squares over several tensors (clip_grad_norm_): stage 1 per chunk of
// each tensor, stage 2 in (tensor, chunk) order.
struct MultiViews {
  int count;
  const float* p[16];
  Flat f[16];
  int64_t n[16];
  int64_t first_part[17];
  int64_t chunk;
};

__global__ void __launch_bounds__(256) sumsq_multi_stage1(MultiViews mv, double* __restrict__ ps) {
  __shared__ double sd[33];
  const int64_t part = blockIdx.x;
  int t = 0;
  while (t + 1 < mv.count && part >= mv.first_part[t + 1]) ++t;
  const int64_t i0 = (part - mv.first_part[t]) * mv.chunk, i1 = min(mv.n[t], i0 + mv.chunk);
  const bool dense = mv.f[t].nd == 1 && mv.f[t].st[0] == 1;
  double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
  int64_t i = i0 + threadIdx.x;
  if (dense && (reinterpret_cast<uintptr_t>(mv.p[t] + i0) & 15) == 0) {
    // 128-bit loads, four independent f64 chains, 4 loads in flight per thread
    const float4* p4 = reinterpret_cast<const float4*>(mv.p[t] + i0);
    const int64_t nv = (i1 - i0) / 4;
    int64_t v = threadIdx.x;
    for (; v + 3 * (int64_t)blockDim.x < nv; v += 4 * blockDim.x) {
      float4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = ld_stream(p4 + v + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a0 = fma((double)q[u].x, (double)q[u].x, a0);
        a1 = fma((double)q[u].y, (double)q[u].y, a1);
        a2 = fma((double)q[u].z, (double)q[u].z, a2);
        a3 = fma((double)q[u].w, (double)q[u].w, a3);
      }
    }
    for (; v < nv; v += blockDim.x) {
      const float4 q = ld_stream(p4 + v);
      a0 = fma((double)q.x, (double)q.x, a0);
      a1 = fma((double)q.y, (double)q.y, a1);
      a2 = fma((double)q.z, (double)q.z, a2);
      a3 = fma((double)q.w, (double)q.w, a3);
    }
    i = i0 + nv * 4 + threadIdx.x;
  }
  for (; i < i1; i += blockDim.x) {
    const float x = dense ? ld_stream(mv.p[t] + i) : __ldg(mv.p[t] + flat_offset(mv.f[t], i));
    a0 = fma((double)x, (double)x, a0);
  }
  const double s = block_sum((a0 + a1) + (a2 + a3), sd);
  if (threadIdx.x == 0) ps[part] = s;
}

// Fixed-order block reduction of the stage-1 partials.
__global__ void __launch_bounds__(256) sumsq_multi_stage2(int64_t nparts, const double* __restrict__ ps,
                                                          double* __restrict__ out) {
  __shared__ double red[33];
  double a = 0.0;
  for (int64_t p = threadIdx.x; p < nparts; p += blockDim.x) a += ps[p];
  const double t = block_sum(a, red);
  if (threadIdx.x == 0) out[0] = t;
}

// ---- host helpers --------------------------------------------------------------------

static oxc_status check_view(const oxc_view* v, const char* fn) {
  if (!v) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null view", fn);
  if (v->ndim < 0 || v->ndim > OXC_MAX_DIMS)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: %s: rank %d", fn, v->ndim);
  for (int i = 0; i < v->ndim; ++i)
    if (v->shape[i] < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative dim", fn);
  return OXC_OK;
}

static Flat make_flat(const oxc_view* v, int64_t* n) {
  Flat f;
  f.nd = 0;
  *n = 1;
  for (int i = 0; i < v->ndim; ++i) *n *= v->shape[i];
  for (int i = 0; i < v->ndim; ++i) {
    if (v->shape[i] == 1) continue;
    if (f.nd > 0 && f.st[f.nd - 1] == v->strides[i] * v->shape[i]) {
      f.n[f.nd - 1] *= v->shape[i];
      f.st[f.nd - 1] = v->strides[i];
    } else {
      f.n[f.nd] = v->shape[i];
      f.st[f.nd] = v->strides[i];
      ++f.nd;
    }
  }
  if (f.nd == 0) { f.nd = 1; f.n[0] = 1; f.st[0] = 1; }
  return f;
}

struct ReducePlan {
  Layout L;
  int64_t nout;
  bool row;
  int64_t nseg, seglen;
};

static oxc_status plan_reduce(int32_t kind, const oxc_view* in, int64_t dim, int32_t keepdim,
                              const oxc_view* out, ReducePlan* P) {
  oxc_status st = check_view(in, "reduce");
  if (st) return st;
  const int nd = in->ndim;
  // layout::normalize_dim (layout.rs:162-179)
  int64_t d = dim < 0 ? nd + dim : dim;
  if (d < 0 || d >= nd)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: dim %lld out of range for %d-D tensor",
                (long long)dim, nd);
  const int64_t len = in->shape[d];
  if (len == 0 && (kind == RK_ARGMAX || kind == RK_ARGMIN))
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: cannot compute argmax/argmin over a zero-length dim");
  if (len == 0 && (kind == RK_MAX || kind == RK_MIN))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: cannot compute max/min over a zero-length dim");
  // expected output shape, dense row-major
  if ((st = check_view(out, "reduce output"))) return st;
  int64_t eshape[OXC_MAX_DIMS];
  int end = 0;
  for (int i = 0; i < nd; ++i) {
    if (i == d) { if (keepdim) eshape[end++] = 1; continue; }
    eshape[end++] = in->shape[i];
  }
  if (out->ndim != end)
    return fail(OXC_ERR_SHAPE_MISMATCH, "shape mismatch: reduce output rank %d vs %d", out->ndim, end);
  int64_t expect = 1;
  for (int i = end - 1; i >= 0; --i) {
    if (out->shape[i] != eshape[i])
      return fail(OXC_ERR_SHAPE_MISMATCH, "shape mismatch: reduce output dim %d", i);
    if (eshape[i] != 1 && out->strides[i] != expect)
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: reduce output must be contiguous");
    expect *= eshape[i];
  }
  P->nout = expect;
  // non-reduced dims, collapsed
  Layout& L = P->L;
  L.nd = 0;
  for (int i = 0; i < nd; ++i) {
    if (i == d || in->shape[i] == 1) continue;
    if (L.nd > 0 && L.st[L.nd - 1] == in->strides[i] * in->shape[i]) {
      L.n[L.nd - 1] *= in->shape[i];
      L.st[L.nd - 1] = in->strides[i];
    } else {
      L.n[L.nd] = in->shape[i];
      L.st[L.nd] = in->strides[i];
      ++L.nd;
    }
  }
  if (L.nd == 0) { L.nd = 1; L.n[0] = 1; L.st[0] = 0; }
  L.len = len;
  L.sd = in->strides[d];
  // row mode when the strip is contiguous or outputs are not contiguous in memory
  const bool inner_unit = L.st[L.nd - 1] == 1 && L.n[L.nd - 1] > 1;
  P->row = L.sd == 1 || !inner_unit;
  P->nseg = 1;
  P->seglen = len;
  if (!P->row) {
    const int64_t want = 64 * 1024;  // threads to keep HBM busy
    if (P->nout < want && len > 512) {
      int64_t nseg = std::min<int64_t>((want + P->nout - 1) / P->nout, (len + 255) / 256);
      nseg = std::max<int64_t>(nseg, 1);
      P->nseg = nseg;
      P->seglen = (len + nseg - 1) / nseg;
      P->nseg = (len + P->seglen - 1) / P->seglen;
    }
  }
  return OXC_OK;
}


// ---- reduce VJPs (crates/oxi-autograd/src/ops.rs:327-388) -------------------------
//
// dx has x's shape, dense; view it as [outer, len, inner] around the reduced
// dim; g and aux (argmax index or norm per strip) are dense [outer, inner].
//   sum:     dx = g                      (expand_to)
//   mean:    dx = g * rn,  rn = f32(1/len)  (expand_to, then mul_scalar(1.0 / n))
//   max/min: dx = g at the strip's first arg position, +0 elsewhere
//            (scatter_along_dim into zeros)
//   norm:    dx = g * (x / (norm + 1e-12))  (add_scalar, div, mul: three roundings)

struct XView {
  int nd;
  int64_t n[OXC_MAX_DIMS];
  int64_t st[OXC_MAX_DIMS];
};

// Offset of the element with dense row-major index j of x's shape.
__device__ __forceinline__ int64_t x_offset(const XView& X, int64_t j) {
  int64_t off = 0;
  for (int d = X.nd - 1; d >= 0; --d) {
    const int64_t q = j / X.n[d];
    off += (j - q * X.n[d]) * X.st[d];
    j = q;
  }
  return off;
}

template <int KIND>
__device__ __forceinline__ float reduce_vjp_elem(float gv, float aux, int64_t l, float xv, float rn) {
  if (KIND == RK_SUM) return gv;
  if (KIND == RK_MEAN) return __fmul_rn(gv, rn);
  if (KIND == RK_MAX) return l == (int64_t)aux ? gv : 0.0f;
  return __fmul_rn(gv, __fdiv_rn(xv, __fadd_rn(aux, 1e-12f)));  // RK_NORM
}

// inner > 1: a CTA walks rows t = o * len + l; its threads cover the inner
// index, so g, aux and dx are read and written contiguously.
template <int KIND>
__global__ void __launch_bounds__(256) reduce_vjp_rows_kernel(
    const float* __restrict__ x, XView X, bool xdense, const float* __restrict__ g,
    const float* __restrict__ aux, float* __restrict__ dx, int64_t nrows, int64_t len,
    int64_t inner, float rn) {
  for (int64_t t = blockIdx.x; t < nrows; t += gridDim.x) {
    const int64_t o = t / len, l = t - o * len;
    const float* gr = g + o * inner;
    const float* ar = aux ? aux + o * inner : nullptr;
    float* dr = dx + t * inner;
    for (int64_t i = threadIdx.x; i < inner; i += blockDim.x) {
      float xv = 0.0f;
      if (KIND == RK_NORM) xv = __ldg(x + (xdense ? t * inner + i : x_offset(X, t * inner + i)));
      dr[i] = reduce_vjp_elem<KIND>(__ldg(gr + i), ar ? __ldg(ar + i) : 0.0f, l, xv, rn);
    }
  }
}

// inner == 1 (the reduced dim is the last one): elementwise over dx.
template <int KIND>
__global__ void __launch_bounds__(256) reduce_vjp_last_kernel(
    const float* __restrict__ x, XView X, bool xdense, const float* __restrict__ g,
    const float* __restrict__ aux, float* __restrict__ dx, int64_t total, int64_t len, float rn) {
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < total;
       j += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = j / len, l = j - s * len;
    float xv = 0.0f;
    if (KIND == RK_NORM) xv = __ldg(x + (xdense ? j : x_offset(X, j)));
    dx[j] = reduce_vjp_elem<KIND>(__ldg(g + s), aux ? __ldg(aux + s) : 0.0f, l, xv, rn);
  }
}

}  // namespace oxc

using namespace oxc;

extern "C" {

size_t oxc_reduce_workspace_size(int32_t kind, const oxc_view* in, int64_t dim) {
  if (!in || in->ndim <= 0) return 0;
  // plan against a fake keepdim output
  oxc_view out;
  out.data = nullptr;
  out.ndim = in->ndim;
  int64_t d = dim < 0 ? in->ndim + dim : dim;
  if (d < 0 || d >= in->ndim) return 0;
  int64_t expect = 1;
  for (int i = in->ndim - 1; i >= 0; --i) {
    out.shape[i] = i == d ? 1 : in->shape[i];
    out.strides[i] = expect;
    expect *= out.shape[i];
  }
  ReducePlan P;
  if (plan_reduce(kind, in, dim, 1, &out, &P) != OXC_OK) { clear_error(); return 0; }
  if (P.row || P.nseg == 1) return 0;
  return (size_t)P.nseg * P.nout * (sizeof(float) + sizeof(long long)) + 256;
}

oxc_status oxc_reduce(int32_t kind, const oxc_view* in, int64_t dim, int32_t keepdim,
                      const oxc_view* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (kind < 0 || kind > 6)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown reduction kind %d", kind);
  ReducePlan P;
  oxc_status st = plan_reduce(kind, in, dim, keepdim, out, &P);
  if (st) return st;
  if (P.nout == 0) return OXC_OK;
  if (!out->data || (P.L.len > 0 && !in->data))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: reduce: null data");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t cap = (int64_t)sm_count() * 16;
  if (P.L.len == 0) {  // empty strips: sum/mean/norm -> 0
    cudaError_t e = cudaMemsetAsync(out->data, 0, (size_t)P.nout * sizeof(float), s);
    return e == cudaSuccess ? OXC_OK : cuda_fail(e, "oxc_reduce");
  }
  if (P.row) {
    // A warp per output whenever there are enough outputs to fill the GPU
    // with warps (64 per SM): no block barrier per output, and many rows in
    // flight per SM.  On B200 over [65536, 11008] this ran sum / max / argmax at
    // 6.7 / 6.8 / 6.6 TB/s against 5.4 / 5.5 / 4.8 with a 256-thread CTA per
    // row.  Long rows with few outputs keep a CTA per output.
    if (P.L.len >= 2048 && P.nout < (int64_t)sm_count() * 64) {
      launch_reduce_row<false>(kind, (unsigned)std::min<int64_t>(P.nout, cap), s, in->data, P.L,
                               P.nout, out->data);
    } else {
      const int64_t blocks = (P.nout + 7) / 8;
      launch_reduce_row<true>(kind, (unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks, cap)),
                              s, in->data, P.L, P.nout, out->data);
    }
    return check_launch("oxc_reduce");
  }
  const int64_t total = P.nout * P.nseg;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, cap));
  if (P.nseg == 1) {
    reduce_col_kernel<<<grid, 256, 0, s>>>(kind, in->data, P.L, P.nout, 1, P.seglen, out->data,
                                           nullptr, nullptr);
    return check_launch("oxc_reduce");
  }
  const size_t need = (size_t)P.nseg * P.nout * (sizeof(float) + sizeof(long long)) + 256;
  if (!workspace || workspace_bytes < need)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: reduce needs a %zu-byte workspace (oxc_reduce_workspace_size), got %zu",
                need, workspace_bytes);
  long long* pi = reinterpret_cast<long long*>((reinterpret_cast<uintptr_t>(workspace) + 15) & ~uintptr_t(15));
  float* pv = reinterpret_cast<float*>(pi + total);
  reduce_col_kernel<<<grid, 256, 0, s>>>(kind, in->data, P.L, P.nout, P.nseg, P.seglen, out->data, pv, pi);
  st = check_launch("oxc_reduce");
  if (st) return st;
  const unsigned g2 = (unsigned)std::max<int64_t>(1, std::min<int64_t>((P.nout + 255) / 256, cap));
  reduce_col_finish_kernel<<<g2, 256, 0, s>>>(kind, in->data, P.L, P.nout, P.nseg, pv, pi, out->data);
  return check_launch("oxc_reduce (finish)");
}

// The forward reduction a VJP needs first (argmax/argmin for max/min, norm
// for norm), or -1.
static int vjp_aux_kind(int32_t kind) {
  return kind == RK_MAX ? RK_ARGMAX : kind == RK_MIN ? RK_ARGMIN : kind == RK_NORM ? RK_NORM : -1;
}

static void keepdim_view(const oxc_view* x, int64_t d, float* data, oxc_view* out) {
  out->data = data;
  out->ndim = x->ndim;
  int64_t expect = 1;
  for (int i = x->ndim - 1; i >= 0; --i) {
    out->shape[i] = i == d ? 1 : x->shape[i];
    out->strides[i] = expect;
    expect *= out->shape[i];
  }
}

size_t oxc_reduce_bwd_workspace_size(int32_t kind, const oxc_view* x, int64_t dim) {
  const int ak = vjp_aux_kind(kind);
  if (ak < 0 || !x || x->ndim <= 0 || x->ndim > OXC_MAX_DIMS) return 0;
  const int64_t d = dim < 0 ? x->ndim + dim : dim;
  if (d < 0 || d >= x->ndim) return 0;
  int64_t nout = 1;
  for (int i = 0; i < x->ndim; ++i) nout *= i == d ? 1 : x->shape[i];
  return (size_t)nout * sizeof(float) + 256 + oxc_reduce_workspace_size(ak, x, d);
}

oxc_status oxc_reduce_bwd(int32_t kind, const oxc_view* x, int64_t dim, const float* g, float* dx,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (kind < 0 || kind > 6)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown reduction kind %d", kind);
  if (kind == RK_ARGMAX || kind == RK_ARGMIN)
    return fail(OXC_ERR_NOT_IMPLEMENTED,
                "not implemented: argmax/argmin are integer outputs and have no gradient");
  oxc_status st = check_view(x, "reduce backward");
  if (st) return st;
  const int nd = x->ndim;
  const int64_t d = dim < 0 ? nd + dim : dim;
  if (d < 0 || d >= nd)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: dim %lld out of range for %d-D tensor",
                (long long)dim, nd);
  int64_t outer = 1, inner = 1;
  for (int i = 0; i < d; ++i) outer *= x->shape[i];
  for (int i = (int)d + 1; i < nd; ++i) inner *= x->shape[i];
  const int64_t len = x->shape[d], total = outer * len * inner;
  if ((kind == RK_MAX || kind == RK_MIN) && len == 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: cannot compute max/min over a zero-length dim");
  if (total == 0) return OXC_OK;
  if (!g || !dx || !x->data)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: reduce backward: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int ak = vjp_aux_kind(kind);
  float* aux = nullptr;
  if (ak >= 0) {
    const size_t need = oxc_reduce_bwd_workspace_size(kind, x, d);
    if (!workspace || workspace_bytes < need)
      return fail(OXC_ERR_INVALID_ARGUMENT,
                  "invalid argument: reduce backward needs a %zu-byte workspace "
                  "(oxc_reduce_bwd_workspace_size), got %zu", need, workspace_bytes);
    aux = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 15) & ~uintptr_t(15));
    const size_t aux_bytes = ((size_t)outer * inner * sizeof(float) + 15) & ~size_t(15);
    unsigned char* rws = reinterpret_cast<unsigned char*>(aux) + aux_bytes;
    const size_t used = (size_t)(rws - static_cast<unsigned char*>(workspace));
    oxc_view av;
    keepdim_view(x, d, aux, &av);
    st = oxc_reduce(ak, x, d, 1, &av, rws, workspace_bytes - used, stream);
    if (st) return st;
  }
  XView X;
  X.nd = nd;
  bool xdense = true;
  int64_t expect = 1;
  for (int i = nd - 1; i >= 0; --i) {
    X.n[i] = x->shape[i] > 0 ? x->shape[i] : 1;
    X.st[i] = x->strides[i];
    if (x->shape[i] != 1 && x->strides[i] != expect) xdense = false;
    expect *= x->shape[i];
  }
  const float rn = 1.0f / (float)len;
  const int64_t cap = (int64_t)sm_count() * 16;
#define OXC_VJP_LAUNCH(K)                                                                        \
  do {                                                                                           \
    if (inner > 1) {                                                                             \
      reduce_vjp_rows_kernel<K><<<(unsigned)std::min<int64_t>(outer * len, cap), 256, 0, s>>>(   \
          x->data, X, xdense, g, aux, dx, outer * len, len, inner, rn);                          \
    } else {                                                                                     \
      reduce_vjp_last_kernel<K><<<(unsigned)std::max<int64_t>(1, std::min<int64_t>(              \
                                      (total + 255) / 256, cap)), 256, 0, s>>>(                   \
          x->data, X, xdense, g, aux, dx, total, len, rn);                                       \
    }                                                                                            \
  } while (0)
  switch (kind) {
    case RK_SUM: OXC_VJP_LAUNCH(RK_SUM); break;
    case RK_MEAN: OXC_VJP_LAUNCH(RK_MEAN); break;
    case RK_NORM: OXC_VJP_LAUNCH(RK_NORM); break;
    default: OXC_VJP_LAUNCH(RK_MAX); break;  // max and min: scatter to the arg position
  }
#undef OXC_VJP_LAUNCH
  return check_launch("oxc_reduce_bwd");
}

static int64_t all_parts(int64_t n, int64_t* chunk) {
  const int64_t cap = (int64_t)sm_count() * 4;
  int64_t parts = std::max<int64_t>(1, std::min<int64_t>(cap, (n + 8191) / 8192));
  *chunk = (n + parts - 1) / parts;
  parts = std::max<int64_t>(1, (n + *chunk - 1) / *chunk);
  return parts;
}

size_t oxc_reduce_all_workspace_size(int64_t numel) {
  int64_t chunk;
  const int64_t parts = all_parts(std::max<int64_t>(numel, 1), &chunk);
  return (size_t)parts * (sizeof(double) + sizeof(float) + sizeof(long long)) + 256;
}

oxc_status oxc_reduce_all(int32_t kind, const oxc_view* in, float* out, double* out_f64,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (kind < 0 || kind > 6)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown reduction kind %d", kind);
  oxc_status st = check_view(in, "reduce_all");
  if (st) return st;
  int64_t n;
  Flat f = make_flat(in, &n);
  if (n == 0 && kind != RK_SUM && kind != RK_MEAN && kind != RK_NORM)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: cannot compute min/max/argmax/argmin over an empty reduction");
  if (!out) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: reduce_all: null output");
  int64_t chunk;
  const int64_t parts = all_parts(std::max<int64_t>(n, 1), &chunk);
  const size_t need = oxc_reduce_all_workspace_size(n);
  if (!workspace || workspace_bytes < need)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: reduce_all needs a %zu-byte workspace, got %zu",
                need, workspace_bytes);
  double* ps = reinterpret_cast<double*>((reinterpret_cast<uintptr_t>(workspace) + 15) & ~uintptr_t(15));
  long long* pi = reinterpret_cast<long long*>(ps + parts);
  float* pv = reinterpret_cast<float*>(pi + parts);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  reduce_all_stage1<<<(unsigned)parts, 256, 0, s>>>(kind, in->data, f, n, chunk, ps, pv, pi);
  st = check_launch("oxc_reduce_all");
  if (st) return st;
  reduce_all_stage2<<<1, 32, 0, s>>>(kind, in->data, f, n, n ? parts : 0, ps, pv, pi, out, out_f64);
  return check_launch("oxc_reduce_all (finish)");
}

size_t oxc_sum_squares_workspace_size(const oxc_view* views, int32_t count) {
  if (!views || count <= 0 || count > 16) return 0;
  int64_t parts = 0;
  for (int i = 0; i < count; ++i) {
    int64_t n = 1;
    for (int d = 0; d < views[i].ndim; ++d) n *= views[i].shape[d];
    parts += (n + (1 << 18) - 1) >> 18;
  }
  return (size_t)std::max<int64_t>(parts, 1) * sizeof(double) + 256;
}

oxc_status oxc_sum_squares(const oxc_view* views, int32_t count, double* out, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (!views || count <= 0 || count > 16)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: sum_squares takes 1..16 tensors, got %d", count);
  if (!out) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: sum_squares: null output");
  MultiViews mv;
  mv.count = count;
  mv.chunk = 1 << 18;
  mv.first_part[0] = 0;
  for (int i = 0; i < count; ++i) {
    oxc_status st = check_view(&views[i], "sum_squares");
    if (st) return st;
    mv.p[i] = views[i].data;
    mv.f[i] = make_flat(&views[i], &mv.n[i]);
    mv.first_part[i + 1] = mv.first_part[i] + (mv.n[i] + mv.chunk - 1) / mv.chunk;
  }
  const size_t need = oxc_sum_squares_workspace_size(views, count);
  if (!workspace || workspace_bytes < need)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: sum_squares needs a %zu-byte workspace, got %zu",
                need, workspace_bytes);
  double* ps = reinterpret_cast<double*>((reinterpret_cast<uintptr_t>(workspace) + 15) & ~uintptr_t(15));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t parts = mv.first_part[count];
  if (parts > 0) {
    sumsq_multi_stage1<<<(unsigned)parts, 256, 0, s>>>(mv, ps);
    oxc_status st = check_launch("oxc_sum_squares");
    if (st) return st;
  }
  sumsq_multi_stage2<<<1, 256, 0, s>>>(parts, ps, out);
  return check_launch("oxc_sum_squares (finish)");
}

}  // extern "C"
