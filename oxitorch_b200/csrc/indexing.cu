// indexing.cu -- row selection for the dim-0 scatter and its VJP (sm_100a).
//
// The reference runs Tensor::scatter_dim0 (crates/oxi-tensor/src/lib.rs:895-933)
// and the VJP of ops::scatter_dim0 (crates/oxi-autograd/src/ops.rs:531-598) as
// host loops over to_vec() copies.  All three results are row selections:
//
//   forward      out[r]  = written(r) ? values[last writer of r] : base[r]
//   d/dbase      gb[r]   = written(r) ? 0 : g[r]
//   d/dvalues    gv[p]   = p is the last writer of its row ? g[row of p] : 0
//
// so one kernel serves them: out[i] = map[i] >= 0 ? a[map[i]] : (b ? b[i] : 0),
// rows of `inner` floats.  The host resolves the last-write-wins map from the
// index list (which the reference's API takes as a host slice), so the device
// work is one coalesced pass: read each selected row once, write each output
// row once.  HBM-bound; a warp per row with 128-bit accesses where the rows
// and pointers allow, grid-stride over rows.
#include <algorithm>

#include "common.cuh"

namespace oxc {

__device__ __forceinline__ void select_record_bad(int32_t* flag, int64_t value, int64_t size) {
  if (flag && atomicCAS(flag, 0, 1) == 0) {
    flag[1] = (int32_t)(uint32_t)((uint64_t)value & 0xffffffffu);
    flag[2] = (int32_t)(uint32_t)((uint64_t)value >> 32);
    flag[3] = (int32_t)size;
  }
}

// T = float4 (inner4 = inner / 4 vectors per row) or float (inner4 = inner).
template <typename T>
__global__ void __launch_bounds__(256) select_rows_kernel(const T* __restrict__ a, int64_t a_rows,
                                                          const int64_t* __restrict__ map, int64_t n,
                                                          const T* __restrict__ b, T* __restrict__ out,
                                                          int64_t vecs, int32_t* err) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t i = warp; i < n; i += nwarps) {
    const int64_t r = map[i];
    T* d = out + i * vecs;
    if (r >= a_rows) {
      if (lane == 0) select_record_bad(err, r, a_rows);
      continue;
    }
    if (r >= 0) {
      const T* s = a + r * vecs;
      for (int64_t k = lane; k < vecs; k += 32) d[k] = __ldg(s + k);
    } else if (b) {
      const T* s = b + i * vecs;
      for (int64_t k = lane; k < vecs; k += 32) d[k] = __ldg(s + k);
    } else {
      const T z{};
      for (int64_t k = lane; k < vecs; k += 32) d[k] = z;
    }
  }
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_select_rows(const float* a, int64_t a_rows, const int64_t* map, int64_t n,
                           const float* b, float* out, int64_t inner, int32_t* err_flag,
                           void* stream) {
  if (a_rows < 0 || n < 0 || inner < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: select_rows: negative size");
  if (n == 0 || inner == 0) return OXC_OK;
  if (!map || !out || (a_rows > 0 && !a))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: select_rows: null pointer");
  const bool v4 = inner % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(out);
  const int64_t vecs = v4 ? inner / 4 : inner;
  const int64_t cap = (int64_t)sm_count() * 8 * 4;  // 8 CTAs of 256 per SM, 4 waves
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, cap));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v4)
    select_rows_kernel<float4><<<grid, 256, 0, s>>>(reinterpret_cast<const float4*>(a), a_rows, map, n,
                                                    reinterpret_cast<const float4*>(b),
                                                    reinterpret_cast<float4*>(out), vecs, err_flag);
  else
    select_rows_kernel<float><<<grid, 256, 0, s>>>(a, a_rows, map, n, b, out, vecs, err_flag);
  return check_launch("oxc_select_rows");
}

}  // extern "C"

// ---- masked_select (Tensor::masked_select) and its VJP ------------------------------
//
// crates/oxi-tensor/src/lib.rs:939-960 picks, in row-major order of the
// broadcast grid, the x values whose mask entry is nonzero (a picked NaN of x
// is dropped too: the reference marks unpicked slots with NaN and filters
// NaN).  The VJP (crates/oxi-autograd/src/ops.rs:610-665) walks the same grid
// and counts picks by the mask alone.  Both are stream compactions over the
// grid: (1) a count per chunk of kMsChunk points, (2) one CTA turning the
// counts into exclusive offsets (and the total), (3) a write pass where each
// warp ballot gives every pick its position.  x and mask arrive as views of
// the grid's shape (broadcast dims have stride 0).

namespace oxc {

constexpr int kMsThreads = 256;
constexpr int kMsTiles = 16;
constexpr int64_t kMsChunk = (int64_t)kMsThreads * kMsTiles;

struct MsGrid {
  const float* x;
  const float* m;
  int32_t nd;
  int64_t shape[OXC_MAX_DIMS];
  int64_t xs[OXC_MAX_DIMS];
  int64_t ms[OXC_MAX_DIMS];
};

__device__ __forceinline__ bool ms_pred(const MsGrid& G, int64_t k, int64_t n, int by_mask, float* xv) {
  if (k >= n) return false;
  int64_t xo = 0, mo = 0, r = k;
  for (int d = G.nd - 1; d >= 0; --d) {
    const int64_t i = r % G.shape[d];
    r /= G.shape[d];
    xo += i * G.xs[d];
    mo += i * G.ms[d];
  }
  if (G.m[mo] == 0.0f) return false;
  if (by_mask) return true;
  const float v = G.x[xo];
  *xv = v;
  return !isnan(v);
}

__global__ void __launch_bounds__(kMsThreads) ms_count_kernel(MsGrid G, int64_t n, int by_mask,
                                                              int64_t* counts) {
  const int64_t base = (int64_t)blockIdx.x * kMsChunk;
  int64_t c = 0;
  for (int t = 0; t < kMsTiles; ++t) {
    float v;
    c += __syncthreads_count(ms_pred(G, base + (int64_t)t * kMsThreads + threadIdx.x, n, by_mask, &v));
  }
  if (threadIdx.x == 0) counts[blockIdx.x] = c;
}

// One CTA of 1024 threads: counts[0..nchunks) -> exclusive offsets in place,
// the total in counts[nchunks].
__global__ void __launch_bounds__(1024) ms_scan_kernel(int64_t* counts, int64_t nchunks) {
  __shared__ int64_t part[1024];
  const int64_t seg = (nchunks + 1023) / 1024;
  const int64_t lo = (int64_t)threadIdx.x * seg;
  const int64_t hi = lo + seg < nchunks ? lo + seg : nchunks;
  int64_t s = 0;
  for (int64_t i = lo; i < hi; ++i) s += counts[i];
  part[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t run = 0;
    for (int i = 0; i < 1024; ++i) {
      const int64_t v = part[i];
      part[i] = run;
      run += v;
    }
    counts[nchunks] = run;
  }
  __syncthreads();
  int64_t run = part[threadIdx.x];
  for (int64_t i = lo; i < hi; ++i) {
    const int64_t v = counts[i];
    counts[i] = run;
    run += v;
  }
}

// MODE 0: out[pos] = x for every pick (forward).  MODE 1: dense grad grid,
// out[k] = g[pos] at picked points (pos < ng), 0 elsewhere (VJP).
template <int MODE>
__global__ void __launch_bounds__(kMsThreads) ms_write_kernel(MsGrid G, int64_t n,
                                                              const int64_t* __restrict__ offsets,
                                                              const float* __restrict__ g, int64_t ng,
                                                              float* __restrict__ out) {
  __shared__ int warp_cnt[kMsThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t base = (int64_t)blockIdx.x * kMsChunk;
  int64_t run = offsets[blockIdx.x];
  for (int t = 0; t < kMsTiles; ++t) {
    const int64_t k = base + (int64_t)t * kMsThreads + threadIdx.x;
    float v = 0.0f;
    const bool p = ms_pred(G, k, n, MODE, &v);
    const unsigned ballot = __ballot_sync(0xffffffffu, p);
    if (lane == 0) warp_cnt[warp] = __popc(ballot);
    __syncthreads();
    int64_t off = 0, tile = 0;
    for (int w = 0; w < kMsThreads / 32; ++w) {
      if (w < warp) off += warp_cnt[w];
      tile += warp_cnt[w];
    }
    const int64_t pos = run + off + __popc(ballot & ((1u << lane) - 1u));
    if (MODE == 0) {
      if (p) out[pos] = v;
    } else if (k < n) {
      out[k] = (p && pos < ng) ? g[pos] : 0.0f;
    }
    run += tile;
    __syncthreads();
  }
}

// Sum of the dense grad grid over the dims where x broadcasts: a thread per x
// element folds its grid points in grid order from +0.0, the order of the
// reference's walk.  Adding the zeros of unpicked points changes no bit (a sum
// that starts at +0.0 is never -0.0).
struct MsFold {
  int32_t nd;
  int64_t xshape[OXC_MAX_DIMS];  // x's shape aligned to the grid (1 where missing)
  int64_t gstride[OXC_MAX_DIMS]; // row-major strides of the grid
  int64_t bshape[OXC_MAX_DIMS];  // grid size on broadcast dims, 1 elsewhere
};

__global__ void __launch_bounds__(256) ms_fold_kernel(MsFold F, const float* __restrict__ gfull,
                                                      int64_t nx, int64_t nb, float* __restrict__ gx) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nx;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = e, base = 0;
    for (int d = F.nd - 1; d >= 0; --d) {
      base += (r % F.xshape[d]) * F.gstride[d];
      r /= F.xshape[d];
    }
    float acc = 0.0f;
    for (int64_t q = 0; q < nb; ++q) {
      int64_t rq = q, off = 0;
      for (int d = F.nd - 1; d >= 0; --d) {
        off += (rq % F.bshape[d]) * F.gstride[d];
        rq /= F.bshape[d];
      }
      acc = __fadd_rn(acc, gfull[base + off]);
    }
    gx[e] = acc;
  }
}

static oxc_status ms_grid(const oxc_view* x, const oxc_view* m, MsGrid* G, int64_t* n) {
  if (!m || (x && x->ndim != m->ndim) || m->ndim < 0 || m->ndim > OXC_MAX_DIMS)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: masked_select: views of the grid's rank");
  G->x = x ? x->data : nullptr;
  G->m = m->data;
  G->nd = m->ndim;
  int64_t total = 1;
  for (int d = 0; d < m->ndim; ++d) {
    if (m->shape[d] < 0 || (x && x->shape[d] != m->shape[d]))
      return fail(OXC_ERR_SHAPE_MISMATCH, "shape mismatch: masked_select views differ in dim %d", d);
    G->shape[d] = m->shape[d];
    G->xs[d] = x ? x->strides[d] : 0;
    G->ms[d] = m->strides[d];
    total *= m->shape[d];
  }
  *n = total;
  return OXC_OK;
}

}  // namespace oxc

extern "C" {

size_t oxc_masked_select_workspace_size(int64_t n) {
  if (n <= 0) return sizeof(int64_t);
  return (size_t)((n + kMsChunk - 1) / kMsChunk + 1) * sizeof(int64_t);
}

oxc_status oxc_masked_select_count(const oxc_view* x, const oxc_view* mask, int32_t by_mask,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  MsGrid G;
  int64_t n = 0;
  oxc_status st = ms_grid(by_mask ? nullptr : x, mask, &G, &n);
  if (st) return st;
  if (!by_mask && !x) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: masked_select: null x");
  const size_t need = oxc_masked_select_workspace_size(n);
  if (!workspace || workspace_bytes < need)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: masked_select needs a %zu-byte workspace, got %zu", need, workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t* counts = static_cast<int64_t*>(workspace);
  if (n == 0) {
    cudaError_t e = cudaMemsetAsync(counts, 0, sizeof(int64_t), s);
    return e == cudaSuccess ? OXC_OK : cuda_fail(e, "oxc_masked_select_count");
  }
  if (!G.m || (!by_mask && !G.x))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: masked_select: null pointer");
  const int64_t nchunks = (n + kMsChunk - 1) / kMsChunk;
  if (nchunks > 0x7fffffff)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: masked_select over %lld points", (long long)n);
  ms_count_kernel<<<(unsigned)nchunks, kMsThreads, 0, s>>>(G, n, by_mask ? 1 : 0, counts);
  oxc_status l = check_launch("oxc_masked_select_count");
  if (l) return l;
  ms_scan_kernel<<<1, 1024, 0, s>>>(counts, nchunks);
  return check_launch("oxc_masked_select_count (scan)");
}

oxc_status oxc_masked_select_fwd(const oxc_view* x, const oxc_view* mask, const void* workspace,
                                 float* out, void* stream) {
  MsGrid G;
  int64_t n = 0;
  oxc_status st = ms_grid(x, mask, &G, &n);
  if (st) return st;
  if (n == 0) return OXC_OK;
  if (!x || !G.x || !G.m || !workspace || !out)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: masked_select: null pointer");
  const int64_t nchunks = (n + kMsChunk - 1) / kMsChunk;
  ms_write_kernel<0><<<(unsigned)nchunks, kMsThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      G, n, static_cast<const int64_t*>(workspace), nullptr, 0, out);
  return check_launch("oxc_masked_select_fwd");
}

oxc_status oxc_masked_select_bwd(const float* g, int64_t ng, const oxc_view* mask,
                                 const void* workspace, float* gfull, void* stream) {
  MsGrid G;
  int64_t n = 0;
  oxc_status st = ms_grid(nullptr, mask, &G, &n);
  if (st) return st;
  if (n == 0) return OXC_OK;
  if (!G.m || !workspace || !gfull || ng < 0 || (ng > 0 && !g))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: masked_select backward: null pointer");
  const int64_t nchunks = (n + kMsChunk - 1) / kMsChunk;
  ms_write_kernel<1><<<(unsigned)nchunks, kMsThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      G, n, static_cast<const int64_t*>(workspace), g, ng, gfull);
  return check_launch("oxc_masked_select_bwd");
}

oxc_status oxc_broadcast_fold(const float* gfull, const int64_t* grid_shape, const int64_t* x_shape,
                              int32_t ndim, float* gx, void* stream) {
  if (ndim < 0 || ndim > OXC_MAX_DIMS || (ndim > 0 && (!grid_shape || !x_shape)))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: broadcast_fold: rank %d", ndim);
  MsFold F;
  F.nd = ndim;
  int64_t nx = 1, nb = 1, stride = 1;
  for (int d = ndim - 1; d >= 0; --d) {
    if (grid_shape[d] < 0 || (x_shape[d] != grid_shape[d] && x_shape[d] != 1))
      return fail(OXC_ERR_SHAPE_MISMATCH, "shape mismatch: broadcast_fold dim %d", d);
    F.xshape[d] = x_shape[d];
    F.gstride[d] = stride;
    F.bshape[d] = x_shape[d] == 1 ? grid_shape[d] : 1;
    stride *= grid_shape[d];
    nx *= x_shape[d];
    nb *= F.bshape[d];
  }
  if (nx == 0) return OXC_OK;
  if (!gx || (nb > 0 && stride > 0 && !gfull))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: broadcast_fold: null pointer");
  if (stride == 0) nb = 0;  // an empty grid: every x element gets +0.0
  const int64_t cap = (int64_t)sm_count() * 8;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((nx + 255) / 256, cap));
  ms_fold_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(F, gfull, nx, nb, gx);
  return check_launch("oxc_broadcast_fold");
}

}  // extern "C"
