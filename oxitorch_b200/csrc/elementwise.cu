// elementwise.cu -- the registry of elementwise ops over strided/broadcast views.
//
// Reference: crates/oxi-tensor/src/ops.rs:55-202 (F32_BINARY_OPS, F32_CMP_OPS,
// F32_UNARY_OPS), dispatched by Tensor::binary_op / cmp_op / unary_op
// (crates/oxi-tensor/src/lib.rs:263-357) over iterate::map_n (iterate.rs:21-75)
// with NumPy broadcasting (layout.rs:67-114).  Every op is the same IEEE f32
// operation: + - * / sqrt are correctly rounded on both sides (bit-identical),
// min/max ignore NaN like f32::min/max, sign follows f32::signum (never 0),
// round is half away from zero; exp/log/log2/log10/sin/cos/tanh/pow call
// CUDA's libm (a few ulp from glibc's).
//
// The host side broadcasts (ShapeMismatch on incompatible shapes), turns every
// operand into strides over the output grid (0 on broadcast dims), drops
// size-1 dims and merges dims that are contiguous for every operand.  Then:
//   contiguous: every operand dense (or a scalar): 128-bit grid-stride loop;
//   pipelined:  a 2-D problem with one column-major input (a transposed view)
//               whose columns are 16-byte aligned, and the other input dense
//               row-major or a scalar: the tile pipeline of tilepipe.cuh (TMA
//               boxes for the transposed input, bulk row copies, long
//               row-major segments);
//   tiled:      other 2-D problems with a column-major operand: 32x32 tiles
//               through shared memory, so both the column-major read and the
//               row-major write are coalesced;
//   general:    any strides, index arithmetic per element (up to 8 dims).
// Outputs are always dense row-major, like the reference's from_results.
#include <math.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "tilepipe.cuh"

namespace oxc {

enum ElemKind { EK_UNARY = 0, EK_BINARY = 1, EK_CMP = 2 };

// Unary op id past the reference registry's 19: the identity, which turns the
// elementwise engine into a strided copy (Tensor::contiguous).
constexpr int kUnaryCopy = 19;

__device__ __forceinline__ float rust_signum(float a) {
  return isnan(a) ? a : (signbit(a) ? -1.0f : 1.0f);
}

__device__ __forceinline__ float unary_op(int op, float a) {
  switch (op) {
    case 0: return -a;
    case 1: return fabsf(a);
    case 2: return __fsqrt_rn(a);
    case 3: return __fdiv_rn(1.0f, __fsqrt_rn(a));
    case 4: return expf(a);
    case 5: return logf(a);
    case 6: return log2f(a);
    case 7: return log10f(a);
    case 8: return sinf(a);
    case 9: return cosf(a);
    case 10: return tanhf(a);
    case 11: return fmaxf(a, 0.0f);
    case 12: return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a)));
    case 13: return floorf(a);
    case 14: return ceilf(a);
    case 15: return roundf(a);
    case 16: return rust_signum(a);
    case 17: return __fmul_rn(a, a);
    case 18: return __fdiv_rn(1.0f, a);
    default: return a;  // kUnaryCopy: the bits of a, for oxc_contiguous
  }
}

__device__ __forceinline__ float binary_op(int op, float a, float b) {
  switch (op) {
    case 0: return __fadd_rn(a, b);
    case 1: return __fsub_rn(a, b);
    case 2: return __fmul_rn(a, b);
    case 3: return __fdiv_rn(a, b);
    case 4: return powf(a, b);
    case 5: return fminf(a, b);
    default: return fmaxf(a, b);
  }
}

__device__ __forceinline__ float cmp_op(int op, float a, float b) {
  bool r;
  switch (op) {
    case 0: r = a == b; break;
    case 1: r = a != b; break;
    case 2: r = a < b; break;
    case 3: r = a <= b; break;
    case 4: r = a > b; break;
    default: r = a >= b; break;
  }
  return r ? 1.0f : 0.0f;
}

__device__ __forceinline__ float apply(int kind, int op, float a, float b) {
  return kind == EK_UNARY ? unary_op(op, a) : kind == EK_BINARY ? binary_op(op, a, b)
                                                                : cmp_op(op, a, b);
}

// r[k] = apply(KIND, OP, a[k], b[k]) with the op a compile-time constant, so
// the switch folds away and the N elements run as straight-line code.
template <int KIND, int OP, int N>
__device__ __forceinline__ void apply_n(const float (&a)[N], const float (&b)[N], float (&r)[N]) {
#pragma unroll
  for (int k = 0; k < N; ++k) r[k] = apply(KIND, OP, a[k], b[k]);
}

// apply() over N elements with one run-time dispatch for all of them (kind and
// op are uniform across the launch): the per-element switch of apply() costs
// branch resolution on every element of the tile kernels.
template <int N>
__device__ __forceinline__ void apply_tile(int kind, int op, const float (&a)[N],
                                           const float (&b)[N], float (&r)[N]) {
#define OXC_U(o) case o: apply_n<EK_UNARY, o, N>(a, b, r); return;
#define OXC_B(o) case o: apply_n<EK_BINARY, o, N>(a, b, r); return;
#define OXC_C(o) case o: apply_n<EK_CMP, o, N>(a, b, r); return;
  if (kind == EK_UNARY) {
    switch (op) {
      OXC_U(0) OXC_U(1) OXC_U(2) OXC_U(3) OXC_U(4) OXC_U(5) OXC_U(6) OXC_U(7) OXC_U(8) OXC_U(9)
      OXC_U(10) OXC_U(11) OXC_U(12) OXC_U(13) OXC_U(14) OXC_U(15) OXC_U(16) OXC_U(17)
      OXC_U(18)
      default: apply_n<EK_UNARY, 19, N>(a, b, r); return;
    }
  } else if (kind == EK_BINARY) {
    switch (op) {
      OXC_B(0) OXC_B(1) OXC_B(2) OXC_B(3) OXC_B(4) OXC_B(5)
      default: apply_n<EK_BINARY, 6, N>(a, b, r); return;
    }
  } else {
    switch (op) {
      OXC_C(0) OXC_C(1) OXC_C(2) OXC_C(3) OXC_C(4)
      default: apply_n<EK_CMP, 5, N>(a, b, r); return;
    }
  }
#undef OXC_U
#undef OXC_B
#undef OXC_C
}

struct Grid {
  int nd;
  int64_t n[OXC_MAX_DIMS];
  int64_t st[2][OXC_MAX_DIMS];  // per input, in elements (0 = broadcast)
};

// One input: a tensor (p, strides in Grid), or a single value broadcast
// everywhere -- read from device memory at p (a zero-stride view) or the
// host-provided v when p is null.
struct Operand {
  const float* p;
  float v;
  int scalar;
};

__device__ __forceinline__ float scalar_value(const Operand& o) { return o.p ? __ldg(o.p) : o.v; }

// Contiguous path: every tensor operand dense.  VW = 4 needs them 16-byte
// aligned.
template <int VW>
__global__ void __launch_bounds__(256) elem_dense_kernel(int kind, int op, Operand a, Operand b,
                                                         float* __restrict__ out, int64_t n) {
  const float sa = a.scalar ? scalar_value(a) : 0.0f;
  const float sb = (kind != EK_UNARY && b.scalar) ? scalar_value(b) : 0.0f;
  const int64_t nv = n / VW;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    if constexpr (VW == 4) {
      const float4 x = a.scalar ? make_float4(sa, sa, sa, sa)
                                : ld_stream(reinterpret_cast<const float4*>(a.p) + v);
      float4 y = make_float4(sb, sb, sb, sb);
      if (kind != EK_UNARY && !b.scalar) y = ld_stream(reinterpret_cast<const float4*>(b.p) + v);
      float4 o;
      o.x = apply(kind, op, x.x, y.x);
      o.y = apply(kind, op, x.y, y.y);
      o.z = apply(kind, op, x.z, y.z);
      o.w = apply(kind, op, x.w, y.w);
      st_stream(reinterpret_cast<float4*>(out) + v, o);
    } else {
      const float x = a.scalar ? sa : ld_stream(a.p + v);
      const float y = (kind == EK_UNARY || b.scalar) ? sb : ld_stream(b.p + v);
      st_stream(out + v, apply(kind, op, x, y));
    }
  }
  if constexpr (VW == 4) {  // tail
    for (int64_t i = nv * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      const float x = a.scalar ? sa : a.p[i];
      const float y = (kind == EK_UNARY || b.scalar) ? sb : b.p[i];
      out[i] = apply(kind, op, x, y);
    }
  }
}

// General strided path (index arithmetic per element, innermost dim fastest).
__global__ void __launch_bounds__(256) elem_strided_kernel(int kind, int op, Operand a, Operand b,
                                                           Grid g, float* __restrict__ out,
                                                           int64_t n) {
  const float sa = a.scalar ? scalar_value(a) : 0.0f;
  const float sb = (kind != EK_UNARY && b.scalar) ? scalar_value(b) : 0.0f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t rem = i, oa = 0, ob = 0;
    for (int d = g.nd - 1; d >= 0; --d) {
      const int64_t q = rem / g.n[d];
      const int64_t idx = rem - q * g.n[d];
      rem = q;
      oa += idx * g.st[0][d];
      ob += idx * g.st[1][d];
    }
    const float x = a.scalar ? sa : __ldg(a.p + oa);
    const float y = (kind == EK_UNARY || b.scalar) ? sb : __ldg(b.p + ob);
    out[i] = apply(kind, op, x, y);
  }
}

// 2-D tiled path: out[r][c] (row-major, cols = g.n[1]); tensor inputs are
// staged through 32x32 shared tiles; `colmajor` bit k says input k is
// contiguous along r (a transposed view) and is read along r.
__global__ void __launch_bounds__(256) elem_tiled_kernel(int kind, int op, Operand a, Operand b,
                                                         Grid g, int colmajor,
                                                         float* __restrict__ out) {
  __shared__ float tiles[2][32][33];
  const float sa = a.scalar ? scalar_value(a) : 0.0f;
  const float sb = (kind != EK_UNARY && b.scalar) ? scalar_value(b) : 0.0f;
  const int64_t R = g.n[0], C = g.n[1];
  const int64_t tiles_c = (C + 31) / 32;
  const int64_t ntiles = ((R + 31) / 32) * tiles_c;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const Operand ops[2] = {a, b};
  const int nin = kind == EK_UNARY ? 1 : 2;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t r0 = (t / tiles_c) * 32, c0 = (t % tiles_c) * 32;
    for (int k = 0; k < nin; ++k) {
      if (ops[k].scalar) continue;
      if (colmajor & (1 << k)) {
        // tiles[k][c][r]: consecutive lanes walk r, the contiguous dim
        for (int j = ty; j < 32; j += 8) {
          const int64_t r = r0 + tx, c = c0 + j;
          tiles[k][j][tx] =
              (r < R && c < C) ? __ldg(ops[k].p + r * g.st[k][0] + c * g.st[k][1]) : 0.0f;
        }
      } else {
        for (int j = ty; j < 32; j += 8) {
          const int64_t r = r0 + j, c = c0 + tx;
          tiles[k][tx][j] =
              (r < R && c < C) ? __ldg(ops[k].p + r * g.st[k][0] + c * g.st[k][1]) : 0.0f;
        }
      }
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
      const int64_t r = r0 + j, c = c0 + tx;
      if (r < R && c < C) {
        const float x = a.scalar ? sa : tiles[0][tx][j];
        const float y = (kind == EK_UNARY || b.scalar) ? sb : tiles[1][tx][j];
        out[r * C + c] = apply(kind, op, x, y);
      }
    }
    __syncthreads();
  }
}

// Transposed-operand path on the tile pipeline (tilepipe.cuh), for 2-D
// problems whose one column-major input has 16-byte aligned columns: that
// input arrives as swizzled 2-D TMA boxes of 32 rows x 192 columns, a dense
// row-major second input (ROW) as 768-byte bulk row copies, and 24 consumer
// warps apply the op and stream the row-major output in full 32-byte sectors.
// GB: the column-major input is operand b (the op keeps its argument order);
// the other operand is the row-major tile or a scalar.
template <bool GB, bool ROW>
__global__ void __launch_bounds__(kTThreads, 1) elem_pipe_kernel(
    const __grid_constant__ CUtensorMap gmap, View2 g, const float* __restrict__ rowp,
    Operand other, int kind, int op, float* __restrict__ out, int64_t R, int64_t C) {
  constexpr int NSLOT = ROW ? 2 : 1;
  extern __shared__ unsigned char smem_raw[];
  const TileRing<NSLOT, true> ring = make_tile_ring<NSLOT, true>(smem_raw, kStageFwd);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == kTCW) {
    const float* const src[2] = {rowp, nullptr};
    tile_producer<true, NSLOT>(ring, &gmap, g, src, ROW ? 1 : 0, R, C);
    return;
  }
  const float so = (!ROW && kind != EK_UNARY) ? scalar_value(other) : 0.0f;
  const int t = 4 * (warp & 7) + (lane & 3);
  const int fl = (warp >> 3) * (kTF / kTParts) + (lane >> 2);
  const int goff = gate_off<true>(t, fl), roff = t * kTP + fl;
  const int64_t nstrips = (R + kTT - 1) / kTT;
  int64_t i = 0;
  for (int64_t strip = blockIdx.x; strip < nstrips; strip += gridDim.x) {
    const int64_t r = strip * kTT + t;
    float* orow = out + r * C + fl;
    for (int64_t c0 = 0; c0 < C; c0 += kTF, ++i) {
      if (!tile_acquire(ring, i)) continue;
      const int stage = (int)(i % ring.stages);
      const float* gs = ring.slot(stage, 0) + goff;
      const float* rs = ring.slot(stage, NSLOT - 1) + roff;
      float gv[kTK], ov[kTK];
#pragma unroll
      for (int k = 0; k < kTK; ++k) {
        gv[k] = gs[k * kGateStep<true>];
        ov[k] = ROW ? rs[8 * k] : so;
      }
      tile_release(ring, i);
      if (r >= R) continue;
      const bool full = c0 + kTF <= C;
      if constexpr (ROW) {
        // two streamed inputs: the per-element dispatch measured faster here
#pragma unroll
        for (int k = 0; k < kTK; ++k) {
          if (full || c0 + fl + 8 * k < C) {
            const float res = kind == EK_UNARY ? apply(kind, op, gv[k], 0.0f)
                              : GB             ? apply(kind, op, ov[k], gv[k])
                                               : apply(kind, op, gv[k], ov[k]);
            st_stream(orow + c0 + 8 * k, res);
          }
        }
      } else {
        // unary or scalar operand: one dispatch per tile (2.3 -> 5.3 TB/s for
        // sigmoid on a transposed view)
        float res[kTK];
        if (GB) apply_tile<kTK>(kind, op, ov, gv, res);
        else apply_tile<kTK>(kind, op, gv, ov, res);  // unary ops ignore ov
#pragma unroll
        for (int k = 0; k < kTK; ++k)
          if (full || c0 + fl + 8 * k < C) st_stream(orow + c0 + 8 * k, res[k]);
      }
    }
  }
}

// ---- host-side view algebra (layout.rs) --------------------------------------

static oxc_status view_ok(const oxc_view* v, const char* what) {
  if (!v) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null view", what);
  if (v->ndim < 0 || v->ndim > OXC_MAX_DIMS)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: %s: rank %d > %d", what, v->ndim,
                OXC_MAX_DIMS);
  for (int i = 0; i < v->ndim; ++i)
    if (v->shape[i] < 0)
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative dim", what);
  return OXC_OK;
}

static void shape_str(const oxc_view* v, char* buf, size_t cap) {
  size_t p = 0;
  p += snprintf(buf + p, cap - p, "[");
  for (int i = 0; i < v->ndim && p < cap; ++i)
    p += snprintf(buf + p, cap - p, i ? ", %lld" : "%lld", (long long)v->shape[i]);
  if (p < cap) snprintf(buf + p, cap - p, "]");
}

// layout::broadcast_shapes (layout.rs:67-88).
static oxc_status broadcast(const oxc_view* a, const oxc_view* b, int* nd, int64_t* out) {
  const int r = std::max(a->ndim, b->ndim);
  for (int i = 0; i < r; ++i) {
    const int ia = a->ndim - r + i, ib = b->ndim - r + i;
    const int64_t da = ia >= 0 ? a->shape[ia] : 1, db = ib >= 0 ? b->shape[ib] : 1;
    if (da != db && da != 1 && db != 1) {
      char sa[160], sb[160];
      shape_str(a, sa, sizeof sa);
      shape_str(b, sb, sizeof sb);
      return fail(OXC_ERR_SHAPE_MISMATCH, "shape mismatch: %s vs %s", sa, sb);
    }
    out[i] = std::max(da, db);
  }
  *nd = r;
  return OXC_OK;
}

// layout::broadcast_strides (layout.rs:97-114): 0 on new and size-1 dims.
static void bstrides(const oxc_view* v, int nd, const int64_t* shape, int64_t* st) {
  const int off = nd - v->ndim;
  for (int i = 0; i < nd; ++i) {
    const int j = i - off;
    st[i] = (j >= 0 && v->shape[j] != 1) ? v->strides[j] : 0;
  }
  (void)shape;
}

// Drops size-1 dims and merges dim i into i+1 when contiguous for all inputs
// (the output is dense, so it merges whenever the inputs do).
static void collapse(Grid* g, int nin) {
  Grid h;
  h.nd = 0;
  for (int d = 0; d < g->nd; ++d) {
    if (g->n[d] == 1) continue;
    h.n[h.nd] = g->n[d];
    for (int k = 0; k < 2; ++k) h.st[k][h.nd] = g->st[k][d];
    ++h.nd;
  }
  Grid m;
  m.nd = 0;
  for (int d = 0; d < h.nd; ++d) {
    if (m.nd > 0) {
      bool merge = true;
      for (int k = 0; k < nin; ++k)
        if (m.st[k][m.nd - 1] != h.st[k][d] * h.n[d]) merge = false;
      if (merge) {
        m.n[m.nd - 1] *= h.n[d];
        for (int k = 0; k < 2; ++k) m.st[k][m.nd - 1] = h.st[k][d];
        continue;
      }
    }
    m.n[m.nd] = h.n[d];
    for (int k = 0; k < 2; ++k) m.st[k][m.nd] = h.st[k][d];
    ++m.nd;
  }
  *g = m;
}

static oxc_status run_elementwise(int kind, int op, const oxc_view* a, const oxc_view* b,
                                  const float* scalar, int scalar_first, const oxc_view* out,
                                  cudaStream_t s, const char* fn) {
  oxc_status st = view_ok(a, fn);
  if (st) return st;
  if (b && (st = view_ok(b, fn))) return st;
  if ((st = view_ok(out, fn))) return st;
  int nd = a->ndim;
  int64_t shape[OXC_MAX_DIMS];
  for (int i = 0; i < nd; ++i) shape[i] = a->shape[i];
  if (b && (st = broadcast(a, b, &nd, shape))) return st;
  // the output must be dense row-major with the broadcast shape
  if (out->ndim != nd)
    return fail(OXC_ERR_SHAPE_MISMATCH, "shape mismatch: output rank %d vs %d", out->ndim, nd);
  int64_t total = 1, expect = 1;
  for (int i = nd - 1; i >= 0; --i) {
    if (out->shape[i] != shape[i])
      return fail(OXC_ERR_SHAPE_MISMATCH, "shape mismatch: output dim %d is %lld, expected %lld",
                  i, (long long)out->shape[i], (long long)shape[i]);
    if (shape[i] != 1 && out->strides[i] != expect)
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s output must be contiguous", fn);
    expect *= shape[i];
  }
  total = expect;
  if (total == 0) return OXC_OK;
  if (!a->data || !out->data || (b && !b->data))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null data", fn);
  Grid g;
  g.nd = nd;
  for (int i = 0; i < nd; ++i) g.n[i] = shape[i];
  bstrides(a, nd, shape, g.st[0]);
  if (b) bstrides(b, nd, shape, g.st[1]);
  else for (int i = 0; i < nd; ++i) g.st[1][i] = 0;
  const int nin = b ? 2 : 1;
  collapse(&g, nin);
  Operand oa{a->data, 0.0f, 0}, ob{b ? b->data : nullptr, 0.0f, kind == EK_UNARY ? 1 : 0};
  if (scalar) {  // one operand is the host scalar argument
    if (scalar_first) {
      ob = Operand{a->data, 0.0f, 0};
      for (int d = 0; d < g.nd; ++d) g.st[1][d] = g.st[0][d];
      oa = Operand{nullptr, *scalar, 1};
    } else {
      ob = Operand{nullptr, *scalar, 1};
    }
  }
  // a tensor operand with all-zero strides is one broadcast value
  bool zero[2] = {true, true};
  for (int d = 0; d < g.nd; ++d)
    for (int k = 0; k < 2; ++k)
      if (g.st[k][d]) zero[k] = false;
  if (!oa.scalar && zero[0]) oa.scalar = 1;
  if (!ob.scalar && zero[1]) ob.scalar = 1;
  const bool a_dense = oa.scalar || (g.nd == 1 && g.st[0][0] == 1);
  const bool b_dense = ob.scalar || (g.nd == 1 && g.st[1][0] == 1);
  const int64_t cap = (int64_t)sm_count() * 8;
  if (g.nd <= 1 && a_dense && b_dense) {
    const bool v4 = aligned16(out->data) && (oa.scalar || aligned16(oa.p)) &&
                    (ob.scalar || aligned16(ob.p));
    const int64_t work = v4 ? total / 4 : total;
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, cap * 4));
    if (v4) elem_dense_kernel<4><<<grid, 256, 0, s>>>(kind, op, oa, ob, out->data, total);
    else elem_dense_kernel<1><<<grid, 256, 0, s>>>(kind, op, oa, ob, out->data, total);
    return check_launch(fn);
  }
  int colmajor = 0;
  if (g.nd == 2) {
    const Operand* os[2] = {&oa, &ob};
    for (int k = 0; k < 2; ++k)
      if (!os[k]->scalar && g.st[k][0] == 1 && g.st[k][1] != 1) colmajor |= 1 << k;
  }
  if (colmajor == 1 || colmajor == 2) {
    // one column-major input: the tile pipeline when its layout allows
    const int k = colmajor == 1 ? 0 : 1;
    const Operand& cm = k == 0 ? oa : ob;
    const Operand& ot = k == 0 ? ob : oa;
    const int64_t R = g.n[0], C = g.n[1];
    const bool unary = kind == EK_UNARY;
    const bool other_row = !unary && !ot.scalar && g.st[1 - k][1] == 1 && g.st[1 - k][0] == C &&
                           aligned16(ot.p);
    const bool shape_ok = C % 4 == 0 && C > 1 && R <= INT32_MAX && C <= INT32_MAX &&
                          aligned16(cm.p) && g.st[k][1] % 4 == 0 && g.st[k][1] >= R;
    if (shape_ok && (unary || ot.scalar || other_row)) {
      const View2 gv{cm.p, g.st[k][0], g.st[k][1]};
      CUtensorMap map{};
      if (!gate_tensor_map(&map, gv, R, C))
        return fail(OXC_ERR_OTHER, "%s: cuTensorMapEncodeTiled failed", fn);
      const float* rowp = other_row ? ot.p : nullptr;
      const size_t smem = other_row ? tile_smem_bytes<2, true>(kStageFwd, false)
                                    : tile_smem_bytes<1, true>(kStageFwd, false);
      if (k == 1 && other_row)
        return launch_tile(elem_pipe_kernel<true, true>, smem, R, s, fn, nullptr, map, gv, rowp,
                           ot, (int)kind, op, out->data, R, C);
      if (k == 1)
        return launch_tile(elem_pipe_kernel<true, false>, smem, R, s, fn, nullptr, map, gv, rowp,
                           ot, (int)kind, op, out->data, R, C);
      if (other_row)
        return launch_tile(elem_pipe_kernel<false, true>, smem, R, s, fn, nullptr, map, gv, rowp,
                           ot, (int)kind, op, out->data, R, C);
      return launch_tile(elem_pipe_kernel<false, false>, smem, R, s, fn, nullptr, map, gv, rowp, ot,
                         (int)kind, op, out->data, R, C);
    }
  }
  if (colmajor) {
    const int64_t ntiles = ((g.n[0] + 31) / 32) * ((g.n[1] + 31) / 32);
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ntiles, cap * 2));
    elem_tiled_kernel<<<grid, 256, 0, s>>>(kind, op, oa, ob, g, colmajor, out->data);
    return check_launch(fn);
  }
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, cap * 4));
  elem_strided_kernel<<<grid, 256, 0, s>>>(kind, op, oa, ob, g, out->data, total);
  return check_launch(fn);
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_unary(int32_t op, const oxc_view* in, const oxc_view* out, void* stream) {
  if (op < 0 || op > 18) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown unary op id %d", op);
  return run_elementwise(EK_UNARY, op, in, nullptr, nullptr, 0, out,
                         static_cast<cudaStream_t>(stream), "oxc_unary");
}

oxc_status oxc_contiguous(const oxc_view* in, const oxc_view* out, void* stream) {
  return run_elementwise(EK_UNARY, kUnaryCopy, in, nullptr, nullptr, 0, out,
                         static_cast<cudaStream_t>(stream), "oxc_contiguous");
}

oxc_status oxc_binary(int32_t op, const oxc_view* a, const oxc_view* b, const oxc_view* out,
                      void* stream) {
  if (op < 0 || op > 6) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown binary op id %d", op);
  return run_elementwise(EK_BINARY, op, a, b, nullptr, 0, out, static_cast<cudaStream_t>(stream),
                         "oxc_binary");
}

oxc_status oxc_cmp(int32_t op, const oxc_view* a, const oxc_view* b, const oxc_view* out,
                   void* stream) {
  if (op < 0 || op > 5) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown comparison op id %d", op);
  return run_elementwise(EK_CMP, op, a, b, nullptr, 0, out, static_cast<cudaStream_t>(stream),
                         "oxc_cmp");
}

oxc_status oxc_binary_scalar(int32_t op, const oxc_view* a, float scalar, int32_t scalar_first,
                             const oxc_view* out, void* stream) {
  if (op < 0 || op > 6) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: unknown binary op id %d", op);
  return run_elementwise(EK_BINARY, op, a, a, &scalar, scalar_first, out,
                         static_cast<cudaStream_t>(stream), "oxc_binary_scalar");
}

}  // extern "C"
