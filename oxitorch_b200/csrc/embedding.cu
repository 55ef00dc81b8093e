// embedding.cu -- F.embedding forward (Tensor::index_select along dim 0) and
// its duplicate-id VJP (scatter_index_select).
//
// Reference: python/oxitorch/nn/functional.py:245-247 -> weight.index_select(0, ids)
//   forward  crates/oxi-tensor/src/lib.rs:665-703: ids validated first (negative
//            ids count from the end; out of range -> OutOfBounds), then a row copy.
//   VJP      crates/oxi-autograd/src/ops.rs:741-769: dtable = zeros, then
//            dtable[id_k] += dout[k] for k in position order -- so every table row
//            is a left-to-right f32 sum, from 0.0, of its occurrences.
//
// B200 design:
//   gather: one CTA per output row (grid-stride), 128-bit copies; table rows
//     are read with L2-allocating loads (hot ids repeat), outputs streamed.
//   VJP:
//     1. prepare: ids -> (key = resolved row, value = position); bad ids
//        recorded in the error flag and keyed past the table (ignored).
//     2. stable radix sort of (key, position) pairs (CUB, header-only, part of
//        the CUDA toolkit): equal keys keep increasing position order.
//     3. offsets: segment starts read straight off the sorted keys.
//     4. split pieces: rows occurring more than P times are cut at the fixed
//        P-position blocks (P = 128) of the sorted array; one CTA per block and
//        column chunk sums its (at most two) pieces of such rows into partial rows.
//     5. rows: one CTA per table row and column chunk writes zeros (no occurrence), the
//        left-to-right sum of its <= P occurrences in position order
//        (bit-identical to the reference), or the sum of its pieces in block
//        order (deterministic; differs from the reference only by summation
//        order).
//   Sharded tables (vocab-parallel): the table holds rows
//   [vocab_offset, vocab_offset + rows); ids outside are zero rows forward
//   and contribute nothing backward.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include <algorithm>

#include "common.cuh"

namespace oxc {

constexpr int kSplitP = 128;  // occurrences per piece for hot rows
constexpr int kEmbChunkThreads = 128;  // threads per CTA of the VJP (one column chunk each)

// Resolved row inside this shard, or -1 (outside the shard / out of range).
// Sets *bad when the id is out of range of the whole table.
__device__ __forceinline__ int64_t emb_row(int64_t id, int64_t vocab_total, int64_t offset,
                                           int64_t rows, bool* bad) {
  const int64_t r = id < 0 ? id + vocab_total : id;
  if (r < 0 || r >= vocab_total) {
    *bad = true;
    return -1;
  }
  *bad = false;
  const int64_t local = r - offset;
  return (local >= 0 && local < rows) ? local : -1;
}

__device__ __forceinline__ void emb_record_bad(int32_t* flag, int64_t value, int64_t size) {
  if (flag && atomicCAS(flag, 0, 1) == 0) {
    flag[1] = (int32_t)(uint32_t)((uint64_t)value & 0xffffffffu);
    flag[2] = (int32_t)(uint32_t)((uint64_t)value >> 32);
    flag[3] = (int32_t)size;
  }
}

template <int VW>
__global__ void __launch_bounds__(256) emb_gather_kernel(
    const float* __restrict__ table, const int64_t* __restrict__ ids, float* __restrict__ out,
    int64_t n, int64_t vocab_total, int64_t offset, int64_t rows, int cols, int32_t* err) {
  const int nvec = cols / VW;
  for (int64_t k = blockIdx.x; k < n; k += gridDim.x) {
    const int64_t id = ids[k];
    bool bad;
    const int64_t r = emb_row(id, vocab_total, offset, rows, &bad);
    if (bad && threadIdx.x == 0) emb_record_bad(err, id, vocab_total);
    float* dst = out + k * (int64_t)cols;
    if constexpr (VW == 4) {
      float4* d4 = reinterpret_cast<float4*>(dst);
      if (r < 0) {
        for (int v = threadIdx.x; v < nvec; v += blockDim.x) st_stream(d4 + v, make_float4(0, 0, 0, 0));
      } else {
        const float4* s4 = reinterpret_cast<const float4*>(table + r * (int64_t)cols);
        int v = threadIdx.x;
        for (; v + 3 * (int)blockDim.x < nvec; v += 4 * blockDim.x) {
          float4 q[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) q[u] = ld_keep(s4 + v + u * blockDim.x);
#pragma unroll
          for (int u = 0; u < 4; ++u) st_stream(d4 + v + u * blockDim.x, q[u]);
        }
        for (; v < nvec; v += blockDim.x) st_stream(d4 + v, ld_keep(s4 + v));
      }
    } else {
      const float* src = r < 0 ? nullptr : table + r * (int64_t)cols;
      for (int c = threadIdx.x; c < cols; c += blockDim.x)
        st_stream(dst + c, src ? ld_keep(src + c) : 0.0f);
    }
  }
}

// keys[k] = row of ids[k] in this shard (rows if outside: sorts after every
// real row and is ignored); vals[k] = k.
__global__ void emb_prepare_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t vocab_total,
                                   int64_t offset, int64_t rows, int32_t* __restrict__ keys,
                                   int32_t* __restrict__ vals, int32_t* err) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n;
       k += (int64_t)gridDim.x * blockDim.x) {
    bool bad;
    const int64_t r = emb_row(ids[k], vocab_total, offset, rows, &bad);
    if (bad) emb_record_bad(err, ids[k], vocab_total);
    keys[k] = (int32_t)(r < 0 ? rows : r);
    vals[k] = (int32_t)k;
  }
}

// offsets[r] = first sorted index with key >= r, for r in [0, rows].
__global__ void emb_offsets_kernel(const int32_t* __restrict__ skeys, int64_t n, int64_t rows,
                                   int32_t* __restrict__ offsets) {
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p <= n;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t prev = p > 0 ? min((int64_t)skeys[p - 1], rows) : -1;
    const int64_t cur = p < n ? min((int64_t)skeys[p], rows) : rows;
    for (int64_t r = prev + 1; r <= cur; ++r) offsets[r] = (int32_t)p;
  }
}

// Sums dout rows spos[p0..p1) (in order) into acc for this thread's columns;
// four rows' loads are in flight before they are added in position order.
template <int VW, int VPT>
__device__ __forceinline__ void sum_positions(const float* __restrict__ dout,
                                              const int32_t* __restrict__ spos, int64_t p0,
                                              int64_t p1, int cols, int c_base,
                                              float (&acc)[VPT][VW]) {
  const int nvec = cols / VW;
  constexpr int U = 4;
  for (int64_t p = p0; p < p1; p += U) {
    float q[U][VPT][VW];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const bool live = p + j < p1;
      const float* row = dout + (live ? (int64_t)spos[p + j] : 0) * cols;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int v = c_base + i * blockDim.x + threadIdx.x;
        if (live && v < nvec) {
          if constexpr (VW == 4) {
            const float4 a = ld_stream(reinterpret_cast<const float4*>(row) + v);
            q[j][i][0] = a.x; q[j][i][1] = a.y; q[j][i][2] = a.z; q[j][i][3] = a.w;
          } else {
            q[j][i][0] = ld_stream(row + v);
          }
        } else {
#pragma unroll
          for (int e = 0; e < VW; ++e) q[j][i][e] = 0.0f;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (p + j < p1) {
#pragma unroll
        for (int i = 0; i < VPT; ++i)
#pragma unroll
          for (int e = 0; e < VW; ++e) acc[i][e] = __fadd_rn(acc[i][e], q[j][i][e]);
      }
  }
}

template <int VW, int VPT>
__device__ __forceinline__ void store_acc(float* dst, int cols, int c_base,
                                          const float (&acc)[VPT][VW], bool streaming) {
  const int nvec = cols / VW;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = c_base + i * blockDim.x + threadIdx.x;
    if (v < nvec) {
      if constexpr (VW == 4) {
        const float4 o = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        if (streaming) st_stream(reinterpret_cast<float4*>(dst) + v, o);
        else reinterpret_cast<float4*>(dst)[v] = o;
      } else {
        if (streaming) st_stream(dst + v, acc[i][0]);
        else dst[v] = acc[i][0];
      }
    }
  }
}

// The split and row kernels run on a linear grid: CTA b takes column chunk
// b % chunks of row slot b / chunks, so the chunks of one row (or one block of
// positions) run side by side and each dout row is read whole at about the
// same time, instead of in chunk-sized pieces far apart in time.
struct ChunkGrid {
  int64_t slot, slots;
  int chunk, chunks;
};
__device__ __forceinline__ ChunkGrid chunk_grid(int chunks) {
  return ChunkGrid{(int64_t)(blockIdx.x / (unsigned)chunks), (int64_t)(gridDim.x / (unsigned)chunks),
                   (int)(blockIdx.x % (unsigned)chunks), chunks};
}

// Block j of the sorted array: partial sums of the (at most two) pieces of
// rows that occur more than kSplitP times.  Slot 2j: the row covering
// position j*P (if split); slot 2j+1: a split row that starts inside block j.
// With outer > 1 (index_select's VJP along an inner dim) the same segments
// serve every outer index o (blockIdx.z): its dout rows start at o * n * cols,
// its table rows at o * rows * cols and its pieces at o * 2 * nblocks * cols.
template <int VW, int VPT, int MAXT>
__global__ void __launch_bounds__(MAXT) emb_split_kernel(
    const float* __restrict__ dout, const int32_t* __restrict__ skeys,
    const int32_t* __restrict__ spos, const int32_t* __restrict__ offsets, int64_t n,
    int64_t rows, int cols, float* __restrict__ parts, int64_t outer, int chunks) {
  // emb_rows_kernel may start on the rows that need no pieces while this grid
  // runs (it was launched after the sort and offsets had completed)
  pdl_launch_dependents();
  const ChunkGrid cg = chunk_grid(chunks);
  const int nvec = cols / VW;
  const int64_t nblocks = (n + kSplitP - 1) / kSplitP;
  for (int64_t j = cg.slot; j < nblocks; j += cg.slots) {
  const int64_t b0 = j * kSplitP, b1 = min(n, b0 + kSplitP);
  const int64_t keys2[2] = {skeys[b0], skeys[b1 - 1]};
  for (int64_t o = blockIdx.z; o < outer; o += gridDim.z) {
    const float* od = dout + o * n * (int64_t)cols;
    for (int side = 0; side < 2; ++side) {
      const int64_t r = keys2[side];
      if (r >= rows) continue;
      if (side == 1 && r == keys2[0]) continue;
      const int64_t s0 = offsets[r], s1 = offsets[r + 1];
      if (s1 - s0 <= kSplitP) continue;
      const int64_t p0 = max(s0, b0), p1 = min(s1, b1);
      float* dst = parts + (o * 2 * nblocks + 2 * j + side) * (int64_t)cols;
      for (int c_base = cg.chunk * VPT * blockDim.x; c_base < nvec;
           c_base += cg.chunks * VPT * blockDim.x) {
        float acc[VPT][VW];
#pragma unroll
        for (int i = 0; i < VPT; ++i)
#pragma unroll
          for (int e = 0; e < VW; ++e) acc[i][e] = 0.0f;
        sum_positions<VW, VPT>(od, spos, p0, p1, cols, c_base, acc);
        store_acc<VW, VPT>(dst, cols, c_base, acc, false);
      }
    }
  }
  }
}

// Ownership under a push table.  Contiguous shards: owner p holds rows
// [lo[p], lo[p+1]).  Cyclic: owner p holds rows p, p + world, p + 2 world, ...
// The presence scan runs in owner-major order, so each owner's occurring rows
// take consecutive slots: position push_pos(r) in that order, owner p's first
// position push_base(p).  Contiguous: the order of the rows themselves.
// Cyclic: p * span + r / world, span = ceil(rows / world) positions per owner,
// the positions past the last row of an owner empty.  Every position is below
// rows + OXC_PUSH_MAX_RANKS.  r's index in its owner's region for this source
// is then slot[push_pos(r)] - slot[push_base(p)].
__device__ __forceinline__ int push_owner(const oxc_emb_push* __restrict__ push, int64_t r) {
  if (push->cyclic) return (int)(r % push->world);
  int p = 0;
  while (p + 1 < push->world && r >= push->lo[p + 1]) ++p;
  return p;
}
__device__ __forceinline__ int64_t push_span(const oxc_emb_push* __restrict__ push, int64_t rows) {
  return (rows + push->world - 1) / push->world;
}
__device__ __forceinline__ int64_t push_pos(const oxc_emb_push* __restrict__ push, int64_t r,
                                            int64_t rows) {
  if (!push->cyclic) return r;
  return (r % push->world) * push_span(push, rows) + r / push->world;
}
__device__ __forceinline__ int64_t push_base(const oxc_emb_push* __restrict__ push, int p,
                                             int64_t rows) {
  return push->cyclic ? (int64_t)p * push_span(push, rows) : push->lo[p];
}
// The table row at owner-major position q, or -1 (an empty cyclic position).
__device__ __forceinline__ int64_t push_row_at(const oxc_emb_push* __restrict__ push, int64_t q,
                                               int64_t rows) {
  if (!push->cyclic) return q < rows ? q : -1;
  const int64_t span = push_span(push, rows);
  const int64_t r = (q % span) * push->world + q / span;
  return q / span < push->world && r < rows ? r : -1;
}

// With `slot` (the compact VJP, outer == 1), rows without occurrences are
// skipped and row r is written at dtable + slot[r] * cols; with PUSH (and
// `slot`), at its owner's region instead (peer memory), and the stores are
// fenced at system scope before the grid completes.  PUSH is a template
// argument so that the plain VJP carries none of its registers (70 against
// 54 per thread at float4 rows, which cost two CTAs per SM).
template <int VW, int VPT, int MAXT, bool PUSH>
__global__ void __launch_bounds__(MAXT) emb_rows_kernel(
    const float* __restrict__ dout_all, const int32_t* __restrict__ spos,
    const int32_t* __restrict__ offsets, const float* __restrict__ parts_all, int64_t rows,
    int cols, float* __restrict__ dtable, int64_t n, int64_t outer,
    const int32_t* __restrict__ slot, const oxc_emb_push* __restrict__ push, int32_t* err,
    int chunks) {
  // Launched as a programmatic dependent of emb_split_kernel: rows with at
  // most kSplitP occurrences read only the sort's output and run while the
  // split grid is still working; rows made of pieces wait for it (pdl_wait)
  // before reading `parts`, and every CTA waits once more before it exits,
  // so this grid never completes ahead of the split grid.
  const ChunkGrid cg = chunk_grid(chunks);
  const int nvec = cols / VW;
  const int64_t nblocks = (n + kSplitP - 1) / kSplitP;
  bool remote = false;  // PUSH: this thread stored a row into another rank's memory
  // PUSH walks the rows interleaved across their owners (row q of owner 0,
  // of owner 1, ..., then row q + 1), so the stores into other ranks' memory
  // spread over the whole launch instead of crowding NVLink while the rows
  // of one shard pass.
  // (Cyclic ownership interleaves the owners in row order already.)
  int64_t span = rows;
  if constexpr (PUSH) {
    if (!push->cyclic) {
      int64_t widest = 0;  // the largest shard: every row of every shard is visited
      for (int q = 0; q < push->world; ++q) widest = max(widest, push->lo[q + 1] - push->lo[q]);
      span = (int64_t)push->world * widest;
    }
  }
  for (int64_t o = blockIdx.z; o < outer; o += gridDim.z)
  for (int64_t j = cg.slot; j < span; j += cg.slots) {
    int64_t r = j;
    int p = 0;
    if constexpr (PUSH) {
      if (push->cyclic) {
        p = (int)(j % push->world);
      } else {
        p = (int)(j % push->world);
        r = push->lo[p] + j / push->world;
        if (r >= push->lo[p + 1] || r >= rows || r < 0) continue;
      }
    }
    const float* dout = dout_all + o * n * (int64_t)cols;
    const float* parts = parts_all + o * 2 * nblocks * (int64_t)cols;
    const int64_t s0 = offsets[r], s1 = offsets[r + 1];
    if (slot && s1 == s0) continue;
    float* dst = dtable + (slot ? (int64_t)slot[r] : o * rows + r) * (int64_t)cols;
    if constexpr (PUSH) {
      const int64_t idx =
          (int64_t)slot[push_pos(push, r, rows)] - slot[push_base(push, p, rows)];
      if (idx >= push->cap) {
        if (err && threadIdx.x == 0 && atomicCAS(err, 0, 1) == 0) {
          err[1] = (int32_t)r;
          err[2] = 0;
          err[3] = (int32_t)push->cap;
        }
        continue;
      }
      dst = push->rows[p] + idx * (int64_t)cols;
      remote |= p != push->source && !push->local;
    }
    for (int c_base = cg.chunk * VPT * blockDim.x; c_base < nvec;
         c_base += cg.chunks * VPT * blockDim.x) {
      float acc[VPT][VW];
#pragma unroll
      for (int i = 0; i < VPT; ++i)
#pragma unroll
        for (int e = 0; e < VW; ++e) acc[i][e] = 0.0f;
      if (s1 - s0 <= kSplitP) {
        sum_positions<VW, VPT>(dout, spos, s0, s1, cols, c_base, acc);
      } else {
        pdl_wait();  // the pieces are the split grid's output
        // pieces in block order, eight partial rows in flight per step
        const int64_t j0 = s0 / kSplitP, j1 = (s1 - 1) / kSplitP;
        constexpr int UJ = 8;
        for (int64_t jb = j0; jb <= j1; jb += UJ) {
          float q[UJ][VPT][VW];
#pragma unroll
          for (int u = 0; u < UJ; ++u) {
            const int64_t j = jb + u;
            const int side = (j == j0 && s0 != j0 * kSplitP) ? 1 : 0;
            const float* src = parts + (2 * min(j, j1) + side) * (int64_t)cols;
#pragma unroll
            for (int i = 0; i < VPT; ++i) {
              const int v = c_base + i * blockDim.x + threadIdx.x;
              if (j <= j1 && v < nvec) {
                if constexpr (VW == 4) {
                  const float4 a = reinterpret_cast<const float4*>(src)[v];
                  q[u][i][0] = a.x; q[u][i][1] = a.y; q[u][i][2] = a.z; q[u][i][3] = a.w;
                } else {
                  q[u][i][0] = src[v];
                }
              } else {
#pragma unroll
                for (int e = 0; e < VW; ++e) q[u][i][e] = 0.0f;
              }
            }
          }
#pragma unroll
          for (int u = 0; u < UJ; ++u)
            if (jb + u <= j1) {
#pragma unroll
              for (int i = 0; i < VPT; ++i)
#pragma unroll
                for (int e = 0; e < VW; ++e) acc[i][e] = __fadd_rn(acc[i][e], q[u][i][e]);
            }
        }
      }
      store_acc<VW, VPT>(dst, cols, c_base, acc, true);
    }
  }
  pdl_wait();
  if constexpr (PUSH) {
    // The peer stores are visible at system scope before the grid completes:
    // one fence per CTA that stored into another rank's memory, after a
    // barrier that orders every thread's stores before it (a fence's release
    // covers the writes that happen before it), instead of a fence in every
    // thread, each waiting for its own stores.
    if (__syncthreads_or(remote) && threadIdx.x == 0) __threadfence_system();
  }
}

// ---- index_select along any dim (Tensor::index_select, lib.rs:665-703) ----------

// Records the first bad id of an index_select along `dim`: flag[0] = 1 + dim.
__device__ __forceinline__ void isel_record_bad(int32_t* flag, int64_t value, int64_t size,
                                                int dim) {
  if (flag && atomicCAS(flag, 0, 1 + dim) == 0) {
    flag[1] = (int32_t)(uint32_t)((uint64_t)value & 0xffffffffu);
    flag[2] = (int32_t)(uint32_t)((uint64_t)value >> 32);
    flag[3] = (int32_t)size;
  }
}

// Resolved index in [0, len) (negative ids count from the end), or -1.
__device__ __forceinline__ int64_t isel_resolve(int64_t id, int64_t len) {
  const int64_t r = id < 0 ? id + len : id;
  return (r >= 0 && r < len) ? r : -1;
}

// Contiguous x viewed as [outer, len, inner] with inner >= 32: one CTA per
// output slice (o, k), which copies x[o, ids[k], :] (128-bit when VW = 4).
template <int VW>
__global__ void __launch_bounds__(256) isel_rows_kernel(
    const float* __restrict__ x, const int64_t* __restrict__ ids, float* __restrict__ out,
    int64_t outer, int64_t len, int64_t n, int64_t inner, int dim, int32_t* err) {
  const int64_t nvec = inner / VW, slices = outer * n;
  for (int64_t row = blockIdx.x; row < slices; row += gridDim.x) {
    const int64_t o = row / n, k = row - o * n;
    const int64_t r = isel_resolve(ids[k], len);
    if (r < 0 && threadIdx.x == 0) isel_record_bad(err, ids[k], len, dim);
    float* dst = out + row * inner;
    if constexpr (VW == 4) {
      float4* d4 = reinterpret_cast<float4*>(dst);
      const float4* s4 = reinterpret_cast<const float4*>(x + (o * len + (r < 0 ? 0 : r)) * inner);
      for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x)
        st_stream(d4 + v, r < 0 ? make_float4(0, 0, 0, 0) : ld_keep(s4 + v));
    } else {
      const float* src = x + (o * len + (r < 0 ? 0 : r)) * inner;
      for (int64_t c = threadIdx.x; c < inner; c += blockDim.x)
        st_stream(dst + c, r < 0 ? 0.0f : ld_keep(src + c));
    }
  }
}

// Any strides: one thread per output element.  g.n is the output shape
// (n[dim] = number of ids), g.st the strides of x.
struct ISelGrid {
  int nd, dim;
  int64_t len;
  int64_t n[OXC_MAX_DIMS];
  int64_t st[OXC_MAX_DIMS];
};

__global__ void __launch_bounds__(256) isel_elem_kernel(const float* __restrict__ x,
                                                        const int64_t* __restrict__ ids,
                                                        ISelGrid g, float* __restrict__ out,
                                                        int64_t total, int32_t* err) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = e, off = 0;
    bool bad = false;
    for (int d = g.nd - 1; d >= 0; --d) {
      const int64_t q = rem / g.n[d];
      int64_t idx = rem - q * g.n[d];
      rem = q;
      if (d == g.dim) {
        const int64_t r = isel_resolve(ids[idx], g.len);
        if (r < 0) {
          isel_record_bad(err, ids[idx], g.len, g.dim);
          bad = true;
        }
        idx = r < 0 ? 0 : r;
      }
      off += idx * g.st[d];
    }
    out[e] = bad ? 0.0f : __ldg(x + off);
  }
}

// The VJP for slices narrower than a float4 chunk row (inner < 128): one
// thread per gx element (o, r, i) sums g[o, k, i] over the occurrences k of
// row r in position order, from 0.0 -- the reference's accumulation order
// (crates/oxi-autograd/src/ops.rs:756-763), so every element is bit-identical.
__global__ void __launch_bounds__(256) isel_bwd_narrow_kernel(
    const float* __restrict__ g, const int32_t* __restrict__ spos,
    const int32_t* __restrict__ offsets, int64_t outer, int64_t len, int64_t n, int64_t inner,
    float* __restrict__ gx) {
  const int64_t total = outer * len * inner;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e % inner, t = e / inner;
    const int64_t r = t % len, o = t / len;
    const int64_t s0 = offsets[r], s1 = offsets[r + 1];
    const float* go = g + o * n * inner + i;
    float acc = 0.0f;
    for (int64_t p = s0; p < s1; ++p) acc = __fadd_rn(acc, __ldg(go + (int64_t)spos[p] * inner));
    gx[e] = acc;
  }
}

// ---- the compact VJP and the sparse exchange of a replicated table's gradient ----

// present[r] = 1 if table row r occurs, for the exclusive scan that gives
// each occurring row its compact slot.
__global__ void emb_present_kernel(const int32_t* __restrict__ offsets, int64_t rows,
                                   int32_t* __restrict__ present) {
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows;
       r += (int64_t)gridDim.x * blockDim.x)
    present[r] = offsets[r + 1] > offsets[r] ? 1 : 0;
}

// Compact ids (global table rows), the distinct count, and per destination
// shard the number of distinct rows it owns (shard s = rows [V*s/G, V*(s+1)/G)
// of the whole vocab_total-row table, this table covering [offset, offset +
// rows)).
__global__ void emb_compact_meta_kernel(const int32_t* __restrict__ present,
                                        const int32_t* __restrict__ slot, int64_t rows,
                                        int64_t vocab_total, int64_t offset, int32_t shards,
                                        int32_t* __restrict__ out_ids,
                                        int64_t* __restrict__ count,
                                        int64_t* __restrict__ shard_counts) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t r = tid; r < rows; r += (int64_t)gridDim.x * blockDim.x)
    if (present[r]) out_ids[slot[r]] = (int32_t)(r + offset);
  if (tid == 0) *count = rows ? (int64_t)slot[rows - 1] + present[rows - 1] : 0;
  if (shard_counts && tid < shards) {
    const int64_t s = tid;
    // rows of shard s inside this table, clamped
    auto bound = [&](int64_t g) -> int64_t {
      const int64_t l = vocab_total * g / shards - offset;
      return l < 0 ? 0 : (l > rows ? rows : l);
    };
    const int64_t lo = bound(s), hi = bound(s + 1);
    auto pre = [&](int64_t r) -> int64_t {
      return r >= rows ? (rows ? (int64_t)slot[rows - 1] + present[rows - 1] : 0) : slot[r];
    };
    shard_counts[s] = pre(hi) - pre(lo);
  }
}

// The push presence flags in owner-major order (push_pos): position q holds 1
// if its table row occurs; the positions past the rows, up to rows +
// OXC_PUSH_MAX_RANKS, hold 0, so the exclusive scan of all of them defines
// slot[q] for every position an owner's bounds can name.
__global__ void emb_push_present_kernel(const int32_t* __restrict__ offsets, int64_t rows,
                                        const oxc_emb_push* __restrict__ push,
                                        int32_t* __restrict__ present) {
  const int64_t len = rows + OXC_PUSH_MAX_RANKS;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < len;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = push_row_at(push, q, rows);
    present[q] = r >= 0 && offsets[r + 1] > offsets[r] ? 1 : 0;
  }
}

// The push meta: every occurring row's id into its owner's id region, and
// each owner's count of this source's rows (differences of the owner-major
// slots at the owners' bounds).
__global__ void emb_push_meta_kernel(const int32_t* __restrict__ present,
                                     const int32_t* __restrict__ slot, int64_t rows,
                                     const oxc_emb_push* __restrict__ push, int32_t* err) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t len = rows + OXC_PUSH_MAX_RANKS;
  auto pre = [&](int64_t q) -> int64_t {
    q = q < 0 ? 0 : q;
    return q >= len ? (int64_t)slot[len - 1] + present[len - 1] : slot[q];
  };
  for (int64_t q = tid; q < len; q += (int64_t)gridDim.x * blockDim.x) {
    if (!present[q]) continue;
    const int64_t r = push_row_at(push, q, rows);
    const int p = push_owner(push, r);
    const int64_t idx = (int64_t)slot[q] - pre(push_base(push, p, rows));
    if (idx < push->cap) push->ids[p][idx] = (int32_t)r;
  }
  if (tid < push->world) {
    const int p = (int)tid;
    const int64_t hi = p + 1 < push->world ? push_base(push, p + 1, rows)
                       : (push->cyclic ? push->world * push_span(push, rows) : push->lo[p + 1]);
    const int64_t c = pre(hi) - pre(push_base(push, p, rows));
    if (c > push->cap && err && atomicCAS(err, 0, 1) == 0) {
      err[1] = (int32_t)c;
      err[2] = 0;
      err[3] = (int32_t)push->cap;
    }
    *push->count[p] = c < push->cap ? c : push->cap;
  }
  __syncthreads();  // one system-scope fence per CTA covers every thread's stores
  if (threadIdx.x == 0) __threadfence_system();
}

// The pull form's owner side.  map[s * shard_rows + v] = the index in source
// s's region of the owner's shard row v (table row shard_lo + v *
// shard_stride), or -1.  The counts are read once per CTA.
__global__ void emb_pull_map_kernel(const oxc_emb_pull* __restrict__ pull, int32_t sources,
                                    int64_t cap, int64_t shard_lo, int64_t shard_stride,
                                    int64_t shard_rows, int32_t* __restrict__ map, int32_t* err) {
  __shared__ int64_t cnt[OXC_PUSH_MAX_RANKS];
  if (threadIdx.x < sources) cnt[threadIdx.x] = *pull->count[threadIdx.x];
  __syncthreads();
  const int64_t total = (int64_t)sources * cap;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int s = (int)(i / cap);
    const int64_t k = i - (int64_t)s * cap;
    if (k >= cnt[s]) continue;
    const int64_t id = pull->ids[s][k];
    const int64_t d = id - shard_lo;
    const int64_t v = d / shard_stride;
    if (d < 0 || d % shard_stride != 0 || v >= shard_rows) {
      if (err && atomicCAS(err, 0, 1) == 0) {
        err[1] = (int32_t)id;
        err[2] = 0;
        err[3] = (int32_t)shard_rows;
      }
      continue;
    }
    map[(int64_t)s * shard_rows + v] = (int32_t)k;
  }
}

// dshard[v] = sum over sources s in rank order, from 0.0, of row map[s][v] of
// s's region (skipped where -1): the same sums as emb_exchange_reduce_kernel.
// Every source's load is issued before the adds, so a thread keeps up to
// `sources` NVLink reads in flight.
template <int VW>
__global__ void __launch_bounds__(128) emb_pull_reduce_kernel(
    const oxc_emb_pull* __restrict__ pull, const int32_t* __restrict__ map, int32_t sources,
    int64_t shard_rows, int cols, float* __restrict__ dshard) {
  __shared__ const float* src[OXC_PUSH_MAX_RANKS];
  if (threadIdx.x < sources) src[threadIdx.x] = pull->rows[threadIdx.x];
  __syncthreads();
  const int nvec = cols / VW;
  for (int64_t v = blockIdx.x; v < shard_rows; v += gridDim.x) {
    int32_t idx[OXC_PUSH_MAX_RANKS];
#pragma unroll
    for (int s = 0; s < OXC_PUSH_MAX_RANKS; ++s)
      idx[s] = s < sources ? map[(int64_t)s * shard_rows + v] : -1;
    for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < nvec; c += gridDim.y * blockDim.x) {
      float q[OXC_PUSH_MAX_RANKS][VW];
#pragma unroll
      for (int s = 0; s < OXC_PUSH_MAX_RANKS; ++s) {
        if (idx[s] >= 0) {
          if constexpr (VW == 4) {
            const float4 a =
                ld_stream(reinterpret_cast<const float4*>(src[s] + (int64_t)idx[s] * cols) + c);
            q[s][0] = a.x; q[s][1] = a.y; q[s][2] = a.z; q[s][3] = a.w;
          } else {
            q[s][0] = ld_stream(src[s] + (int64_t)idx[s] * cols + c);
          }
        }
      }
      float acc[VW];
#pragma unroll
      for (int e = 0; e < VW; ++e) acc[e] = 0.0f;
#pragma unroll
      for (int s = 0; s < OXC_PUSH_MAX_RANKS; ++s)
        if (idx[s] >= 0) {
#pragma unroll
          for (int e = 0; e < VW; ++e) acc[e] = __fadd_rn(acc[e], q[s][e]);
        }
      if constexpr (VW == 4)
        st_stream(reinterpret_cast<float4*>(dshard + v * cols) + c,
                  make_float4(acc[0], acc[1], acc[2], acc[3]));
      else
        st_stream(dshard + v * cols + c, acc[0]);
    }
  }
}

// The owner's side of the fused exchange: region s of recv holds counts[s]
// rows; map[s * shard_rows + v] = the region index of table row shard_lo +
// v * shard_stride (the owner's shard row v), or -1.
__global__ void emb_region_map_kernel(const int32_t* __restrict__ recv_ids,
                                      const int64_t* __restrict__ counts, int32_t sources,
                                      int64_t cap, int64_t shard_lo, int64_t shard_stride,
                                      int64_t shard_rows, int32_t* __restrict__ map,
                                      int32_t* err) {
  const int64_t total = (int64_t)sources * cap;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = i / cap, k = i - s * cap;
    if (k >= counts[s]) continue;
    const int64_t d = (int64_t)recv_ids[i] - shard_lo;
    const int64_t v = d / shard_stride;
    if (d < 0 || d % shard_stride != 0 || v >= shard_rows) {
      if (err && atomicCAS(err, 0, 1) == 0) {
        err[1] = recv_ids[i];
        err[2] = 0;
        err[3] = (int32_t)shard_rows;
      }
      continue;
    }
    map[s * shard_rows + v] = (int32_t)i;
  }
}

// The owner's side of the sparse exchange: dshard[v] (v < shard_rows) is the
// sum, in source-rank order from 0.0, of the rows received for table row
// shard_lo + v.  map[s * shard_rows + v] = index of that row in recv_rows, or
// -1; filled by emb_exchange_map_kernel.
__global__ void emb_exchange_map_kernel(const int32_t* __restrict__ recv_ids,
                                        const int64_t* __restrict__ src_off, int32_t sources,
                                        int64_t shard_lo, int64_t shard_rows,
                                        int32_t* __restrict__ map, int32_t* err) {
  const int64_t total = src_off[sources];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int s = 0;
    while (s + 1 < sources && src_off[s + 1] <= i) ++s;
    const int64_t v = (int64_t)recv_ids[i] - shard_lo;
    if (v < 0 || v >= shard_rows) {
      if (err && atomicCAS(err, 0, 1) == 0) {
        err[1] = recv_ids[i];
        err[2] = 0;
        err[3] = (int32_t)shard_rows;
      }
      continue;
    }
    map[(int64_t)s * shard_rows + v] = (int32_t)i;
  }
}

template <int VW>
__global__ void __launch_bounds__(128) emb_exchange_reduce_kernel(
    const float* __restrict__ recv_rows, const int32_t* __restrict__ map, int32_t sources,
    int64_t shard_rows, int cols, float* __restrict__ dshard) {
  const int nvec = cols / VW;
  for (int64_t v = blockIdx.x; v < shard_rows; v += gridDim.x) {
    int32_t idx[8];
    const int ns = sources < 8 ? sources : 8;
    for (int s = 0; s < ns; ++s) idx[s] = map[(int64_t)s * shard_rows + v];
    for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < nvec; c += gridDim.y * blockDim.x) {
      float acc[VW];
#pragma unroll
      for (int e = 0; e < VW; ++e) acc[e] = 0.0f;
      for (int s = 0; s < sources; ++s) {
        const int32_t i = s < 8 ? idx[s] : map[(int64_t)s * shard_rows + v];
        if (i < 0) continue;
        if constexpr (VW == 4) {
          const float4 q = ld_stream(reinterpret_cast<const float4*>(recv_rows + (int64_t)i * cols) + c);
          acc[0] = __fadd_rn(acc[0], q.x); acc[1] = __fadd_rn(acc[1], q.y);
          acc[2] = __fadd_rn(acc[2], q.z); acc[3] = __fadd_rn(acc[3], q.w);
        } else {
          acc[0] = __fadd_rn(acc[0], ld_stream(recv_rows + (int64_t)i * cols + c));
        }
      }
      if constexpr (VW == 4)
        st_stream(reinterpret_cast<float4*>(dshard + v * cols) + c,
                  make_float4(acc[0], acc[1], acc[2], acc[3]));
      else
        st_stream(dshard + v * cols + c, acc[0]);
    }
  }
}

struct EmbLayout {
  size_t keys_in, vals_in, keys_out, vals_out, offsets, parts, cub, total;
  size_t cub_bytes;
  int end_bit;
  size_t present, slot, scan, scan_bytes;  // the compact VJP only
};

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static oxc_status emb_layout(int64_t n, int64_t rows, int64_t cols, EmbLayout* L,
                             int64_t outer = 1, bool compact = false) {
  int end_bit = 1;
  while (end_bit < 31 && ((int64_t)1 << end_bit) <= rows) ++end_bit;  // keys in [0, rows]
  size_t cub_bytes = 0;
  cudaError_t e = cub::DeviceRadixSort::SortPairs(nullptr, cub_bytes, (const int32_t*)nullptr,
                                                  (int32_t*)nullptr, (const int32_t*)nullptr,
                                                  (int32_t*)nullptr, (int)n, 0, end_bit);
  if (e != cudaSuccess) return cuda_fail(e, "embedding backward (sort workspace size)");
  const int64_t nblocks = (n + kSplitP - 1) / kSplitP;
  size_t off = 0;
  L->keys_in = off; off += align256((size_t)n * 4);
  L->vals_in = off; off += align256((size_t)n * 4);
  L->keys_out = off; off += align256((size_t)n * 4);
  L->vals_out = off; off += align256((size_t)n * 4);
  L->offsets = off; off += align256((size_t)(rows + 1) * 4);
  L->parts = off; off += align256((size_t)2 * nblocks * cols * 4 * (size_t)outer);
  L->cub = off; off += align256(cub_bytes);
  L->present = L->slot = L->scan = L->scan_bytes = 0;
  if (compact) {
    size_t scan_bytes = 0;
    // rows + OXC_PUSH_MAX_RANKS positions: the owner-major order of the push
    // VJP (cyclic ownership pads each owner's positions to the same span)
    const int64_t positions = rows + OXC_PUSH_MAX_RANKS;
    e = cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, (const int32_t*)nullptr,
                                      (int32_t*)nullptr, (int)positions);
    if (e != cudaSuccess) return cuda_fail(e, "embedding backward (scan workspace size)");
    L->present = off; off += align256((size_t)(positions + 1) * 4);
    L->slot = off; off += align256((size_t)(positions + 1) * 4);
    L->scan = off; off += align256(scan_bytes);
    L->scan_bytes = scan_bytes;
  }
  L->total = off;
  L->cub_bytes = cub_bytes;
  L->end_bit = end_bit;
  return OXC_OK;
}

static oxc_status emb_check(const char* fn, int64_t n, int64_t vocab_total, int64_t offset,
                            int64_t rows, int64_t cols) {
  if (n < 0 || rows < 0 || cols < 0 || vocab_total < 0 || offset < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative size", fn);
  if (offset + rows > vocab_total)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: %s: shard [%lld, %lld) exceeds the table of %lld rows", fn,
                (long long)offset, (long long)(offset + rows), (long long)vocab_total);
  if (n > 0x7fffffff || rows >= 0x7fffffff || cols > 0x7fffffff)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: %s: sizes beyond 2^31", fn);
  return OXC_OK;
}

// prepare -> stable radix sort of (row, position) -> segment offsets.
static oxc_status emb_sort_phase(const int64_t* ids, int64_t n, int64_t vocab_total,
                                 int64_t vocab_offset, int64_t rows, int32_t* err_flag, char* ws,
                                 const EmbLayout& L, cudaStream_t s) {
  int32_t* keys_in = reinterpret_cast<int32_t*>(ws + L.keys_in);
  int32_t* vals_in = reinterpret_cast<int32_t*>(ws + L.vals_in);
  int32_t* keys_out = reinterpret_cast<int32_t*>(ws + L.keys_out);
  int32_t* vals_out = reinterpret_cast<int32_t*>(ws + L.vals_out);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  const unsigned g1 = (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 8);
  emb_prepare_kernel<<<g1, 256, 0, s>>>(ids, n, vocab_total, vocab_offset, rows, keys_in, vals_in,
                                        err_flag);
  oxc_status st = check_launch("oxc_embedding_bwd (prepare)");
  if (st) return st;
  size_t cub_bytes = L.cub_bytes;
  cudaError_t e = cub::DeviceRadixSort::SortPairs(ws + L.cub, cub_bytes, keys_in, keys_out,
                                                  vals_in, vals_out, (int)n, 0, L.end_bit, s);
  if (e != cudaSuccess) return cuda_fail(e, "oxc_embedding_bwd (sort)");
  const unsigned g2 = (unsigned)std::min<int64_t>((n + 1 + 255) / 256, (int64_t)sm_count() * 8);
  emb_offsets_kernel<<<g2, 256, 0, s>>>(keys_out, n, rows, offsets);
  return check_launch("oxc_embedding_bwd (offsets)");
}

// gridDim.x of a chunk grid: `slots` row slots (or position blocks) of
// `chunks` CTAs each, fewer slots if that would pass 2^31 - 1 CTAs (the
// kernels loop over their slots).
static unsigned chunk_grid_size(int64_t slots, int chunks) {
  const int64_t most = (int64_t)0x7fffffff / chunks;
  return (unsigned)(std::max<int64_t>(1, std::min<int64_t>(slots, most)) * chunks);
}

// hot-row pieces -> per-row sums in position order, into dtable (every row)
// or, with `slot`, into the compact rows of the occurring ids.
static oxc_status emb_sum_phase(const float* dout, int64_t n, int64_t rows, int64_t cols,
                                char* ws, const EmbLayout& L, float* dtable, const int32_t* slot,
                                cudaStream_t s, const oxc_emb_push* push = nullptr,
                                int32_t* err = nullptr) {
  const int32_t* keys_out = reinterpret_cast<const int32_t*>(ws + L.keys_out);
  const int32_t* vals_out = reinterpret_cast<const int32_t*>(ws + L.vals_out);
  const int32_t* offsets = reinterpret_cast<const int32_t*>(ws + L.offsets);
  float* parts = reinterpret_cast<float*>(ws + L.parts);
  const bool v4 = cols % 4 == 0 && aligned16(dout) && aligned16(dtable);
  const int64_t nblocks = (n + kSplitP - 1) / kSplitP;
  const unsigned grows = (unsigned)std::min<int64_t>(rows, (int64_t)sm_count() * 32);
  // Each CTA takes one column chunk of a row (chunk_grid): kEmbChunkThreads
  // threads with one float4 (or four floats) each.  Small CTAs keep many rows'
  // gathers in flight on every SM: on B200 at [32000, 4096] the VJP ran at
  // 4.7 / 4.9 / 5.0 / 5.1 / 5.0 / 4.8 TB/s with 1024 / 512 / 256 / 128 / 64 / 32
  // threads per CTA.
  const int vpt = v4 ? 1 : 4, vw = v4 ? 4 : 1;
  const int64_t per_thread = (int64_t)vpt * vw;
  const int block = (int)std::min<int64_t>(
      kEmbChunkThreads, std::max<int64_t>(32, ((cols / per_thread + 31) / 32) * 32));
  const int chunks = (int)std::min<int64_t>(65535, (cols + block * per_thread - 1) / (block * per_thread));
  const dim3 gsplit(chunk_grid_size(nblocks, chunks)), grow(chunk_grid_size(grows, chunks));
#define OXC_EMB_ROWS(VW, VPT, PUSH)                                                          \
  launch_dependent(emb_rows_kernel<VW, VPT, kEmbChunkThreads, PUSH>, grow, block, s, dout,   \
                   vals_out, offsets, (const float*)parts, rows, (int)cols, dtable, n,       \
                   (int64_t)1, slot, push, err, chunks)
  if (v4) {
    emb_split_kernel<4, 1, kEmbChunkThreads><<<gsplit, block, 0, s>>>(
        dout, keys_out, vals_out, offsets, n, rows, (int)cols, parts, (int64_t)1, chunks);
    if (push) OXC_EMB_ROWS(4, 1, true);
    else OXC_EMB_ROWS(4, 1, false);
  } else {
    emb_split_kernel<1, 4, kEmbChunkThreads><<<gsplit, block, 0, s>>>(
        dout, keys_out, vals_out, offsets, n, rows, (int)cols, parts, (int64_t)1, chunks);
    if (push) OXC_EMB_ROWS(1, 4, true);
    else OXC_EMB_ROWS(1, 4, false);
  }
#undef OXC_EMB_ROWS
  return check_launch("oxc_embedding_bwd");
}

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_embedding_fwd(const float* table, const int64_t* ids, float* out, int64_t n,
                             int64_t vocab_total, int64_t vocab_offset, int64_t rows,
                             int64_t cols, int32_t* err_flag, void* stream) {
  oxc_status st = emb_check("embedding", n, vocab_total, vocab_offset, rows, cols);
  if (st) return st;
  if (n == 0 || cols == 0) return OXC_OK;
  if (!ids || !out || (rows > 0 && !table))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: embedding: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool v4 = cols % 4 == 0 && aligned16(table) && aligned16(out);
  const unsigned grid = (unsigned)std::min<int64_t>(n, (int64_t)sm_count() * 16);
  const int block = v4 ? (int)std::min<int64_t>(256, std::max<int64_t>(32, ((cols / 4 + 31) / 32) * 32))
                       : (int)std::min<int64_t>(256, std::max<int64_t>(32, ((cols + 31) / 32) * 32));
  if (v4)
    emb_gather_kernel<4><<<grid, block, 0, s>>>(table, ids, out, n, vocab_total, vocab_offset,
                                                rows, (int)cols, err_flag);
  else
    emb_gather_kernel<1><<<grid, block, 0, s>>>(table, ids, out, n, vocab_total, vocab_offset,
                                                rows, (int)cols, err_flag);
  return check_launch("oxc_embedding_fwd");
}

size_t oxc_embedding_bwd_workspace_size(int64_t n, int64_t rows, int64_t cols) {
  if (n <= 0 || rows < 0 || cols <= 0) return 0;
  EmbLayout L;
  if (emb_layout(n, rows, cols, &L) != OXC_OK) return 0;
  return L.total;
}

oxc_status oxc_embedding_bwd(const float* dout, const int64_t* ids, float* dtable, int64_t n,
                             int64_t vocab_total, int64_t vocab_offset, int64_t rows,
                             int64_t cols, int32_t* err_flag, void* workspace,
                             size_t workspace_bytes, void* stream) {
  oxc_status st = emb_check("embedding backward", n, vocab_total, vocab_offset, rows, cols);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0 || cols == 0) return OXC_OK;
  if (!dtable) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: embedding backward: null pointer");
  if (n == 0) {
    cudaError_t e = cudaMemsetAsync(dtable, 0, (size_t)rows * cols * sizeof(float), s);
    return e == cudaSuccess ? OXC_OK : cuda_fail(e, "oxc_embedding_bwd");
  }
  if (!dout || !ids)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: embedding backward: null pointer");
  EmbLayout L;
  st = emb_layout(n, rows, cols, &L);
  if (st) return st;
  if (!workspace || workspace_bytes < L.total)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: embedding backward needs a %zu-byte workspace, got %zu",
                L.total, workspace_bytes);
  char* ws = static_cast<char*>(workspace);
  st = emb_sort_phase(ids, n, vocab_total, vocab_offset, rows, err_flag, ws, L, s);
  if (st) return st;
  return emb_sum_phase(dout, n, rows, cols, ws, L, dtable, nullptr, s);
}

size_t oxc_embedding_bwd_compact_workspace_size(int64_t n, int64_t rows, int64_t cols) {
  if (n <= 0 || rows <= 0 || cols <= 0) return 0;
  EmbLayout L;
  if (emb_layout(n, rows, cols, &L, 1, true) != OXC_OK) return 0;
  return L.total;
}

oxc_status oxc_embedding_bwd_compact_plan(const int64_t* ids, int64_t n, int64_t vocab_total,
                                          int64_t vocab_offset, int64_t rows, int64_t cols,
                                          int32_t* out_ids, int64_t* count, int32_t shards,
                                          int64_t* shard_counts, int32_t* err_flag,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  const char* fn = "embedding backward (compact)";
  oxc_status st = emb_check(fn, n, vocab_total, vocab_offset, rows, cols);
  if (st) return st;
  if (shards < 0 || (shard_counts && shards == 0))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: %d shards", fn, (int)shards);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!count) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null count", fn);
  if (n == 0 || rows == 0 || cols == 0) {
    cudaError_t e = cudaMemsetAsync(count, 0, sizeof(int64_t), s);
    if (e == cudaSuccess && shard_counts)
      e = cudaMemsetAsync(shard_counts, 0, (size_t)shards * sizeof(int64_t), s);
    return e == cudaSuccess ? OXC_OK : cuda_fail(e, "oxc_embedding_bwd_compact");
  }
  if (!ids || !out_ids)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  EmbLayout L;
  st = emb_layout(n, rows, cols, &L, 1, true);
  if (st) return st;
  if (!workspace || workspace_bytes < L.total)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: %s needs a %zu-byte workspace, got %zu", fn, L.total,
                workspace_bytes);
  char* ws = static_cast<char*>(workspace);
  st = emb_sort_phase(ids, n, vocab_total, vocab_offset, rows, err_flag, ws, L, s);
  if (st) return st;
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* present = reinterpret_cast<int32_t*>(ws + L.present);
  int32_t* slot = reinterpret_cast<int32_t*>(ws + L.slot);
  const unsigned gr = (unsigned)std::min<int64_t>((rows + 255) / 256, (int64_t)sm_count() * 8);
  emb_present_kernel<<<gr, 256, 0, s>>>(offsets, rows, present);
  st = check_launch("oxc_embedding_bwd_compact (present)");
  if (st) return st;
  size_t scan_bytes = L.scan_bytes;
  cudaError_t e = cub::DeviceScan::ExclusiveSum(ws + L.scan, scan_bytes, present, slot, (int)rows, s);
  if (e != cudaSuccess) return cuda_fail(e, "oxc_embedding_bwd_compact (scan)");
  const unsigned gm = std::max<unsigned>(gr, (unsigned)((shards + 255) / 256));
  emb_compact_meta_kernel<<<gm, 256, 0, s>>>(present, slot, rows, vocab_total, vocab_offset,
                                             shards, out_ids, count, shard_counts);
  return check_launch("oxc_embedding_bwd_compact (meta)");
}

oxc_status oxc_embedding_bwd_compact_sum(const float* dout, int64_t n, int64_t rows, int64_t cols,
                                         float* out_rows, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  const char* fn = "embedding backward (compact sums)";
  oxc_status st = emb_check(fn, n, rows, 0, rows, cols);
  if (st) return st;
  if (n == 0 || rows == 0 || cols == 0) return OXC_OK;
  if (!dout || !out_rows)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  EmbLayout L;
  st = emb_layout(n, rows, cols, &L, 1, true);
  if (st) return st;
  if (!workspace || workspace_bytes < L.total)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: %s needs a %zu-byte workspace, got %zu", fn, L.total,
                workspace_bytes);
  char* ws = static_cast<char*>(workspace);
  const int32_t* slot = reinterpret_cast<const int32_t*>(ws + L.slot);
  return emb_sum_phase(dout, n, rows, cols, ws, L, out_rows, slot, static_cast<cudaStream_t>(stream));
}

oxc_status oxc_embedding_bwd_compact(const float* dout, const int64_t* ids, int64_t n,
                                     int64_t vocab_total, int64_t vocab_offset, int64_t rows,
                                     int64_t cols, int32_t* out_ids, float* out_rows,
                                     int64_t* count, int32_t shards, int64_t* shard_counts,
                                     int32_t* err_flag, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  if (n > 0 && rows > 0 && cols > 0 && (!dout || !out_rows))
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: embedding backward (compact): null pointer");
  oxc_status st = oxc_embedding_bwd_compact_plan(ids, n, vocab_total, vocab_offset, rows, cols,
                                                 out_ids, count, shards, shard_counts, err_flag,
                                                 workspace, workspace_bytes, stream);
  if (st) return st;
  return oxc_embedding_bwd_compact_sum(dout, n, rows, cols, out_rows, workspace, workspace_bytes,
                                       stream);
}

size_t oxc_embedding_exchange_reduce_workspace_size(int32_t sources, int64_t shard_rows) {
  if (sources <= 0 || shard_rows <= 0) return 0;
  return align256((size_t)sources * (size_t)shard_rows * sizeof(int32_t));
}

oxc_status oxc_embedding_exchange_reduce(const int32_t* recv_ids, const float* recv_rows,
                                         const int64_t* src_offsets, int32_t sources,
                                         int64_t shard_lo, int64_t shard_rows, int64_t cols,
                                         float* dshard, int32_t* err_flag, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  const char* fn = "embedding gradient exchange";
  if (sources <= 0 || shard_rows < 0 || cols < 0 || shard_lo < 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: bad sizes", fn);
  if (shard_rows >= 0x7fffffff || cols > 0x7fffffff || (int64_t)sources * shard_rows >= 0x7fffffff)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: %s: sizes beyond 2^31", fn);
  if (shard_rows == 0 || cols == 0) return OXC_OK;
  if (!src_offsets || !dshard || !recv_ids || !recv_rows)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  const size_t need = oxc_embedding_exchange_reduce_workspace_size(sources, shard_rows);
  if (!workspace || workspace_bytes < need)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: %s needs a %zu-byte workspace, got %zu", fn, need,
                workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* map = static_cast<int32_t*>(workspace);
  cudaError_t e = cudaMemsetAsync(map, 0xff, (size_t)sources * shard_rows * sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "oxc_embedding_exchange_reduce");
  const unsigned gmap = (unsigned)sm_count() * 4;
  emb_exchange_map_kernel<<<gmap, 256, 0, s>>>(recv_ids, src_offsets, sources, shard_lo,
                                               shard_rows, map, err_flag);
  oxc_status st = check_launch("oxc_embedding_exchange_reduce (map)");
  if (st) return st;
  const bool v4 = cols % 4 == 0 && aligned16(recv_rows) && aligned16(dshard);
  const int64_t per = v4 ? cols / 4 : cols;
  const unsigned chunks = (unsigned)std::min<int64_t>(65535, (per + 127) / 128);
  const dim3 grid((unsigned)std::min<int64_t>(shard_rows, (int64_t)sm_count() * 32), chunks);
  if (v4)
    emb_exchange_reduce_kernel<4><<<grid, 128, 0, s>>>(recv_rows, map, sources, shard_rows,
                                                       (int)cols, dshard);
  else
    emb_exchange_reduce_kernel<1><<<grid, 128, 0, s>>>(recv_rows, map, sources, shard_rows,
                                                       (int)cols, dshard);
  return check_launch("oxc_embedding_exchange_reduce");
}

oxc_status oxc_embedding_bwd_push(const float* dout, const int64_t* ids, int64_t n,
                                  int64_t vocab_total, int64_t cols, const oxc_emb_push* push,
                                  int32_t* err_flag, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  const char* fn = "embedding backward (push)";
  oxc_status st = emb_check(fn, n, vocab_total, 0, vocab_total, cols);
  if (st) return st;
  if (!push) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null push table", fn);
  if (n == 0 || vocab_total == 0 || cols == 0)
    return fail(OXC_ERR_NOT_IMPLEMENTED,
                "not implemented: %s: empty inputs (every rank must still signal its counts)", fn);
  if (!dout || !ids) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  EmbLayout L;
  st = emb_layout(n, vocab_total, cols, &L, 1, true);
  if (st) return st;
  if (!workspace || workspace_bytes < L.total)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: %s needs a %zu-byte workspace, got %zu", fn, L.total,
                workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const int64_t rows = vocab_total;
  st = emb_sort_phase(ids, n, vocab_total, 0, rows, err_flag, ws, L, s);
  if (st) return st;
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* present = reinterpret_cast<int32_t*>(ws + L.present);
  int32_t* slot = reinterpret_cast<int32_t*>(ws + L.slot);
  const int64_t positions = rows + OXC_PUSH_MAX_RANKS;
  const unsigned gr =
      (unsigned)std::min<int64_t>((positions + 255) / 256, (int64_t)sm_count() * 8);
  emb_push_present_kernel<<<gr, 256, 0, s>>>(offsets, rows, push, present);
  st = check_launch("oxc_embedding_bwd_push (present)");
  if (st) return st;
  size_t scan_bytes = L.scan_bytes;
  cudaError_t e =
      cub::DeviceScan::ExclusiveSum(ws + L.scan, scan_bytes, present, slot, (int)positions, s);
  if (e != cudaSuccess) return cuda_fail(e, "oxc_embedding_bwd_push (scan)");
  emb_push_meta_kernel<<<gr, 256, 0, s>>>(present, slot, rows, push, err_flag);
  st = check_launch("oxc_embedding_bwd_push (meta)");
  if (st) return st;
  // the compact rows are not kept locally: every row goes to its owner's region
  return emb_sum_phase(dout, n, rows, cols, ws, L, nullptr, slot, s, push, err_flag);
}

oxc_status oxc_embedding_exchange_reduce_regions(const int32_t* recv_ids, const float* recv_rows,
                                                 const int64_t* counts, int32_t sources,
                                                 int64_t cap, int64_t shard_lo,
                                                 int64_t shard_stride, int64_t shard_rows,
                                                 int64_t cols, float* dshard, int32_t* err_flag,
                                                 void* workspace, size_t workspace_bytes,
                                                 void* stream) {
  const char* fn = "embedding gradient exchange (regions)";
  if (sources <= 0 || cap < 0 || shard_rows < 0 || cols < 0 || shard_lo < 0 || shard_stride < 1)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: bad sizes", fn);
  if (shard_rows >= 0x7fffffff || cols > 0x7fffffff || (int64_t)sources * cap >= 0x7fffffff ||
      (int64_t)sources * shard_rows >= 0x7fffffff)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: %s: sizes beyond 2^31", fn);
  if (shard_rows == 0 || cols == 0) return OXC_OK;
  if (!counts || !dshard || (cap > 0 && (!recv_ids || !recv_rows)))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  const size_t need = oxc_embedding_exchange_reduce_workspace_size(sources, shard_rows);
  if (!workspace || workspace_bytes < need)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: %s needs a %zu-byte workspace, got %zu", fn, need,
                workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* map = static_cast<int32_t*>(workspace);
  cudaError_t e = cudaMemsetAsync(map, 0xff, (size_t)sources * shard_rows * sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "oxc_embedding_exchange_reduce_regions");
  if (cap > 0) {
    emb_region_map_kernel<<<(unsigned)sm_count() * 4, 256, 0, s>>>(
        recv_ids, counts, sources, cap, shard_lo, shard_stride, shard_rows, map, err_flag);
    oxc_status st = check_launch("oxc_embedding_exchange_reduce_regions (map)");
    if (st) return st;
  }
  const bool v4 = cols % 4 == 0 && (cap == 0 || aligned16(recv_rows)) && aligned16(dshard);
  const int64_t per = v4 ? cols / 4 : cols;
  const unsigned chunks = (unsigned)std::min<int64_t>(65535, (per + 127) / 128);
  const dim3 grid((unsigned)std::min<int64_t>(shard_rows, (int64_t)sm_count() * 32), chunks);
  if (v4)
    emb_exchange_reduce_kernel<4><<<grid, 128, 0, s>>>(recv_rows, map, sources, shard_rows,
                                                       (int)cols, dshard);
  else
    emb_exchange_reduce_kernel<1><<<grid, 128, 0, s>>>(recv_rows, map, sources, shard_rows,
                                                       (int)cols, dshard);
  return check_launch("oxc_embedding_exchange_reduce_regions");
}

oxc_status oxc_embedding_exchange_pull(const oxc_emb_pull* pull, int32_t sources, int64_t cap,
                                       int64_t shard_lo, int64_t shard_stride,
                                       int64_t shard_rows, int64_t cols, float* dshard,
                                       int32_t* err_flag, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  const char* fn = "embedding gradient exchange (pull)";
  if (sources <= 0 || sources > OXC_PUSH_MAX_RANKS || cap < 0 || shard_rows < 0 || cols < 0 ||
      shard_lo < 0 || shard_stride < 1)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: bad sizes", fn);
  if (shard_rows >= 0x7fffffff || cols > 0x7fffffff || (int64_t)sources * cap >= 0x7fffffff ||
      (int64_t)sources * shard_rows >= 0x7fffffff)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: %s: sizes beyond 2^31", fn);
  if (shard_rows == 0 || cols == 0) return OXC_OK;
  if (!pull || !dshard) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  const size_t need = oxc_embedding_exchange_reduce_workspace_size(sources, shard_rows);
  if (!workspace || workspace_bytes < need)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: %s needs a %zu-byte workspace, got %zu", fn, need,
                workspace_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* map = static_cast<int32_t*>(workspace);
  cudaError_t e = cudaMemsetAsync(map, 0xff, (size_t)sources * shard_rows * sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "oxc_embedding_exchange_pull");
  if (cap > 0) {
    emb_pull_map_kernel<<<(unsigned)sm_count() * 4, 256, 0, s>>>(
        pull, sources, cap, shard_lo, shard_stride, shard_rows, map, err_flag);
    oxc_status st = check_launch("oxc_embedding_exchange_pull (map)");
    if (st) return st;
  }
  // the regions are the callers' buffers at cols-float strides: float4 rows
  // when cols % 4 == 0 (the regions' bases are 256-byte aligned allocations
  // plus multiples of 16 bytes)
  const bool v4 = cols % 4 == 0 && aligned16(dshard);
  const int64_t per = v4 ? cols / 4 : cols;
  const unsigned chunks = (unsigned)std::min<int64_t>(65535, (per + 127) / 128);
  const dim3 grid((unsigned)std::min<int64_t>(shard_rows, (int64_t)sm_count() * 32), chunks);
  if (v4)
    emb_pull_reduce_kernel<4><<<grid, 128, 0, s>>>(pull, map, sources, shard_rows, (int)cols,
                                                   dshard);
  else
    emb_pull_reduce_kernel<1><<<grid, 128, 0, s>>>(pull, map, sources, shard_rows, (int)cols,
                                                   dshard);
  return check_launch("oxc_embedding_exchange_pull");
}

oxc_status oxc_index_select(const oxc_view* x, int64_t dim, const int64_t* ids, int64_t n,
                            float* out, int32_t* err_flag, void* stream) {
  const char* fn = "index_select";
  if (!x) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null view", fn);
  if (x->ndim < 0 || x->ndim > OXC_MAX_DIMS)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: %s: rank %d > %d", fn, x->ndim,
                OXC_MAX_DIMS);
  if (x->ndim == 0)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: dim %lld out of range for 0-D tensor",
                (long long)dim);
  const int nd = x->ndim;
  const int64_t d = dim < 0 ? dim + nd : dim;
  if (d < 0 || d >= nd)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: dim %lld out of range for %d-D tensor",
                (long long)dim, nd);
  if (n < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative id count", fn);
  int64_t total = 1, outer = 1, inner = 1;
  for (int i = 0; i < nd; ++i) {
    if (x->shape[i] < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: negative dim", fn);
    total *= i == d ? n : x->shape[i];
    if (i < d) outer *= x->shape[i];
    if (i > d) inner *= x->shape[i];
  }
  if (total == 0) return OXC_OK;
  const int64_t len = x->shape[d];
  if (!x->data || !ids || !out)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: %s: null pointer", fn);
  bool contiguous = true;
  for (int64_t i = nd - 1, expect = 1; i >= 0; --i) {
    if (x->shape[i] != 1 && x->strides[i] != expect) contiguous = false;
    expect *= x->shape[i];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t cap = (int64_t)sm_count() * 16;
  if (contiguous && inner >= 32) {
    const bool v4 = inner % 4 == 0 && aligned16(x->data) && aligned16(out);
    const int64_t per = v4 ? inner / 4 : inner;
    const int block = (int)std::min<int64_t>(256, std::max<int64_t>(32, ((per + 31) / 32) * 32));
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(outer * n, cap));
    if (v4)
      isel_rows_kernel<4><<<grid, block, 0, s>>>(x->data, ids, out, outer, len, n, inner, (int)d,
                                                 err_flag);
    else
      isel_rows_kernel<1><<<grid, block, 0, s>>>(x->data, ids, out, outer, len, n, inner, (int)d,
                                                 err_flag);
    return check_launch("oxc_index_select");
  }
  ISelGrid g;
  g.nd = nd;
  g.dim = (int)d;
  g.len = len;
  for (int i = 0; i < nd; ++i) {
    g.n[i] = i == d ? n : x->shape[i];
    g.st[i] = x->strides[i];
  }
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, cap * 4));
  isel_elem_kernel<<<grid, 256, 0, s>>>(x->data, ids, g, out, total, err_flag);
  return check_launch("oxc_index_select");
}

oxc_status oxc_gather_dim0(const oxc_view* x, const int64_t* ids, int64_t n, float* out,
                           int32_t* err_flag, void* stream) {
  if (x && x->ndim == 0)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: gather_dim0 requires at least a 1-D tensor");
  return oxc_index_select(x, 0, ids, n, out, err_flag, stream);
}

// [outer, len, inner] of `shape` around `dim`, or an error.
static oxc_status isel_geometry(const int64_t* shape, int32_t ndim, int64_t dim, int64_t* outer,
                                int64_t* len, int64_t* inner, int64_t* d_out) {
  if (!shape || ndim <= 0 || ndim > OXC_MAX_DIMS)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: index_select backward: rank %d",
                (int)ndim);
  const int64_t d = dim < 0 ? dim + ndim : dim;
  if (d < 0 || d >= ndim)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: dim %lld out of range for %d-D tensor",
                (long long)dim, (int)ndim);
  *outer = 1;
  *inner = 1;
  for (int i = 0; i < ndim; ++i) {
    if (shape[i] < 0)
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: index_select backward: negative dim");
    if (i < d) *outer *= shape[i];
    if (i > d) *inner *= shape[i];
  }
  *len = shape[d];
  *d_out = d;
  return OXC_OK;
}

size_t oxc_index_select_bwd_workspace_size(const int64_t* shape, int32_t ndim, int64_t dim,
                                           int64_t n) {
  int64_t outer, len, inner, d;
  if (isel_geometry(shape, ndim, dim, &outer, &len, &inner, &d) != OXC_OK) return 0;
  if (n <= 0 || len <= 0 || inner <= 0 || outer <= 0) return 0;
  EmbLayout L;
  if (emb_layout(n, len, inner, &L, inner >= 128 ? outer : 0) != OXC_OK) return 0;
  return L.total;
}

oxc_status oxc_index_select_bwd(const float* g, const int64_t* ids, int64_t n,
                                const int64_t* shape, int32_t ndim, int64_t dim, float* gx,
                                int32_t* err_flag, void* workspace, size_t workspace_bytes,
                                void* stream) {
  int64_t outer, len, inner, d;
  oxc_status st = isel_geometry(shape, ndim, dim, &outer, &len, &inner, &d);
  if (st) return st;
  if (n < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: index_select backward: negative id count");
  if (n > 0x7fffffff || len >= 0x7fffffff || inner > 0x7fffffff)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: index_select backward: sizes beyond 2^31");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t total = outer * len * inner;
  if (total == 0) return OXC_OK;
  if (!gx) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: index_select backward: null pointer");
  if (n == 0) {
    cudaError_t e = cudaMemsetAsync(gx, 0, (size_t)total * sizeof(float), s);
    return e == cudaSuccess ? OXC_OK : cuda_fail(e, "oxc_index_select_bwd");
  }
  if (!g || !ids)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: index_select backward: null pointer");
  const bool wide = inner >= 128;
  EmbLayout L;
  st = emb_layout(n, len, inner, &L, wide ? outer : 0);
  if (st) return st;
  if (!workspace || workspace_bytes < L.total)
    return fail(OXC_ERR_INVALID_ARGUMENT,
                "invalid argument: index_select backward needs a %zu-byte workspace, got %zu",
                L.total, workspace_bytes);
  char* ws = static_cast<char*>(workspace);
  int32_t* keys_in = reinterpret_cast<int32_t*>(ws + L.keys_in);
  int32_t* vals_in = reinterpret_cast<int32_t*>(ws + L.vals_in);
  int32_t* keys_out = reinterpret_cast<int32_t*>(ws + L.keys_out);
  int32_t* vals_out = reinterpret_cast<int32_t*>(ws + L.vals_out);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  float* parts = reinterpret_cast<float*>(ws + L.parts);
  const unsigned g1 = (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 8);
  emb_prepare_kernel<<<g1, 256, 0, s>>>(ids, n, len, 0, len, keys_in, vals_in, err_flag);
  st = check_launch("oxc_index_select_bwd (prepare)");
  if (st) return st;
  size_t cub_bytes = L.cub_bytes;
  cudaError_t e = cub::DeviceRadixSort::SortPairs(ws + L.cub, cub_bytes, keys_in, keys_out,
                                                  vals_in, vals_out, (int)n, 0, L.end_bit, s);
  if (e != cudaSuccess) return cuda_fail(e, "oxc_index_select_bwd (sort)");
  const unsigned g2 = (unsigned)std::min<int64_t>((n + 1 + 255) / 256, (int64_t)sm_count() * 8);
  emb_offsets_kernel<<<g2, 256, 0, s>>>(keys_out, n, len, offsets);
  st = check_launch("oxc_index_select_bwd (offsets)");
  if (st) return st;
  if (!wide) {
    const unsigned grid =
        (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 32));
    isel_bwd_narrow_kernel<<<grid, 256, 0, s>>>(g, vals_out, offsets, outer, len, n, inner, gx);
    return check_launch("oxc_index_select_bwd");
  }
  // wide slices: the embedding VJP's kernels, one z-slice per outer index
  const bool v4 = inner % 4 == 0 && aligned16(g) && aligned16(gx);
  const int64_t nblocks = (n + kSplitP - 1) / kSplitP;
  const unsigned zs = (unsigned)std::min<int64_t>(outer, 65535);
  const unsigned grows = (unsigned)std::min<int64_t>(len, std::max<int64_t>(1, (int64_t)sm_count() * 32 / zs));
  const int vpt = v4 ? 1 : 4, vw = v4 ? 4 : 1;
  const int64_t per_thread = (int64_t)vpt * vw;
  const int block = (int)std::min<int64_t>(
      kEmbChunkThreads, std::max<int64_t>(32, ((inner / per_thread + 31) / 32) * 32));
  const int chunks = (int)std::min<int64_t>(65535, (inner + block * per_thread - 1) / (block * per_thread));
  const dim3 gsplit(chunk_grid_size(nblocks, chunks), 1, zs), grow(chunk_grid_size(grows, chunks), 1, zs);
  if (v4) {
    emb_split_kernel<4, 1, kEmbChunkThreads><<<gsplit, block, 0, s>>>(
        g, keys_out, vals_out, offsets, n, len, (int)inner, parts, outer, chunks);
    launch_dependent(emb_rows_kernel<4, 1, kEmbChunkThreads, false>, grow, block, s, g, vals_out,
                     offsets, (const float*)parts, len, (int)inner, gx, n, outer,
                     (const int32_t*)nullptr, (const oxc_emb_push*)nullptr, (int32_t*)nullptr,
                     chunks);
  } else {
    emb_split_kernel<1, 4, kEmbChunkThreads><<<gsplit, block, 0, s>>>(
        g, keys_out, vals_out, offsets, n, len, (int)inner, parts, outer, chunks);
    launch_dependent(emb_rows_kernel<1, 4, kEmbChunkThreads, false>, grow, block, s, g, vals_out,
                     offsets, (const float*)parts, len, (int)inner, gx, n, outer,
                     (const int32_t*)nullptr, (const oxc_emb_push*)nullptr, (int32_t*)nullptr,
                     chunks);
  }
  return check_launch("oxc_index_select_bwd");
}

}  // extern "C"
