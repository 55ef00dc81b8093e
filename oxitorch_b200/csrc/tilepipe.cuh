// tilepipe.cuh -- the tile pipeline shared by the SwiGLU kernels and the
// elementwise registry's transposed-operand path: a warp-specialised ring of
// bulk/TMA copies feeding consumer warps, for 2-D problems [tokens, features]
// whose outputs are row-major and whose inputs are row-major or column-major
// (a transposed view).  Included by one .cu file each; everything here is
// internal to the including translation unit.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "pipeline.cuh"

namespace oxc {

// A 2-D view: base pointer and strides (elements) of its two dims.
struct View2 {
  const float* p;
  int64_t sr, sc;  // strides in elements
};

// ---- tile pipeline: bulk/TMA copies into a shared-memory ring ----------------------------
//
// A persistent CTA (one per SM) owns strips of 32 tokens and walks each strip's
// features in tiles of kTF.  The last warp produces: for every tile it copies
// the gate, up and (VJP) dh tiles into one stage of a ring with asynchronous
// bulk copies whose completion a "full" mbarrier counts in bytes.  The kTCW
// other warps consume: each reads its share of the tile from shared memory into
// registers, releases the stage ("empty" mbarrier, one arrive per warp), then
// computes and streams its outputs to HBM.  Loads of later tiles stay in flight
// while the arithmetic runs, so the SM's memory pipe never waits on the
// consumers.
//
// Tile layouts in shared memory:
//  * row-major operands (up, dh, a row-major gate): [32 tokens][kTF + 8 floats],
//    one 1-D bulk copy per token row (the 8-float pad makes the row pitch 8
//    banks);
//  * a column-major (transposed) gate: one 2-D TMA box of 32 tokens x kTF
//    features from a tensor map over its storage [features][tokens], landing
//    as [kTF features][32 tokens] with the 128-byte swizzle (the 16-byte chunk
//    index within each 128-byte row is XORed with the row index mod 8).
// Consumer warp w covers token quad w % 8 and feature part w / 8 of kTParts:
// lane l handles token 4*(w % 8) + l % 4 and features part*kTF/kTParts + 8k +
// l / 4 (k = 0..kTK-1).  Both layouts are then read without bank conflicts (a
// padded row gives bank 8t + f mod 32; the swizzled tile gives bank
// 4((t/4) ^ (f % 8)) + t % 4), and each store instruction writes four full
// 32-byte sectors (8 consecutive features of 4 tokens).
constexpr int kTT = 32;                    // tokens per strip
constexpr int kTCW = 24;                   // consumer warps
constexpr int kTF = 192;                   // features per tile
constexpr int kStageFwd = 4, kStageBwd = 3;
constexpr int kTP = kTF + 8;               // padded row pitch (floats)
constexpr int kTParts = kTCW / 8;          // feature parts per tile
constexpr int kTK = kTF / kTParts / 8;     // elements per lane per tile
constexpr int kTileBytes = kTT * kTP * 4;  // one row-major operand slot
constexpr int kTThreads = (kTCW + 1) * 32;

// The swizzled gate tile needs no pad.  Stage sizes are multiples of 1 KiB, so
// every stage's gate slot keeps the 1 KiB alignment the swizzle pattern needs.
template <bool GT>
constexpr int kGateSlotBytes = GT ? kTT * kTF * 4 : kTileBytes;
template <int NSLOT, bool GT>
constexpr int kStageBytes = kGateSlotBytes<GT> + (NSLOT - 1) * kTileBytes;
constexpr int kStatFloats = 2 * kTParts * kTT * 4;  // forward row-statistics exchange

static_assert(kTCW % 8 == 0 && kTF % (8 * kTParts) == 0 && kTF % 32 == 0, "tile geometry");
static_assert(kTF <= 256, "TMA box dims are at most 256");
static_assert(kTileBytes % 1024 == 0 && (kTT * kTF * 4) % 1024 == 0, "1 KiB aligned slots");

template <int NSLOT, bool GT>
inline size_t tile_smem_bytes(int stages, bool stats) {
  return 1024 + (size_t)stages * kStageBytes<NSLOT, GT> + 2 * stages * sizeof(uint64_t) + 16 +
         (kTCW + 1) * sizeof(double) + (stats ? kStatFloats * sizeof(float) : 0);
}

template <int NSLOT, bool GT>
struct TileRing {
  unsigned char* buf;
  uint64_t* full;
  uint64_t* empty;
  int* abort;
  double* red;      // [kTCW + 1] VJP sum-of-squares combine
  float* stat;      // [2][kTParts][32][4] forward row statistics (when allocated)
  int stages;

  __device__ float* slot(int stage, int k) const {
    return reinterpret_cast<float*>(buf + (size_t)stage * kStageBytes<NSLOT, GT> +
                                    (k == 0 ? 0 : kGateSlotBytes<GT> + (k - 1) * kTileBytes));
  }
};

template <int NSLOT, bool GT>
__device__ __forceinline__ TileRing<NSLOT, GT> make_tile_ring(unsigned char* smem, int stages) {
  TileRing<NSLOT, GT> r;
  uintptr_t p = (reinterpret_cast<uintptr_t>(smem) + 1023) & ~uintptr_t(1023);
  r.buf = reinterpret_cast<unsigned char*>(p);
  p += (size_t)stages * kStageBytes<NSLOT, GT>;
  r.full = reinterpret_cast<uint64_t*>(p);
  r.empty = r.full + stages;
  r.abort = reinterpret_cast<int*>(r.empty + stages);
  r.red = reinterpret_cast<double*>(r.abort + 4);
  r.stat = reinterpret_cast<float*>(r.red + kTCW + 1);
  r.stages = stages;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&r.full[s], 1);
      mbar_init(&r.empty[s], kTCW);
    }
    *r.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  return r;
}

// 2-D tiled TMA load (no multicast): box at (x = token, y = feature).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Offset of (token t, feature f) in a gate slot, and the offset step per k
// (f += 8 keeps f % 8, so the swizzled offset just moves 8 rows).
template <bool GT>
__device__ __forceinline__ int gate_off(int t, int f) {
  return GT ? f * kTT + (((t >> 2) ^ (f & 7)) << 2) + (t & 3) : t * kTP + f;
}
template <bool GT>
constexpr int kGateStep = GT ? 8 * kTT : 8;

// Producer warp: fills the ring with tiles of the CTA's strips, in the order the
// consumers read them.  NSLOT = gate + the nrow_src row-major sources.
template <bool GT, int NSLOT>
__device__ void tile_producer(const TileRing<NSLOT, GT>& ring, const CUtensorMap* gmap, View2 g,
                              const float* const (&rows_src)[2], int nrow_src, int64_t R,
                              int64_t C) {
  const int lane = threadIdx.x & 31;
  const int64_t nstrips = (R + kTT - 1) / kTT;
  int64_t issued = 0;
  for (int64_t strip = blockIdx.x; strip < nstrips; strip += gridDim.x) {
    const int64_t r0 = strip * kTT;
    const int nt = (int)(R - r0 < kTT ? R - r0 : kTT);
    for (int64_t c0 = 0; c0 < C; c0 += kTF, ++issued) {
      const int stage = (int)(issued % ring.stages);
      const uint32_t round = (uint32_t)(issued / ring.stages);
      if (lane == 0 && round > 0 && !mbar_wait(&ring.empty[stage], (round - 1) & 1)) {
        record_kernel_error(OXC_KERR_PIPELINE_TIMEOUT);
        *(volatile int*)ring.abort = 1;
      }
      __syncwarp();
      if (*(volatile int*)ring.abort) goto drain;
      {
        const uint32_t row_bytes = (uint32_t)(C - c0 < kTF ? C - c0 : kTF) * 4u;
        const uint32_t gbytes = GT ? (uint32_t)(kTT * kTF * 4) : nt * row_bytes;
        if (lane == 0)
          mbar_arrive_expect_tx(&ring.full[stage], gbytes + nrow_src * nt * row_bytes);
        __syncwarp();
        if (GT) {
          if (lane == 0) tma_load_2d(ring.slot(stage, 0), gmap, (int)r0, (int)c0, &ring.full[stage]);
        } else if (lane < nt) {
          bulk_g2s(ring.slot(stage, 0) + lane * kTP, g.p + (r0 + lane) * g.sr + c0, row_bytes,
                   &ring.full[stage]);
        }
        if (lane < nt) {
          for (int k = 0; k < nrow_src; ++k)
            bulk_g2s(ring.slot(stage, 1 + k) + lane * kTP, rows_src[k] + (r0 + lane) * C + c0,
                     row_bytes, &ring.full[stage]);
        }
      }
    }
  }
drain:
  // leave only after every issued copy has landed (bounded)
  if (lane == 0) {
    for (int64_t i = issued > ring.stages ? issued - ring.stages : 0; i < issued; ++i) {
      const int stage = (int)(i % ring.stages);
      if (!mbar_wait(&ring.full[stage], (uint32_t)(i / ring.stages) & 1))
        record_kernel_error(OXC_KERR_PIPELINE_TIMEOUT);
    }
  }
  __syncwarp();
}

template <class Ring>
__device__ __forceinline__ bool tile_acquire(const Ring& ring, int64_t i) {
  if (*(volatile int*)ring.abort) return false;
  if (!mbar_wait(&ring.full[(int)(i % ring.stages)], (uint32_t)(i / ring.stages) & 1)) {
    record_kernel_error(OXC_KERR_PIPELINE_TIMEOUT);
    *(volatile int*)ring.abort = 1;
    return false;
  }
  return true;
}

template <class Ring>
__device__ __forceinline__ void tile_release(const Ring& ring, int64_t i) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&ring.empty[(int)(i % ring.stages)]);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the library
// links only the static CUDA runtime).
static inline PFN_cuTensorMapEncodeTiled_v12000 encode_tiled_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Tensor map over a column-major gate's storage [C features][R tokens] (token
// stride 1, feature stride g.sc elements), box 32 tokens x 128 features.
static inline bool gate_tensor_map(CUtensorMap* map, const View2& g, int64_t R, int64_t C) {
  auto fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)R, (cuuint64_t)C};
  const cuuint64_t strides[1] = {(cuuint64_t)g.sc * 4};
  const cuuint32_t box[2] = {kTT, kTF};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(g.p), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename K, typename... A>
static oxc_status launch_tile(K kernel, size_t smem, int64_t R, cudaStream_t s,
                              const char* what, int64_t* ctas_out, A... args) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return cuda_fail(e, what);
  const int64_t ctas = std::min<int64_t>((R + kTT - 1) / kTT, sm_count());
  if (ctas_out) *ctas_out = ctas;
  kernel<<<(unsigned)ctas, kTThreads, smem, s>>>(args...);
  return check_launch(what);
}

}  // namespace oxc
