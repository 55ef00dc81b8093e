// loader.cu -- the data path: dataset columns resident in HBM, batches built
// on the device, and staged host<->device copies.
//
// The reference's DataLoader (crates/oxi-bindings/src/data.rs:116-330,
// crates/oxi-data/src/batch.rs) builds every batch on CPU worker threads:
// index_select(0, batch indices) per column (batch.rs:411-425), then, for the
// image column, the augmentation pipeline (transform.rs:105-223: per-plane
// random crop, per-sample horizontal flip, per-channel normalize) seeded per
// batch.  Here the columns are uploaded once and stay in device memory; for
// each epoch the host computes the shuffled order and every random draw of
// every batch (the draws depend only on seeds and shapes, never on pixel
// values), and two launches materialise the whole epoch:
//   gather_rows_kernel   -- out_c[i] = column_c[order[i]] for the plain columns;
//   image_epoch_kernel   -- the image column gathered, cropped, flipped and
//                           normalised in one pass, one warp per output row.
// Batches are then views of the epoch buffers: no per-batch launch, no
// per-batch host->device traffic.
//
// Host-side helpers restate the reference's randomness exactly:
//   MT19937 (Matsumoto & Nishimura 1998; rng.rs:1-125) with NumPy's
//     masked-rejection bounded draws and 53-bit doubles rounded to f32;
//   the SplitMix64 finaliser (Steele, Lea & Flood 2014) for per-epoch seeds
//     (data.rs:43-55) and per-batch seeds (transform.rs:231-244);
//   FNV-1a over the batch's indices (batch.rs:394-404).
#include <limits.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"

namespace oxc {

// ---- host-side randomness ------------------------------------------------------

namespace {

class Mt19937 {
 public:
  explicit Mt19937(uint32_t seed) {
    s_[0] = seed;
    for (int i = 1; i < kN; ++i) s_[i] = 1812433253u * (s_[i - 1] ^ (s_[i - 1] >> 30)) + (uint32_t)i;
    pos_ = kN;
  }
  uint32_t next_u32() {
    if (pos_ >= kN) regenerate();
    uint32_t y = s_[pos_++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
  }
  // 53-bit double from two words (27 + 26 bits), rounded to f32.
  float random() {
    const double a = (double)(next_u32() >> 5);
    const double b = (double)(next_u32() >> 6);
    return (float)((a * 67108864.0 + b) / 9007199254740992.0);
  }
  // Uniform in [0, bound): the smallest all-ones mask covering bound - 1,
  // redrawn until the masked word is in range.
  uint64_t below(uint64_t bound) {
    const uint32_t hi = (uint32_t)(bound - 1);
    uint32_t mask = hi;
    mask |= mask >> 1;
    mask |= mask >> 2;
    mask |= mask >> 4;
    mask |= mask >> 8;
    mask |= mask >> 16;
    for (;;) {
      const uint32_t v = next_u32() & mask;
      if (v <= hi) return v;
    }
  }

 private:
  static constexpr int kN = 624;
  static constexpr int kM = 397;
  static uint32_t twist(uint32_t hi, uint32_t lo, uint32_t far) {
    const uint32_t y = (hi & 0x80000000u) | (lo & 0x7fffffffu);
    return far ^ (y >> 1) ^ ((0u - (y & 1u)) & 0x9908b0dfu);
  }
  // The recurrence over the state in place, in three index ranges so that no
  // index wraps inside a loop.
  void regenerate() {
    int i = 0;
    for (; i < kN - kM; ++i) s_[i] = twist(s_[i], s_[i + 1], s_[i + kM]);
    for (; i < kN - 1; ++i) s_[i] = twist(s_[i], s_[i + 1], s_[i + kM - kN]);
    s_[kN - 1] = twist(s_[kN - 1], s_[0], s_[kM - 1]);
    pos_ = 0;
  }
  uint32_t s_[kN];
  int pos_;
};

uint64_t splitmix_finish(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

uint64_t fnv1a_indices(const int64_t* idx, int64_t n) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t v = (uint64_t)idx[i];
    for (int b = 0; b < 8; ++b) {
      h ^= (v >> (8 * b)) & 0xffu;
      h *= 0x00000100000001b3ull;
    }
  }
  return h;
}

}  // namespace

// ---- device kernels -------------------------------------------------------------

struct GatherColumn {
  const unsigned char* src;
  unsigned char* dst;
  int64_t row_bytes;
  int32_t width;  // bytes per lane access: 16, 4 or 1
};
struct GatherArgs {
  GatherColumn col[OXC_MAX_GATHER_COLUMNS];
};

__device__ __forceinline__ void loader_record_bad(int32_t* flag, int64_t value, int64_t size) {
  if (flag && atomicCAS(flag, 0, 1) == 0) {
    flag[1] = (int32_t)(uint32_t)((uint64_t)value & 0xffffffffu);
    flag[2] = (int32_t)(uint32_t)((uint64_t)value >> 32);
    flag[3] = (int32_t)size;
  }
}

template <typename T>
__device__ __forceinline__ void copy_row_chunks(const unsigned char* s, unsigned char* d,
                                                int64_t chunks, int64_t first, int64_t step) {
  const T* sp = reinterpret_cast<const T*>(s);
  T* dp = reinterpret_cast<T*>(d);
  for (int64_t k = first; k < chunks; k += step) dp[k] = __ldg(sp + k);
}

// blockIdx.y = column.  A row of at least 32 lane-chunks is copied by one
// warp; shorter rows are packed several to a warp (32 / chunks rows, each on
// `chunks` lanes), so a 4-byte label column still moves 128 bytes per warp
// instruction.
__global__ void __launch_bounds__(256) gather_rows_kernel(GatherArgs args, const int64_t* __restrict__ idx,
                                                          int64_t nidx, int64_t nrows, int32_t* err) {
  const GatherColumn c = args.col[blockIdx.y];
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t chunks = c.row_bytes / c.width;
  if (chunks >= 32) {
    for (int64_t i = warp; i < nidx; i += nwarps) {
      const int64_t id = idx[i];
      if (id < 0 || id >= nrows) {
        if (lane == 0) loader_record_bad(err, id, nrows);
        continue;
      }
      const unsigned char* s = c.src + id * c.row_bytes;
      unsigned char* d = c.dst + i * c.row_bytes;
      if (c.width == 16)
        copy_row_chunks<int4>(s, d, chunks, lane, 32);
      else if (c.width == 4)
        copy_row_chunks<uint32_t>(s, d, chunks, lane, 32);
      else
        copy_row_chunks<unsigned char>(s, d, chunks, lane, 32);
    }
    return;
  }
  const int per_warp = 32 / (int)chunks;
  const int sub = lane / (int)chunks;
  const int64_t k = lane % chunks;
  if (sub >= per_warp) return;
  for (int64_t i = warp * per_warp + sub; i < nidx; i += nwarps * per_warp) {
    const int64_t id = idx[i];
    if (id < 0 || id >= nrows) {
      if (k == 0) loader_record_bad(err, id, nrows);
      continue;
    }
    const unsigned char* s = c.src + id * c.row_bytes;
    unsigned char* d = c.dst + i * c.row_bytes;
    if (c.width == 16)
      copy_row_chunks<int4>(s, d, chunks, k, chunks);
    else if (c.width == 4)
      copy_row_chunks<uint32_t>(s, d, chunks, k, chunks);
    else
      copy_row_chunks<unsigned char>(s, d, chunks, k, chunks);
  }
}

// Each warp takes two output planes at a time.  Output plane q, row r,
// column x reads source row r + row_offset, column col_base + col_step * x
// of its plane, where the plane sits at element src_offset of the virtual
// tensor column[order[0..nidx)] (rows of row_elems elements; a plane never
// spans two rows); then every normalize step in order:
// v = (v - mean[c]) * inv[c], each operation rounded.  A plane's source row,
// its bounds and its normalize constants are resolved once, for both planes
// together (their map -> order -> pixel chains overlap); rows then stream
// four at a time per plane, lanes across columns, so eight loads per lane
// are in flight.
constexpr int kMaxFusedNorm = 4;
constexpr int kPlanesPerWarp = 2;

// NORM_SLOTS: normalize steps held in registers (2: the common pipelines, 64
// registers without spills; 4: up to four steps).
template <int NORM_SLOTS>
__global__ void __launch_bounds__(256, 4) image_epoch_kernel(
    const float* __restrict__ src, int64_t row_elems, const int64_t* __restrict__ order, int64_t nidx,
    int64_t nrows, const oxc_plane_map* __restrict__ planes, int64_t nplanes, int in_h, int in_w,
    int out_h, int out_w, const float* __restrict__ norm, int nnorm, int channels,
    float* __restrict__ out, int32_t* err) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t plane_out = (int64_t)out_h * out_w;
  for (int64_t q0 = warp * kPlanesPerWarp; q0 < nplanes; q0 += nwarps * kPlanesPerWarp) {
    oxc_plane_map pm[kPlanesPerWarp];
    bool ok[kPlanesPerWarp];
#pragma unroll
    for (int j = 0; j < kPlanesPerWarp; ++j) {
      ok[j] = q0 + j < nplanes;
      if (ok[j]) pm[j] = planes[q0 + j];
    }
    int64_t ds[kPlanesPerWarp], off[kPlanesPerWarp], id[kPlanesPerWarp];
#pragma unroll
    for (int j = 0; j < kPlanesPerWarp; ++j) {
      id[j] = -1;
      if (!ok[j]) continue;
      ds[j] = pm[j].src_offset / row_elems;
      off[j] = pm[j].src_offset - ds[j] * row_elems;
      const int x_last = pm[j].col_base + pm[j].col_step * (out_w - 1);
      const bool geom_ok = pm[j].src_offset >= 0 && ds[j] < nidx &&
                           off[j] + (int64_t)in_h * in_w <= row_elems && pm[j].row_offset >= 0 &&
                           pm[j].row_offset + out_h <= in_h && pm[j].col_base >= 0 &&
                           pm[j].col_base < in_w && x_last >= 0 && x_last < in_w &&
                           pm[j].channel >= 0 && pm[j].channel < channels;
      if (geom_ok) id[j] = order[ds[j]];
      if (!geom_ok || id[j] < 0 || id[j] >= nrows) {
        if (lane == 0)
          loader_record_bad(err, geom_ok ? id[j] : pm[j].src_offset, geom_ok ? nrows : row_elems);
        ok[j] = false;
      }
    }
    float mean[kPlanesPerWarp][NORM_SLOTS], inv[kPlanesPerWarp][NORM_SLOTS];
    const float* sp[kPlanesPerWarp];
    float* dp[kPlanesPerWarp];
    int step[kPlanesPerWarp];
#pragma unroll
    for (int j = 0; j < kPlanesPerWarp; ++j) {
      const int c = ok[j] ? pm[j].channel : 0;
#pragma unroll
      for (int k = 0; k < NORM_SLOTS; ++k) {
        mean[j][k] = (ok[j] && k < nnorm) ? norm[(2 * k) * channels + c] : 0.0f;
        inv[j][k] = (ok[j] && k < nnorm) ? norm[(2 * k + 1) * channels + c] : 1.0f;
      }
      sp[j] = ok[j] ? src + id[j] * row_elems + off[j] + (int64_t)pm[j].row_offset * in_w + pm[j].col_base
                    : src;
      dp[j] = out + (q0 + j) * plane_out;
      step[j] = ok[j] ? pm[j].col_step : 0;
    }
    for (int x = lane; x < out_w; x += 32) {
      int r = 0;
      for (; r + 4 <= out_h; r += 4) {
        float v[kPlanesPerWarp][4];
#pragma unroll
        for (int j = 0; j < kPlanesPerWarp; ++j)
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (ok[j]) v[j][u] = __ldg(sp[j] + step[j] * x + (int64_t)(r + u) * in_w);
#pragma unroll
        for (int j = 0; j < kPlanesPerWarp; ++j) {
          if (!ok[j]) continue;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float w = v[j][u];
#pragma unroll
            for (int k = 0; k < NORM_SLOTS; ++k)
              if (k < nnorm) w = __fmul_rn(__fsub_rn(w, mean[j][k]), inv[j][k]);
            dp[j][(int64_t)(r + u) * out_w + x] = w;
          }
        }
      }
      for (; r < out_h; ++r) {
#pragma unroll
        for (int j = 0; j < kPlanesPerWarp; ++j) {
          if (!ok[j]) continue;
          float w = __ldg(sp[j] + step[j] * x + (int64_t)r * in_w);
#pragma unroll
          for (int k = 0; k < NORM_SLOTS; ++k)
            if (k < nnorm) w = __fmul_rn(__fsub_rn(w, mean[j][k]), inv[j][k]);
          dp[j][(int64_t)r * out_w + x] = w;
        }
      }
    }
  }
}

static unsigned loader_grid(int64_t warps_of_work) {
  const int64_t cap = (int64_t)sm_count() * 8 * 4;  // 8 CTAs of 256 per SM, 4 waves
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((warps_of_work + 7) / 8, cap));
}

// ---- staged host<->device copies ---------------------------------------------------

namespace {

constexpr size_t kStageBytes = 8u << 20;  // per slot; two slots alternate
std::mutex g_stage_mu;
unsigned char* g_stage[2] = {nullptr, nullptr};

oxc_status stage_init() {
  for (int i = 0; i < 2; ++i) {
    if (g_stage[i]) continue;
    void* p = nullptr;
    cudaError_t e = cudaHostAlloc(&p, kStageBytes, cudaHostAllocPortable);
    if (e != cudaSuccess) return cuda_fail(e, "staging buffer (cudaHostAlloc)");
    g_stage[i] = static_cast<unsigned char*>(p);
  }
  return OXC_OK;
}

// Waits for `ev` with a deadline (60 s): a copy that never completes returns
// OXC_ERR_TIMEOUT instead of blocking the caller for good.
oxc_status wait_event(cudaEvent_t ev, const char* what) {
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(60);
  for (;;) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return OXC_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, what);
    if (std::chrono::steady_clock::now() >= deadline)
      return fail(OXC_ERR_TIMEOUT, "timeout: %s did not complete within 60 s", what);
    std::this_thread::yield();
  }
}

// Host memcpy split over up to 4 threads for large pieces (one thread moves
// roughly 10 GB/s from pageable memory, below what the PCIe link takes).
void host_copy(void* dst, const void* src, size_t n) {
  const size_t kMin = 1u << 20;
  const int threads = n >= 4 * kMin ? 4 : 1;
  if (threads == 1) {
    memcpy(dst, src, n);
    return;
  }
  const size_t part = (n / threads + 63) & ~size_t(63);
  std::thread pool[3];
  for (int t = 1; t < threads; ++t) {
    const size_t lo = std::min(n, part * t), hi = std::min(n, part * (t + 1));
    pool[t - 1] = std::thread([=] { memcpy((unsigned char*)dst + lo, (const unsigned char*)src + lo, hi - lo); });
  }
  memcpy(dst, src, std::min(n, part));
  for (int t = 1; t < threads; ++t) pool[t - 1].join();
}

struct EventPair {
  cudaEvent_t ev[2] = {nullptr, nullptr};
  ~EventPair() {
    for (cudaEvent_t e : ev)
      if (e) cudaEventDestroy(e);
  }
  oxc_status init() {
    for (auto& e : ev) {
      cudaError_t err = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
      if (err != cudaSuccess) return cuda_fail(err, "cudaEventCreateWithFlags");
    }
    return OXC_OK;
  }
};

}  // namespace

}  // namespace oxc

using namespace oxc;

extern "C" {

oxc_status oxc_gather_rows(const oxc_gather_column* columns, int32_t ncols, const int64_t* idx,
                           int64_t nidx, int64_t nrows, int32_t* err_flag, void* stream) {
  if (ncols < 1 || ncols > OXC_MAX_GATHER_COLUMNS || !columns)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: gather of %d columns (1 to %d)", ncols,
                OXC_MAX_GATHER_COLUMNS);
  if (nidx < 0 || nrows < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: negative size");
  if (nidx == 0) return OXC_OK;
  if (!idx) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: null index pointer");
  GatherArgs args;
  memset(&args, 0, sizeof(args));
  for (int c = 0; c < ncols; ++c) {
    const oxc_gather_column& g = columns[c];
    if (g.row_bytes <= 0 || !g.src || !g.dst)
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: gather column %d (row_bytes %lld)", c,
                  (long long)g.row_bytes);
    int width = 1;
    if (g.row_bytes % 16 == 0 && aligned16(g.src) && aligned16(g.dst))
      width = 16;
    else if (g.row_bytes % 4 == 0 && ((uintptr_t)g.src & 3u) == 0 && ((uintptr_t)g.dst & 3u) == 0)
      width = 4;
    args.col[c] = GatherColumn{static_cast<const unsigned char*>(g.src), static_cast<unsigned char*>(g.dst),
                               g.row_bytes, width};
  }
  // warps of work: the widest column decides (short rows pack several per warp)
  int64_t warps = 1;
  for (int c = 0; c < ncols; ++c) {
    const int64_t chunks = args.col[c].row_bytes / args.col[c].width;
    warps = std::max<int64_t>(warps, chunks >= 32 ? nidx : (nidx + 32 / chunks - 1) / (32 / chunks));
  }
  dim3 grid(loader_grid(warps), (unsigned)ncols);
  gather_rows_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(args, idx, nidx, nrows, err_flag);
  return check_launch("oxc_gather_rows");
}

oxc_status oxc_image_epoch(const float* src, int64_t row_elems, const int64_t* order, int64_t nidx,
                           int64_t nrows, const oxc_plane_map* planes, int64_t nplanes, int32_t in_h,
                           int32_t in_w, int32_t out_h, int32_t out_w, const float* norm, int32_t nnorm,
                           int32_t channels, float* out, int32_t* err_flag, void* stream) {
  if (nplanes < 0 || nidx < 0 || nrows < 0 || row_elems <= 0 || in_h <= 0 || in_w <= 0 || out_h <= 0 ||
      out_w <= 0 || channels <= 0 || nnorm < 0 || out_h > in_h || out_w > in_w)
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: image epoch geometry");
  if (nplanes == 0) return OXC_OK;
  if (!src || !order || !planes || !out || (nnorm > 0 && !norm))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: image epoch: null pointer");
  if (nnorm > kMaxFusedNorm)
    return fail(OXC_ERR_NOT_IMPLEMENTED, "not implemented: more than %d normalize steps in one pipeline",
                kMaxFusedNorm);
  const dim3 grid(loader_grid((nplanes + kPlanesPerWarp - 1) / kPlanesPerWarp));
  auto kernel = nnorm <= 2 ? image_epoch_kernel<2> : image_epoch_kernel<kMaxFusedNorm>;
  kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src, row_elems, order, nidx, nrows, planes, nplanes, in_h, in_w, out_h, out_w, norm, nnorm, channels,
      out, err_flag);
  return check_launch("oxc_image_epoch");
}

uint64_t oxc_epoch_seed(uint64_t base, uint64_t epoch) {
  return splitmix_finish(base + epoch * kGolden);
}

uint64_t oxc_batch_seed(uint64_t epoch_seed, const int64_t* indices, int64_t n) {
  return splitmix_finish(epoch_seed ^ (fnv1a_indices(indices, n) * kGolden));
}

oxc_status oxc_permutation(uint32_t seed, int64_t n, int64_t* out) {
  if (n < 0 || n > 0xffffffffll) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: permutation of %lld",
                                             (long long)n);
  if (n == 0) return OXC_OK;
  if (!out) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: null output");
  for (int64_t i = 0; i < n; ++i) out[i] = i;
  Mt19937 rng(seed);
  for (int64_t i = n - 1; i >= 1; --i) std::swap(out[i], out[(int64_t)rng.below((uint64_t)i + 1)]);
  return OXC_OK;
}

oxc_status oxc_epoch_transform_plan(const int64_t* order, int64_t nidx, int64_t batch_size,
                                    uint64_t epoch_seed, const int32_t* kinds, const int64_t* args,
                                    const float* norm_params, int32_t nsteps, int32_t rank,
                                    const int64_t* row_shape, oxc_plane_map* planes, int64_t planes_cap,
                                    int64_t* result) {
  if (!result || !order || batch_size < 1 || nidx < 0 || nsteps < 0 || (nsteps > 0 && (!kinds || !args)))
    return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: transform plan");
  result[0] = result[1] = result[2] = 0;
  result[3] = -1;
  if (rank < 2) {
    result[3] = 0;
    return fail(OXC_ERR_SHAPE_MISMATCH, "shape mismatch: rank %d vs image batches need at least (h, w)", rank);
  }
  if (rank < 3 || rank > 4)
    return fail(OXC_ERR_NOT_IMPLEMENTED,
                "not implemented: device transforms take image columns of rank 3 or 4 (got rank %d)", rank);
  if (!row_shape) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: transform plan: null row shape");
  for (int d = 0; d < rank - 1; ++d)
    if (row_shape[d] <= 0 || row_shape[d] > (int64_t)INT32_MAX)
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: transform plan: row dim %d is %lld", d,
                  (long long)row_shape[d]);
  for (int s = 0; s < nsteps; ++s) {
    if (kinds[s] < OXC_TRANSFORM_CROP || kinds[s] > OXC_TRANSFORM_NORMALIZE)
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: transform kind %d", kinds[s]);
    if (kinds[s] == OXC_TRANSFORM_NORMALIZE && (args[s] < 1 || !norm_params))
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: normalize step %d without parameters", s);
    if (kinds[s] == OXC_TRANSFORM_CROP && args[s] < 0)
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: crop size %lld", (long long)args[s]);
  }
  if (!planes && nidx > 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: null plane buffer");
  const int64_t h0 = row_shape[rank - 3], w0 = row_shape[rank - 2];
  int64_t row_elems = 1;
  for (int d = 0; d < rank - 1; ++d) row_elems *= row_shape[d];
  struct StepDraws {
    std::vector<int32_t> a, b;
  };
  std::vector<StepDraws> draws(nsteps);
  int64_t filled = 0;
  int64_t out_h = h0, out_w = w0;
  result[1] = h0;
  result[2] = w0;
  for (int64_t start = 0, k = 0; start < nidx; start += batch_size, ++k) {
    const int64_t bsz = std::min(batch_size, nidx - start);
    // Geometry of the batch tensor (bsz, *row_shape): rank 4 -> samples =
    // bsz, channels = row_shape[0]; rank 3 -> one sample of bsz channels.
    const int64_t samples = rank == 4 ? bsz : 1;
    const int64_t channels = rank == 4 ? row_shape[0] : bsz;
    const int64_t nplanes = samples * channels;
    if (filled + nplanes > planes_cap)
      return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: plane buffer holds %lld planes",
                  (long long)planes_cap);
    Mt19937 rng((uint32_t)([&] {
      const uint64_t s = oxc_batch_seed(epoch_seed, order + start, bsz);
      return s ^ (s >> 32);
    }()));
    int64_t h = h0, w = w0;
    const float* np = norm_params;
    std::vector<int64_t> hs(nsteps), ws(nsteps);
    for (int s = 0; s < nsteps; ++s) {
      hs[s] = h;
      ws[s] = w;
      draws[s].a.assign(nplanes, 0);
      draws[s].b.assign(nplanes, 0);
      if (kinds[s] == OXC_TRANSFORM_CROP) {
        const int64_t size = args[s];
        if (size == 0 || size > h || size > w) {
          result[3] = k;
          return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: crop size %lld exceeds image %lldx%lld",
                      (long long)size, (long long)h, (long long)w);
        }
        for (int64_t p = 0; p < nplanes; ++p) {
          draws[s].a[p] = (int32_t)rng.below((uint64_t)(h - size + 1));
          draws[s].b[p] = (int32_t)rng.below((uint64_t)(w - size + 1));
        }
        h = w = size;
      } else if (kinds[s] == OXC_TRANSFORM_FLIP) {
        // The reference draws one coin per sample, at its first plane, and
        // keeps that plane unflipped when the coin is >= 0.5; every other
        // plane of the sample is reversed unconditionally
        // (transform.rs:148-153).
        for (int64_t p = 0; p < nplanes; ++p)
          draws[s].a[p] = (p % channels != 0) ? 1 : (rng.random() >= 0.5f ? 0 : 1);
      } else if (kinds[s] == OXC_TRANSFORM_NORMALIZE) {
        const int64_t len = args[s];
        if (len != channels) {
          result[3] = k;
          return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: normalize expects %lld channels, got mean %lld / std %lld",
                      (long long)channels, (long long)len, (long long)len);
        }
        for (int64_t c = 0; c < len; ++c)
          if (!(np[len + c] > 0.0f)) {
            result[3] = k;
            return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: normalize std must be > 0");
          }
        np += 2 * len;
      } else {
        return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: transform kind %d", kinds[s]);
      }
    }
    out_h = h;
    out_w = w;
    // Compose the spatial steps from the last to the first: the source
    // column of output column x is col_step * x + col_base, its row r + row_offset.
    for (int64_t p = 0; p < nplanes; ++p) {
      int32_t step = 1, base = 0, top = 0;
      for (int s = nsteps - 1; s >= 0; --s) {
        if (kinds[s] == OXC_TRANSFORM_CROP) {
          top += draws[s].a[p];
          base += draws[s].b[p];
        } else if (kinds[s] == OXC_TRANSFORM_FLIP && draws[s].a[p]) {
          step = -step;
          base = (int32_t)ws[s] - 1 - base;
        }
      }
      oxc_plane_map& m = planes[filled + p];
      m.src_offset = start * row_elems + p * h0 * w0;
      m.row_offset = top;
      m.col_base = base;
      m.col_step = step;
      m.channel = (int32_t)(p % channels);
    }
    filled += nplanes;
    result[0] = filled;
    result[1] = out_h;
    result[2] = out_w;
  }
  return OXC_OK;
}

oxc_status oxc_upload(void* dst_device, const void* src_host, int64_t bytes, void* stream) {
  if (bytes < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: negative size");
  if (bytes == 0) return OXC_OK;
  if (!dst_device || !src_host) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: null pointer");
  std::lock_guard<std::mutex> lock(g_stage_mu);
  oxc_status st = stage_init();
  if (st != OXC_OK) return st;
  EventPair ev;
  if ((st = ev.init()) != OXC_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bool used[2] = {false, false};
  for (int64_t off = 0, piece = 0; off < bytes; off += (int64_t)kStageBytes, ++piece) {
    const int slot = (int)(piece & 1);
    const size_t n = (size_t)std::min<int64_t>((int64_t)kStageBytes, bytes - off);
    if (used[slot] && (st = wait_event(ev.ev[slot], "oxc_upload copy")) != OXC_OK) return st;
    host_copy(g_stage[slot], static_cast<const unsigned char*>(src_host) + off, n);
    cudaError_t e = cudaMemcpyAsync(static_cast<unsigned char*>(dst_device) + off, g_stage[slot], n,
                                    cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaEventRecord(ev.ev[slot], s);
    if (e != cudaSuccess) return cuda_fail(e, "oxc_upload");
    used[slot] = true;
  }
  for (int slot = 0; slot < 2; ++slot)
    if (used[slot] && (st = wait_event(ev.ev[slot], "oxc_upload copy")) != OXC_OK) return st;
  return OXC_OK;
}

oxc_status oxc_download(void* dst_host, const void* src_device, int64_t bytes, void* stream) {
  if (bytes < 0) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: negative size");
  if (bytes == 0) return OXC_OK;
  if (!dst_host || !src_device) return fail(OXC_ERR_INVALID_ARGUMENT, "invalid argument: null pointer");
  std::lock_guard<std::mutex> lock(g_stage_mu);
  oxc_status st = stage_init();
  if (st != OXC_OK) return st;
  EventPair ev;
  if ((st = ev.init()) != OXC_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t pieces = (bytes + (int64_t)kStageBytes - 1) / (int64_t)kStageBytes;
  auto issue = [&](int64_t piece) -> oxc_status {
    const int slot = (int)(piece & 1);
    const int64_t off = piece * (int64_t)kStageBytes;
    const size_t n = (size_t)std::min<int64_t>((int64_t)kStageBytes, bytes - off);
    cudaError_t e = cudaMemcpyAsync(g_stage[slot], static_cast<const unsigned char*>(src_device) + off, n,
                                    cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaEventRecord(ev.ev[slot], s);
    return e == cudaSuccess ? OXC_OK : cuda_fail(e, "oxc_download");
  };
  if ((st = issue(0)) != OXC_OK) return st;
  for (int64_t piece = 0; piece < pieces; ++piece) {
    const int slot = (int)(piece & 1);
    if ((st = wait_event(ev.ev[slot], "oxc_download copy")) != OXC_OK) return st;
    // the next piece lands in the other slot while this one is copied out
    if (piece + 1 < pieces && (st = issue(piece + 1)) != OXC_OK) return st;
    const int64_t off = piece * (int64_t)kStageBytes;
    host_copy(static_cast<unsigned char*>(dst_host) + off, g_stage[slot],
              (size_t)std::min<int64_t>((int64_t)kStageBytes, bytes - off));
  }
  return OXC_OK;
}

}  // extern "C"
