// pipeline.cuh -- bulk-copy (TMA, cp.async.bulk) row pipeline for sm_100a.
//
// A persistent CTA owns a contiguous range of rows.  Warp NCW (the last warp)
// is the producer: one lane streams whole rows of each input from HBM into a
// ring of shared-memory stages with cp.async.bulk, completion tracked by a
// "full" mbarrier per stage (transaction bytes).  Warps 0..NCW-1 consume:
// they wait on the stage's full barrier, copy their slice into registers,
// release the stage through its "empty" mbarrier (one arrive per consumer
// warp) and compute while the producer refills it.  So several rows of every
// input are in flight per SM at any time, independent of how long the
// arithmetic on the current row takes.
//
// Every wait is bounded in time (%globaltimer).  A wait that runs out sets
// bit OXC_KERR_PIPELINE_TIMEOUT in the device error word, marks the CTA as
// aborted (later waits and copies are skipped, but every barrier of the
// consumer loop is still executed so no warp is left behind), and the
// producer finally waits, again bounded, for copies it has in flight.  The
// host reads the word with oxc_kernel_error().
#pragma once

#include "common.cuh"

namespace oxc {

// Device error word of this translation unit (each .cu that includes this
// header gets its own, registered with the library-wide reader list so
// oxc_kernel_error() sees all of them).
static __device__ unsigned int g_kernel_error = 0;

static cudaError_t read_tu_kernel_error(unsigned int* value, int clear) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_kernel_error, sizeof(unsigned int));
  if (e == cudaSuccess && clear && *value) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_kernel_error, &zero, sizeof(unsigned int));
  }
  return e;
}
static const int g_tu_kernel_error_registered = register_kernel_error_reader(&read_tu_kernel_error);

constexpr unsigned long long kWaitTimeoutNs = 4000000000ull;  // 4 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with `parity` to complete; false after kWaitTimeoutNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
  }
}

// One bulk copy global -> shared, completing `bytes` transactions on `bar`.
// src, dst 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Barrier over the consumer warps only (named barrier 1).
template <int NCW>
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
}

// Sum over the NCW consumer warps; every consumer thread gets the result.
// `scratch` holds >= NCW + 1 floats.  Fixed combination order.
template <int NCW>
__device__ __forceinline__ float consumer_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  consumer_sync<NCW>();
  if (lane == 0) scratch[warp] = v;
  consumer_sync<NCW>();
  float t = lane < NCW ? scratch[lane] : 0.0f;
  return warp_sum(t);
}

template <int NCW>
__device__ __forceinline__ float consumer_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  consumer_sync<NCW>();
  if (lane == 0) scratch[warp] = v;
  consumer_sync<NCW>();
  float t = lane < NCW ? scratch[lane] : -INFINITY;
  return warp_max(t);
}

// Sum over one consumer group of NWG warps (warps [g*NWG, (g+1)*NWG)),
// synchronised on named barrier `bar` (1 + g).  `scratch` holds >= NWG floats
// private to the group.  Fixed combination order.
template <int NWG>
__device__ __forceinline__ float group_sum(float v, float* scratch, int bar) {
  const int lane = threadIdx.x & 31, wig = (threadIdx.x >> 5) % NWG;
  v = warp_sum(v);
  asm volatile("bar.sync %0, %1;" ::"r"(bar), "n"(NWG * 32) : "memory");
  if (lane == 0) scratch[wig] = v;
  asm volatile("bar.sync %0, %1;" ::"r"(bar), "n"(NWG * 32) : "memory");
  const float t = lane < NWG ? scratch[lane] : 0.0f;
  return warp_sum(t);
}

// Barrier over all consumer threads (named barrier 15).
template <int NCONS_THREADS>
__device__ __forceinline__ void all_consumers_sync() {
  asm volatile("bar.sync 15, %0;" ::"n"(NCONS_THREADS) : "memory");
}

// Ring of `stages` stages, each holding one row of each of NIN inputs.
template <int NIN>
struct RowRing {
  float* buf;       // stages * NIN * cols floats
  uint64_t* full;   // [stages]
  uint64_t* empty;  // [stages]
  int* abort;       // CTA-wide abort flag
  int stages;
  int cols;

  __device__ float* row(int stage, int input) const {
    return buf + ((size_t)stage * NIN + input) * cols;
  }
};

// Shared-memory bytes for a ring of `stages` stages plus `extra_floats`
// floats of kernel-owned space after the 64-float reduction scratch.
inline size_t ring_smem_bytes(int nin, int64_t cols, int stages, int64_t extra_floats = 0) {
  return 128 /* align */ + (size_t)stages * nin * cols * sizeof(float) +
         2 * (size_t)stages * sizeof(uint64_t) + 16 + 64 * sizeof(float) +
         (size_t)extra_floats * sizeof(float);
}

// Carves the ring out of dynamic shared memory; `red` gets 64 floats for
// reductions followed by the kernel's extra floats.  Call from every thread;
// thread 0 initialises the barriers.  NCW = consumer warps that release each
// row (the warps of one consumer group).
template <int NIN, int NCW>
__device__ __forceinline__ RowRing<NIN> make_ring(unsigned char* smem, int stages, int cols,
                                                  float** red) {
  RowRing<NIN> r;
  uintptr_t p = (reinterpret_cast<uintptr_t>(smem) + 127) & ~uintptr_t(127);
  r.buf = reinterpret_cast<float*>(p);
  p += (size_t)stages * NIN * cols * sizeof(float);
  r.full = reinterpret_cast<uint64_t*>(p);
  r.empty = r.full + stages;
  r.abort = reinterpret_cast<int*>(r.empty + stages);
  *red = reinterpret_cast<float*>(r.abort + 4);
  r.stages = stages;
  r.cols = cols;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&r.full[s], 1);
      mbar_init(&r.empty[s], NCW);
    }
    *r.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  return r;
}

__device__ __forceinline__ void record_kernel_error(unsigned int bits) {
  atomicOr(&g_kernel_error, bits);
}

// Producer loop (one lane): streams rows [r0, r1) of the NIN inputs.
template <int NIN>
__device__ __forceinline__ void produce_rows(const RowRing<NIN>& ring,
                                             const float* const (&src)[NIN], int64_t r0,
                                             int64_t r1) {
  const uint32_t row_bytes = (uint32_t)ring.cols * sizeof(float);
  int64_t issued = 0;
  for (int64_t row = r0; row < r1; ++row, ++issued) {
    const int stage = (int)(issued % ring.stages);
    const uint32_t round = (uint32_t)(issued / ring.stages);
    if (round > 0 && !mbar_wait(&ring.empty[stage], (round - 1) & 1)) {
      record_kernel_error(OXC_KERR_PIPELINE_TIMEOUT);
      *(volatile int*)ring.abort = 1;
    }
    if (*(volatile int*)ring.abort) break;
    mbar_arrive_expect_tx(&ring.full[stage], row_bytes * NIN);
#pragma unroll
    for (int k = 0; k < NIN; ++k)
      bulk_g2s(ring.row(stage, k), src[k] + row * (int64_t)ring.cols, row_bytes,
               &ring.full[stage]);
  }
  // Leave only after every issued copy has landed (bounded).
  for (int64_t i = issued > ring.stages ? issued - ring.stages : 0; i < issued; ++i) {
    const int stage = (int)(i % ring.stages);
    if (!mbar_wait(&ring.full[stage], (uint32_t)(i / ring.stages) & 1))
      record_kernel_error(OXC_KERR_PIPELINE_TIMEOUT);
  }
}

// Consumer side: waits for row `i` (0-based within the CTA's range).
// Returns false if the CTA is aborting (data must not be read).
template <int NIN>
__device__ __forceinline__ bool consumer_acquire(const RowRing<NIN>& ring, int64_t i) {
  if (*(volatile int*)ring.abort) return false;
  const int stage = (int)(i % ring.stages);
  if (!mbar_wait(&ring.full[stage], (uint32_t)(i / ring.stages) & 1)) {
    record_kernel_error(OXC_KERR_PIPELINE_TIMEOUT);
    *(volatile int*)ring.abort = 1;
    return false;
  }
  return true;
}

// Called by every lane of a consumer warp once it has read row `i`.
template <int NIN>
__device__ __forceinline__ void consumer_release(const RowRing<NIN>& ring, int64_t i) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&ring.empty[(int)(i % ring.stages)]);
}

}  // namespace oxc
