// rowvec.cuh -- register-resident row tiles for the row-wise kernels.
//
// A CTA owns one row (or, in the persistent VJP kernels, one row at a time)
// and each thread keeps VPT vectors of VW consecutive floats in registers:
// thread t holds elements [(i*blockDim + t)*VW, +VW) for i < VPT, so every
// warp-wide access is a contiguous, coalesced 512-byte (VW=4) transaction.
#pragma once

#include "common.cuh"

namespace oxc {

template <int VW>
__device__ __forceinline__ void load_vec(float (&d)[VW], const float* p, bool streaming) {
  if constexpr (VW == 4) {
    float4 t = streaming ? ld_stream(reinterpret_cast<const float4*>(p))
                         : ld_keep(reinterpret_cast<const float4*>(p));
    d[0] = t.x; d[1] = t.y; d[2] = t.z; d[3] = t.w;
  } else {
    d[0] = streaming ? ld_stream(p) : ld_keep(p);
  }
}

template <int VW>
__device__ __forceinline__ void store_vec(float* p, const float (&d)[VW]) {
  if constexpr (VW == 4) {
    st_stream(reinterpret_cast<float4*>(p), make_float4(d[0], d[1], d[2], d[3]));
  } else {
    st_stream(p, d[0]);
  }
}

// Launch geometry for a row of `cols` floats with vector width VW.
// VPT = the smallest of {1,2,4,8} (VW=4) or {1,...,32} (VW=1) whose thread
// count fits `first_limit`, else 1024 threads; rows of up to 32768 floats fit.
// `maxt` is the __launch_bounds__ bucket (256, 512 or 1024) of the kernel
// instantiation, so narrow launches are not register-capped for 1024 threads.
struct RowGeom {
  int vw = 1;
  int vpt = 1;
  int block = 32;
  int maxt = 1024;
  bool ok = false;  // false when the row does not fit in registers
};

inline RowGeom row_geom(int64_t cols, bool vec4, int first_limit = 256) {
  RowGeom g;
  g.vw = vec4 ? 4 : 1;
  const int64_t nvec = (cols + g.vw - 1) / g.vw;
  const int vpts[6] = {1, 2, 4, 8, 16, 32};
  const int nv = vec4 ? 4 : 6;
  for (int limit : {first_limit, 1024}) {
    for (int k = 0; k < nv; ++k) {
      const int v = vpts[k];
      int64_t threads = (nvec + v - 1) / v;
      threads = ((threads + 31) / 32) * 32;
      if (threads < 32) threads = 32;
      if (threads <= limit) {
        g.vpt = v;
        g.block = (int)threads;
        g.maxt = !vec4 ? 1024 : threads <= 256 ? 256 : threads <= 512 ? 512 : 1024;
        g.ok = true;
        return g;
      }
    }
  }
  return g;
}

// Geometry that favours depth per thread, for float4 rows: the largest VPT of
// {8, 4, 2, 1} that still gives the block at least `min_threads` threads
// (rows too narrow for that take VPT 1).  ok = false when the row needs more
// than 1024 threads.  On B200 the persistent LayerNorm(+GELU) forward ran
// 5-40% faster from 2048 to 16384 columns with 8 vectors per thread on 128-512
// threads than with wider blocks holding fewer vectors each.
inline RowGeom row_geom_deep(int64_t cols, int min_threads = 128) {
  RowGeom g;
  g.vw = 4;
  const int64_t nvec = (cols + 3) / 4;
  for (int v : {8, 4, 2, 1}) {
    int64_t threads = ((nvec + v - 1) / v + 31) / 32 * 32;
    if (threads < 32) threads = 32;
    if (threads >= min_threads || v == 1) {
      if (threads > 1024) return g;
      g.vpt = v;
      g.block = (int)threads;
      g.maxt = threads <= 256 ? 256 : threads <= 512 ? 512 : 1024;
      g.ok = true;
      return g;
    }
  }
  return g;
}

// Dispatch a templated launcher on (VW, VPT, MAXT).
#define OXC_DISPATCH_VPT4(geom, LAUNCH, MAXT)               \
  switch ((geom).vpt) {                                     \
    case 1: LAUNCH(4, 1, MAXT); break;                      \
    case 2: LAUNCH(4, 2, MAXT); break;                      \
    case 4: LAUNCH(4, 4, MAXT); break;                      \
    default: LAUNCH(4, 8, MAXT); break;                     \
  }
#define OXC_DISPATCH_ROW(geom, LAUNCH)                      \
  do {                                                      \
    if ((geom).vw == 4) {                                   \
      if ((geom).maxt == 256) {                             \
        OXC_DISPATCH_VPT4(geom, LAUNCH, 256)                \
      } else if ((geom).maxt == 512) {                      \
        OXC_DISPATCH_VPT4(geom, LAUNCH, 512)                \
      } else {                                              \
        OXC_DISPATCH_VPT4(geom, LAUNCH, 1024)               \
      }                                                     \
    } else {                                                \
      switch ((geom).vpt) {                                 \
        case 1: LAUNCH(1, 1, 1024); break;                  \
        case 2: LAUNCH(1, 2, 1024); break;                  \
        case 4: LAUNCH(1, 4, 1024); break;                  \
        case 8: LAUNCH(1, 8, 1024); break;                  \
        case 16: LAUNCH(1, 16, 1024); break;                \
        default: LAUNCH(1, 32, 1024); break;                \
      }                                                     \
    }                                                       \
  } while (0)

}  // namespace oxc
