/*
 * oxiref.c -- CPU ORACLE (test infrastructure only).
 *
 * A plain-C restatement of the arithmetic of oxitorch's CPU tensor engine
 * (crates/oxi-tensor) for the memory-bound layer path.  It exists so the
 * tests and the CPU-baseline leg of bench.py can check the CUDA library
 * against the reference's algorithm; nothing in the product links it.
 *
 * Fidelity rules (why this file is compiled with -O2 -ffp-contract=off
 * -fno-fast-math against glibc libm):
 *   - Rust never contracts a*b+c into an FMA, so neither may this file.
 *   - Rust's f32::{exp,ln,log2,log10,sin,cos,tanh,powf} lower to the
 *     platform libm's expf/logf/... ; sqrt/floor/ceil are exact IEEE ops.
 *   - Every reduction is a sequential f32 fold in element order, exactly
 *     like ReduceKind::reduce_strip (crates/oxi-tensor/src/ops.rs:246-285).
 *
 * Parity status: the Rust reference cannot be built here (no cargo), so this
 * restatement is pinned against the known answers held by the reference's
 * own unit and Python tests (tests/golden/reference_kats.json), not against
 * a run of the reference binary.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define OXR_API __attribute__((visibility("default")))

/* ---- unary registry: order of F32_UNARY_OPS (ops.rs:125-202) ---------- */
enum {
  U_NEG = 0, U_ABS, U_SQRT, U_RSQRT, U_EXP, U_LOG, U_LOG2, U_LOG10, U_SIN,
  U_COS, U_TANH, U_RELU, U_SIGMOID, U_FLOOR, U_CEIL, U_ROUND, U_SIGN,
  U_SQUARE, U_RECIPROCAL, U_COUNT
};

/* Rust f32::max / f32::min: a NaN argument yields the other argument. */
static inline float rust_max(float a, float b) {
  if (isnan(a)) return b;
  if (isnan(b)) return a;
  return a > b ? a : b;
}
static inline float rust_min(float a, float b) {
  if (isnan(a)) return b;
  if (isnan(b)) return a;
  return a < b ? a : b;
}

/* Rust f32::signum: 1.0 for +0.0 and positives, -1.0 for -0.0 and
 * negatives, NaN for NaN (it never returns 0). */
static inline float rust_signum(float a) {
  if (isnan(a)) return a;
  return signbit(a) ? -1.0f : 1.0f;
}

static inline float unary_one(int op, float a) {
  switch (op) {
    case U_NEG: return -a;                                  /* ops.rs:128 */
    case U_ABS: return fabsf(a);                            /* ops.rs:132 */
    case U_SQRT: return sqrtf(a);                           /* ops.rs:136 */
    case U_RSQRT: return 1.0f / sqrtf(a);                   /* ops.rs:140 */
    case U_EXP: return expf(a);                             /* ops.rs:144 */
    case U_LOG: return logf(a);                             /* ops.rs:148 */
    case U_LOG2: return log2f(a);                           /* ops.rs:152 */
    case U_LOG10: return log10f(a);                         /* ops.rs:156 */
    case U_SIN: return sinf(a);                             /* ops.rs:160 */
    case U_COS: return cosf(a);                             /* ops.rs:164 */
    case U_TANH: return tanhf(a);                           /* ops.rs:168 */
    case U_RELU: return rust_max(a, 0.0f);                  /* ops.rs:172 */
    case U_SIGMOID: return 1.0f / (1.0f + expf(-a));        /* ops.rs:176 */
    case U_FLOOR: return floorf(a);                         /* ops.rs:180 */
    case U_CEIL: return ceilf(a);                           /* ops.rs:184 */
    case U_ROUND: return roundf(a);                         /* ops.rs:188: half away from zero */
    case U_SIGN: return rust_signum(a);                     /* ops.rs:192 */
    case U_SQUARE: return a * a;                            /* ops.rs:196 */
    case U_RECIPROCAL: return 1.0f / a;                     /* ops.rs:200 */
  }
  return NAN;
}

OXR_API int oxr_unary(int op, const float* in, float* out, int64_t n) {
  if (op < 0 || op >= U_COUNT) return 1;
  for (int64_t i = 0; i < n; ++i) out[i] = unary_one(op, in[i]);
  return 0;
}

/* ---- binary registry: order of F32_BINARY_OPS (ops.rs:55-91) ---------- */
enum { B_ADD = 0, B_SUB, B_MUL, B_DIV, B_POW, B_MIN, B_MAX, B_COUNT };

OXR_API int oxr_binary(int op, const float* a, const float* b, float* out, int64_t n) {
  if (op < 0 || op >= B_COUNT) return 1;
  for (int64_t i = 0; i < n; ++i) {
    float x = a[i], y = b[i], r;
    switch (op) {
      case B_ADD: r = x + y; break;
      case B_SUB: r = x - y; break;
      case B_MUL: r = x * y; break;
      case B_DIV: r = x / y; break;
      case B_POW: r = powf(x, y); break;
      case B_MIN: r = rust_min(x, y); break;
      default: r = rust_max(x, y); break;
    }
    out[i] = r;
  }
  return 0;
}

/* ---- comparison registry: order of F32_CMP_OPS (ops.rs:96-121) -------- */
OXR_API int oxr_cmp(int op, const float* a, const float* b, float* out, int64_t n) {
  if (op < 0 || op > 5) return 1;
  for (int64_t i = 0; i < n; ++i) {
    float x = a[i], y = b[i];
    int r;
    switch (op) {
      case 0: r = x == y; break;
      case 1: r = x != y; break;
      case 2: r = x < y; break;
      case 3: r = x <= y; break;
      case 4: r = x > y; break;
      default: r = x >= y; break;
    }
    out[i] = r ? 1.0f : 0.0f; /* bool -> Elem::from (lib.rs:302) */
  }
  return 0;
}

/* ---- reductions: ReduceKind order (ops.rs:224-239) --------------------- */
enum { R_SUM = 0, R_MEAN, R_MAX, R_MIN, R_ARGMAX, R_ARGMIN, R_NORM };

/* One strip, read with element stride `es` (ops.rs:246-285).  Returns 0 on
 * success, 1 for min/max/arg* over an empty strip. */
static int reduce_one(int kind, const float* d, int64_t len, int64_t es, double* res) {
  if (len == 0) {
    if (kind == R_SUM || kind == R_MEAN || kind == R_NORM) { *res = 0.0; return 0; }
    return 1;
  }
  switch (kind) {
    case R_SUM: case R_MEAN: {
      float acc = -0.0f; /* std's float Sum folds from -0.0 */
      for (int64_t i = 0; i < len; ++i) acc = acc + d[i * es];
      if (kind == R_MEAN) acc = acc / (float)len;
      *res = (double)acc;
      return 0;
    }
    case R_MAX: {
      float acc = -INFINITY;
      for (int64_t i = 0; i < len; ++i) acc = rust_max(acc, d[i * es]);
      *res = (double)acc;
      return 0;
    }
    case R_MIN: {
      float acc = INFINITY;
      for (int64_t i = 0; i < len; ++i) acc = rust_min(acc, d[i * es]);
      *res = (double)acc;
      return 0;
    }
    case R_ARGMAX: case R_ARGMIN: {
      int64_t best = 0;
      float bv = d[0];
      for (int64_t i = 0; i < len; ++i) {
        float v = d[i * es];
        if (kind == R_ARGMAX ? (v > bv) : (v < bv)) { bv = v; best = i; }
      }
      *res = (double)best;
      return 0;
    }
    case R_NORM: {
      float acc = -0.0f;
      for (int64_t i = 0; i < len; ++i) { float v = d[i * es]; float sq = v * v; acc = acc + sq; }
      *res = (double)sqrtf(acc);
      return 0;
    }
  }
  return 2;
}

/* Reduces `strips` strips of `len` elements.  Strip s starts at
 * data + s_off[s] (element offsets precomputed by the caller from the
 * logical row-major grid, i.e. after Tensor::to_vec, lib.rs:537-558) and
 * walks with element stride `es`.  Results are written as f32, the
 * reference's carrier for every reduction output (lib.rs:568-575). */
OXR_API int oxr_reduce_strips(int kind, const float* data, const int64_t* s_off, int64_t strips,
                              int64_t len, int64_t es, float* out) {
  for (int64_t s = 0; s < strips; ++s) {
    double r;
    int rc = reduce_one(kind, data + s_off[s], len, es, &r);
    if (rc) return rc;
    out[s] = (float)r;
  }
  return 0;
}

/* The same strips folded in f64 and rounded once to f32 (sum, mean, norm
 * only): the reference's composition with exact-as-possible sums, used by the
 * tests to measure how much of a result is the reference's own left-to-right
 * f32 rounding. */
OXR_API int oxr_reduce_strips_f64acc(int kind, const float* data, const int64_t* s_off,
                                     int64_t strips, int64_t len, int64_t es, float* out) {
  if (kind != R_SUM && kind != R_MEAN && kind != R_NORM)
    return oxr_reduce_strips(kind, data, s_off, strips, len, es, out);
  for (int64_t s = 0; s < strips; ++s) {
    const float* d = data + s_off[s];
    double acc = 0.0;
    for (int64_t i = 0; i < len; ++i) {
      double v = (double)d[i * es];
      acc += kind == R_NORM ? (double)(float)(d[i * es] * d[i * es]) : v;
    }
    float r = (float)acc;
    if (kind == R_MEAN) r = len ? r / (float)len : 0.0f;
    if (kind == R_NORM) r = sqrtf(r);
    out[s] = len ? r : 0.0f;
  }
  return 0;
}

/* Whole-buffer sequential f32 sum and sum of squares (sum_all, norm over a
 * flattened tensor: lib.rs:582-604), plus exact-as-possible f64 versions
 * used as the accuracy yardstick for large reductions. */
OXR_API float oxr_sum_all_f32(const float* d, int64_t n) {
  float acc = -0.0f;
  for (int64_t i = 0; i < n; ++i) acc = acc + d[i];
  return acc;
}
OXR_API double oxr_sum_all_f64(const float* d, int64_t n) {
  /* Neumaier-compensated f64 sum: used only as the accuracy yardstick. */
  double s = 0.0, c = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    double v = (double)d[i];
    double t = s + v;
    if (fabs(s) >= fabs(v)) c += (s - t) + v; else c += (v - t) + s;
    s = t;
  }
  return s + c;
}
OXR_API double oxr_sumsq_all_f64(const float* d, int64_t n) {
  double s = 0.0, c = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    double v = (double)d[i] * (double)d[i];
    double t = s + v;
    if (fabs(s) >= fabs(v)) c += (s - t) + v; else c += (v - t) + s;
    s = t;
  }
  return s + c;
}

/* Column-wise f64 sum of |a*b| over rows (condition numbers of the column
 * reductions in the norm VJPs; used to scale absolute tolerances). */
OXR_API void oxr_colsum_abs_prod_f64(const float* a, const float* b, int64_t rows, int64_t cols,
                                     double* out) {
  for (int64_t j = 0; j < cols; ++j) out[j] = 0.0;
  for (int64_t i = 0; i < rows; ++i)
    for (int64_t j = 0; j < cols; ++j)
      out[j] += fabs((double)a[i * cols + j] * (b ? (double)b[i * cols + j] : 1.0));
}

/* ---- index_select / scatter_index_select ------------------------------ */

/* Tensor::index_select along dim of a contiguous [outer, len, inner] tensor
 * (lib.rs:665-703): validates every index first (negative ids wrap) and
 * returns the offending index position + 1 on failure. */
OXR_API int64_t oxr_index_select(const float* src, int64_t outer, int64_t len, int64_t inner,
                                 const int64_t* ids, int64_t n, float* out) {
  for (int64_t k = 0; k < n; ++k) {
    int64_t i = ids[k];
    int64_t idx = i < 0 ? len + i : i;
    if (idx < 0 || idx >= len) return k + 1;
  }
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t k = 0; k < n; ++k) {
      int64_t i = ids[k];
      int64_t idx = i < 0 ? len + i : i;
      memcpy(out + (o * n + k) * inner, src + (o * len + idx) * inner, (size_t)inner * sizeof(float));
    }
  return 0;
}

/* scatter_index_select (crates/oxi-autograd/src/ops.rs:741-769): zeros,
 * then data[dst] += g[src] in index-position order.  `ids` are already
 * resolved to [0, len). */
OXR_API void oxr_scatter_index_select(const float* g, int64_t outer, int64_t len, int64_t inner,
                                      const int64_t* ids, int64_t n, float* out) {
  for (int64_t e = 0; e < outer * len * inner; ++e) out[e] = 0.0f;
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t k = 0; k < n; ++k) {
      int64_t idx = ids[k];
      for (int64_t i = 0; i < inner; ++i) {
        int64_t src = (o * n + k) * inner + i;
        int64_t dst = (o * len + idx) * inner + i;
        out[dst] = out[dst] + g[src];
      }
    }
}
