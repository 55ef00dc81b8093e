/*
 * oxicuda.h -- C ABI of the B200 (sm_100a) backend for oxitorch's
 * memory-bound layer path.
 *
 * Every entry point is what oxitorch's Rust tensor crate (oxi-tensor) would
 * bind through `extern "C"` to run the named reference function on device
 * memory.  Conventions:
 *   - all tensors are float32 in device memory unless stated;
 *   - every call is asynchronous on `stream` (a cudaStream_t passed as
 *     void*; NULL = legacy default stream) and never allocates: scratch comes
 *     from a caller-provided workspace whose size is returned by the matching
 *     *_workspace_size function;
 *   - a call returns an oxc_status; on failure, oxc_last_error() gives the
 *     message (thread-local), worded like the reference's error messages;
 *   - no call panics, traps or aborts; device-side index faults are reported
 *     through an int32 error flag that the caller reads after the stream
 *     synchronises (oxc_check_error_flag).
 *
 * Reference citations are path:line within SirBlocky7747/oxitorch.
 */
#ifndef OXICUDA_H
#define OXICUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------
 * 1..5 map one-to-one onto OxitorchError (crates/oxi-core/src/lib.rs:186-208)
 * and from there onto Python exceptions (crates/oxi-bindings/src/error.rs:22-32):
 * 1,2 -> ValueError, 3 -> NotImplementedError, 4,5,6 -> RuntimeError.      */
typedef int32_t oxc_status;
#define OXC_OK 0
#define OXC_ERR_INVALID_ARGUMENT 1
#define OXC_ERR_SHAPE_MISMATCH 2
#define OXC_ERR_NOT_IMPLEMENTED 3
#define OXC_ERR_OUT_OF_BOUNDS 4
#define OXC_ERR_OTHER 5
#define OXC_ERR_TIMEOUT 6

#define OXC_MAX_DIMS 8

/* A strided view: the device counterpart of oxi-tensor's Tensor
 * {storage, offset, View{shape, strides}} (crates/oxi-tensor/src/lib.rs:24-58).
 * `data` points at element (0,...,0), i.e. the storage offset is applied;
 * strides are in elements and may be 0 (broadcast dims, layout.rs:97-114). */
typedef struct oxc_view {
  float* data;
  int32_t ndim;
  int64_t shape[OXC_MAX_DIMS];
  int64_t strides[OXC_MAX_DIMS];
} oxc_view;

/* Backward semantics of the fused norm VJPs.
 * OXC_GRAD_REF: the reference's graph, where `.apply("rsqrt")` is not in the
 *   differentiable whitelist (crates/oxi-bindings/src/lib.rs:682-697) and the
 *   rsqrt factor is a detached constant.
 * OXC_GRAD_EXACT: the full mathematical gradient (what torch computes). */
#define OXC_GRAD_REF 0
#define OXC_GRAD_EXACT 1

/* Activation fused after a layer norm. */
#define OXC_ACT_NONE 0
#define OXC_ACT_GELU_TANH 1 /* python/oxitorch/nn/functional.py:194-199 */

/* ---- library ---------------------------------------------------------- */
int32_t oxc_abi_version(void);
/* Message of the last failing call on this thread ("" if none). */
const char* oxc_last_error(void);
/* Number of visible CUDA devices; replaces the constant 1 of
 * crates/oxi-bindings/src/lib.rs:781-785. */
int32_t oxc_device_count(void);
/* Waits for `stream` with a deadline; OXC_ERR_TIMEOUT if it has not drained
 * after timeout_ms (negative = wait forever).  Host-side poll, never spins
 * on the device. */
oxc_status oxc_stream_sync(void* stream, int64_t timeout_ms);
/* Synchronises `stream` and reads a device int32 error flag written by a
 * kernel; returns OXC_ERR_OUT_OF_BOUNDS with the reference's message when it
 * holds a recorded bad index (flag[0] = 1, flag[1..2] = index value as two
 * int32 halves, flag[3] = dim size), and clears it. */
oxc_status oxc_check_error_flag(int32_t* flag_dev, void* stream, int64_t timeout_ms);

/* Device-side error bits recorded by kernels since the last clear (synchronous;
 * call after the stream has drained).  Bit 1: a bounded wait inside a
 * bulk-copy pipeline ran out (the kernel stopped early, its outputs are not
 * valid).  clear != 0 resets the bits. */
#define OXC_KERR_PIPELINE_TIMEOUT 1u
oxc_status oxc_kernel_error(uint32_t* bits, int32_t clear);

/* ---- optimizer step (crates/oxi-autograd/src/optim.rs) ------------------
 * Both update one flat f32 parameter in place, the per-element arithmetic in
 * the reference's order and rounding, so results are the reference's bits.
 * The caller owns the state buffers (zero-initialised before a parameter's
 * first step, as the reference's lazily created slots are) and skips
 * parameters that have no gradient.
 *
 * oxc_sgd_step: Sgd::step_param (optim.rs:104-138).  velocity [n] is used
 *   (and may be null otherwise) when momentum > 0; nesterov needs
 *   momentum > 0 (OXC_ERR_INVALID_ARGUMENT, the reference's ValueError).
 * oxc_adamw_step: AdamW::step_param (optim.rs:223-261): decoupled != 0 is
 *   AdamW (decay on the parameter), 0 classic Adam (decay added to the
 *   gradient).  step = the parameter's own step counter including this step
 *   (1 on its first step); the bias corrections 1 - beta^step use the C
 *   library's powf, like the reference's f32::powf.  m, v: [n]. */
oxc_status oxc_sgd_step(float* param, const float* grad, float* velocity, int64_t n, float lr,
                        float momentum, int32_t nesterov, void* stream);
oxc_status oxc_adamw_step(float* param, const float* grad, float* m, float* v, int64_t n,
                          float lr, float beta1, float beta2, float eps, float weight_decay,
                          int32_t decoupled, int64_t step, void* stream);
/* oxc_clip_grad_value: clip_grad_value_ (python/oxitorch/optim.py:266-272) on
 *   one gradient in place, np.clip(g, -clip_value, clip_value) with NumPy's
 *   NaN rules (a NaN element or bound gives NaN).  The caller applies the
 *   reference's "clip_value must be positive" check to its double value; a
 *   negative f32 bound is refused here with that message. */
oxc_status oxc_clip_grad_value(float* grad, int64_t n, float clip_value, void* stream);

/* ---- data path: dataset columns in device memory, batches built on device --
 * The reference's DataLoader (crates/oxi-bindings/src/data.rs:116-330) gathers
 * each batch on CPU worker threads (TensorBatchSource::get_batch,
 * crates/oxi-data/src/batch.rs:378-387 -> gather_columns :411-425) and runs the
 * augmentation pipeline on the image column (transform.rs:105-223).  Here the
 * columns stay on the device and a whole epoch is materialised by two
 * launches; the host supplies the order and the per-plane draws.
 *
 * oxc_gather_rows: for every column c, dst_c[i] = src_c[idx[i]] (rows of
 *   row_bytes bytes), i < nidx; idx is a device array.  Ids outside
 *   [0, nrows) are recorded in err_flag (int32[4], may be null) and skipped
 *   (read it with oxc_check_error_flag: gather_columns' OutOfBounds).
 * oxc_image_epoch: the image column gathered and transformed in one pass.
 *   Output plane q (out_h x out_w floats at out + q*out_h*out_w) reads, for
 *   row r and column x, element (r + row_offset, col_base + col_step*x) of
 *   the in_h x in_w plane starting at element src_offset of the virtual
 *   tensor src[order[0..nidx)] (rows of row_elems floats), then applies nnorm
 *   normalize steps in order, v = (v - mean[c]) * inv[c] with
 *   c = planes[q].channel; norm is a device array [nnorm][2][channels]
 *   (mean, then 1/std rounded to f32), at most 4 steps.  planes: device
 *   array from oxc_epoch_transform_plan; a plane whose map points outside
 *   its source plane, or whose order entry is outside [0, nrows), is
 *   recorded in err_flag and skipped.
 *
 * Host-side helpers (no device work):
 * oxc_epoch_seed: the per-epoch seed, SplitMix64 of base + epoch*golden
 *   (EpochSeeds::next, data.rs:43-55).
 * oxc_batch_seed: batch_seed(epoch_seed, FNV-1a of the batch's indices)
 *   (transform.rs:231-244, batch.rs:394-404).
 * oxc_permutation: MT19937(seed) Fisher-Yates order of 0..n, NumPy's
 *   RandomState.permutation stream (rng.rs:84-95).
 * oxc_epoch_transform_plan: for the batches order[k*batch_size ..] of an
 *   epoch, draws every batch's random crops and flips from
 *   MT19937(batch_rng(oxc_batch_seed(epoch_seed, batch))) in the reference's
 *   order and composes the steps into one oxc_plane_map per output plane.
 *   kinds[s] is OXC_TRANSFORM_*; args[s] the crop size or the normalize
 *   channel count; norm_params packs each normalize step's mean[] then
 *   std[].  rank is the column's rank (3 or 4), row_shape its dims after
 *   dim 0.  result[4] = {planes written, out_h, out_w, failing batch or -1}:
 *   on a batch whose transform the reference rejects, the planes of the
 *   batches before it are written and the reference's message returned. */
#define OXC_MAX_GATHER_COLUMNS 8
#define OXC_TRANSFORM_CROP 0      /* NativeTransform::RandomCrop(size) */
#define OXC_TRANSFORM_FLIP 1      /* NativeTransform::RandomHorizontalFlip */
#define OXC_TRANSFORM_NORMALIZE 2 /* NativeTransform::Normalize(mean, std) */
typedef struct oxc_gather_column {
  const void* src;
  void* dst;
  int64_t row_bytes;
} oxc_gather_column;
typedef struct oxc_plane_map {
  int64_t src_offset;
  int32_t row_offset;
  int32_t col_base;
  int32_t col_step; /* +1, or -1 for a mirrored plane */
  int32_t channel;
} oxc_plane_map;
oxc_status oxc_gather_rows(const oxc_gather_column* columns, int32_t ncols, const int64_t* idx,
                           int64_t nidx, int64_t nrows, int32_t* err_flag, void* stream);
oxc_status oxc_image_epoch(const float* src, int64_t row_elems, const int64_t* order, int64_t nidx,
                           int64_t nrows, const oxc_plane_map* planes, int64_t nplanes, int32_t in_h,
                           int32_t in_w, int32_t out_h, int32_t out_w, const float* norm, int32_t nnorm,
                           int32_t channels, float* out, int32_t* err_flag, void* stream);
uint64_t oxc_epoch_seed(uint64_t base, uint64_t epoch);
uint64_t oxc_batch_seed(uint64_t epoch_seed, const int64_t* indices, int64_t n);
oxc_status oxc_permutation(uint32_t seed, int64_t n, int64_t* out);
oxc_status oxc_epoch_transform_plan(const int64_t* order, int64_t nidx, int64_t batch_size,
                                    uint64_t epoch_seed, const int32_t* kinds, const int64_t* args,
                                    const float* norm_params, int32_t nsteps, int32_t rank,
                                    const int64_t* row_shape, oxc_plane_map* planes, int64_t planes_cap,
                                    int64_t* result);

/* Host <-> device copies through a pinned two-slot staging ring, the host
 * copy of one slot overlapping the DMA of the other; they return once the
 * bytes have arrived; the two 8 MiB pinned slots are allocated on first use
 * (the reference's from_numpy / Tensor::numpy copies,
 * crates/oxi-bindings/src/lib.rs:769-780, 382-391).  Ordered on `stream`. */
oxc_status oxc_upload(void* dst_device, const void* src_host, int64_t bytes, void* stream);
oxc_status oxc_download(void* dst_host, const void* src_device, int64_t bytes, void* stream);

/* ---- registry ids: the order of the reference registry tables ---------
 * binary: add,sub,mul,div,pow,min,max          (crates/oxi-tensor/src/ops.rs:55-91)
 * cmp:    eq,ne,lt,le,gt,ge                    (ops.rs:96-121)
 * unary:  neg,abs,sqrt,rsqrt,exp,log,log2,log10,sin,cos,tanh,relu,sigmoid,
 *         floor,ceil,round,sign,square,reciprocal (ops.rs:125-202)
 * reduce: sum,mean,max,min,argmax,argmin,norm  (ReduceKind, ops.rs:224-239)
 * Lookups return -1 for unknown names (replace find_*_op, ops.rs:206-220). */
int32_t oxc_binary_op_id(const char* name);
int32_t oxc_cmp_op_id(const char* name);
int32_t oxc_unary_op_id(const char* name);
int32_t oxc_reduce_kind_id(const char* name);

/* ---- elementwise registry engine ---------------------------------------
 * out must be dense row-major with the broadcast shape of the inputs; inputs
 * are arbitrary strided/broadcast views.  Replaces Tensor::binary_op / cmp_op /
 * unary_op (crates/oxi-tensor/src/lib.rs:263-357, iterate.rs:21-75) with
 * NumPy broadcasting (layout.rs:67-114; incompatible shapes ->
 * OXC_ERR_SHAPE_MISMATCH "shape mismatch: [..] vs [..]").  Comparison results
 * are 1.0 / 0.0 (lib.rs:302). */
oxc_status oxc_binary(int32_t op, const oxc_view* a, const oxc_view* b, const oxc_view* out,
                      void* stream);
oxc_status oxc_cmp(int32_t op, const oxc_view* a, const oxc_view* b, const oxc_view* out,
                   void* stream);
oxc_status oxc_unary(int32_t op, const oxc_view* in, const oxc_view* out, void* stream);
/* a op scalar with the scalar as a kernel argument instead of a full-shape
 * constant tensor (replaces const_full, crates/oxi-bindings/src/lib.rs:86-104);
 * scalar_first != 0 computes (scalar op a).  Same values: a Python scalar is
 * rounded to f32 and broadcast either way. */
oxc_status oxc_binary_scalar(int32_t op, const oxc_view* a, float scalar, int32_t scalar_first,
                             const oxc_view* out, void* stream);
/* Tensor::contiguous (crates/oxi-tensor/src/lib.rs:220-240): copies a strided
 * or broadcast view into the dense row-major `out` of the same shape, bit for
 * bit, on the elementwise engine (transposed views through its tiled paths). */
oxc_status oxc_contiguous(const oxc_view* in, const oxc_view* out, void* stream);

/* ---- reductions ----------------------------------------------------------
 * Tensor::reduce(kind, dim, keepdim) (crates/oxi-tensor/src/lib.rs:519-576,
 * ReduceKind::reduce_strip ops.rs:246-285): `out` is dense f32 with the input
 * shape minus `dim` (or with 1 there when keepdim); argmax/argmin come back as
 * float indices, the reference's f32 carrier (lib.rs:568-572).  Strips that
 * are not contiguous are folded left to right per output (the reference's own
 * order); long strips over few outputs need the workspace that
 * oxc_reduce_workspace_size reports (0 otherwise). */
size_t oxc_reduce_workspace_size(int32_t kind, const oxc_view* in, int64_t dim);
oxc_status oxc_reduce(int32_t kind, const oxc_view* in, int64_t dim, int32_t keepdim,
                      const oxc_view* out, void* workspace, size_t workspace_bytes, void* stream);
/* VJP of Tensor::reduce along `dim` (crates/oxi-autograd/src/ops.rs:327-388):
 *   sum: dx = g broadcast along dim;  mean: dx = g * f32(1/len);
 *   max/min: dx = g at each strip's first argmax/argmin, +0 elsewhere (the
 *            reference recomputes argmax/argmin from x, as this call does);
 *   norm: dx = g * (x / (norm + 1e-12)), three roundings as in the reference.
 * x is the forward input (any strides); g is dense with the forward output's
 * shape (keepdim or not: the same memory); dx is dense with x's shape.
 * argmax/argmin: OXC_ERR_NOT_IMPLEMENTED (no gradient, as in the reference).
 * max/min/norm need oxc_reduce_bwd_workspace_size bytes of workspace. */
size_t oxc_reduce_bwd_workspace_size(int32_t kind, const oxc_view* x, int64_t dim);
oxc_status oxc_reduce_bwd(int32_t kind, const oxc_view* x, int64_t dim, const float* g, float* dx,
                          void* workspace, size_t workspace_bytes, void* stream);
/* Whole-tensor reduction (reduce_strip over every element, as the Python
 * t.sum()/t.mean()/... without a dim: crates/oxi-bindings/src/lib.rs:126-143;
 * sum_all/mean_all/norm, lib.rs:582-604).  Deterministic two-stage reduction
 * with f64 partials; writes the f32 result to out[0] and, if out_f64 is not
 * NULL, the f64 value to out_f64[0] (device pointers). */
size_t oxc_reduce_all_workspace_size(int64_t numel);
oxc_status oxc_reduce_all(int32_t kind, const oxc_view* in, float* out, double* out_f64,
                          void* workspace, size_t workspace_bytes, void* stream);
/* sum over 1..16 tensors of sum(v*v), in f64 (device out[0]): the total norm
 * of clip_grad_norm_ (python/oxitorch/optim.py:242-263) without a host round
 * trip per gradient. */
size_t oxc_sum_squares_workspace_size(const oxc_view* views, int32_t count);
oxc_status oxc_sum_squares(const oxc_view* views, int32_t count, double* out, void* workspace,
                           size_t workspace_bytes, void* stream);

/* ---- RMSNorm: F.rms_norm (python/oxitorch/nn/functional.py:236-240) -------
 * x, y, dy, dx: [rows, cols] row-major; w, dw: [cols]; rstd: [rows]
 * (saved 1/sqrt(mean(x^2)+eps) per row). */
oxc_status oxc_rms_norm_fwd(const float* x, const float* w, float* y, float* rstd, int64_t rows,
                            int64_t cols, float eps, void* stream);
size_t oxc_rms_norm_bwd_workspace_size(int64_t rows, int64_t cols);
oxc_status oxc_rms_norm_bwd(const float* x, const float* w, const float* rstd, const float* dy,
                            float* dx, float* dw, int64_t rows, int64_t cols, int32_t grad_mode,
                            void* workspace, size_t workspace_bytes, void* stream);

/* ---- LayerNorm (+ fused activation): F.layer_norm then F.gelu -------------
 * (functional.py:227-233, 194-199).  y is the activation output (or the
 * layer-norm output for OXC_ACT_NONE); mean/rstd: [rows]. */
oxc_status oxc_layer_norm_fwd(const float* x, const float* w, const float* b, float* y,
                              float* mean, float* rstd, int64_t rows, int64_t cols, float eps,
                              int32_t act, void* stream);
size_t oxc_layer_norm_bwd_workspace_size(int64_t rows, int64_t cols);
oxc_status oxc_layer_norm_bwd(const float* x, const float* w, const float* b, const float* mean,
                              const float* rstd, const float* dy, float* dx, float* dw, float* db,
                              int64_t rows, int64_t cols, int32_t act, int32_t grad_mode,
                              void* workspace, size_t workspace_bytes, void* stream);

/* ---- GELU on its own: F.gelu (python/oxitorch/nn/functional.py:194-199) ------
 * y = gelu(x) and dx = dy * gelu'(x) over n dense floats, the tanh form
 * evaluated as the fused LayerNorm+GELU kernels do (OXC_ACT_GELU_TANH).  The
 * VJP takes the forward's input x. */
oxc_status oxc_gelu_fwd(const float* x, float* y, int64_t n, void* stream);
oxc_status oxc_gelu_bwd(const float* x, const float* dy, float* dx, int64_t n, void* stream);

/* ---- softmax / log_softmax: F.softmax, F.log_softmax over the last dim -----
 * (python/oxitorch/nn/functional.py:211-222).  log != 0 selects log_softmax.
 * x, y, dy, dx: [rows, cols] row-major.  The VJP takes the forward output y. */
oxc_status oxc_softmax_fwd(const float* x, float* y, int64_t rows, int64_t cols, int32_t log,
                           void* stream);
oxc_status oxc_softmax_bwd(const float* y, const float* dy, float* dx, int64_t rows, int64_t cols,
                           int32_t log, void* stream);
/* F.softmax / F.log_softmax over any `dim` (negative counts from the end) of a
 * view of any strides (python/oxitorch/nn/functional.py:211-222, whose max and
 * sum are Tensor::reduce strips along dim, crates/oxi-tensor/src/lib.rs:
 * 519-576).  y / dx are dense row-major with x's shape; dy is a view of that
 * shape.  Same per-element arithmetic as oxc_softmax_fwd / _bwd, which these
 * call for dense rows along the last dim.  A zero-length dim is
 * InvalidArgument, as the reference's max over it. */
oxc_status oxc_softmax_dim_fwd(const oxc_view* x, int64_t dim, int32_t log, float* y,
                               void* stream);
oxc_status oxc_softmax_dim_bwd(const float* y, const oxc_view* dy, int64_t dim, int32_t log,
                               float* dx, void* stream);

/* ---- cross-entropy, mean reduction: F.cross_entropy --------------------------
 * (functional.py:277-293).  logits [rows, cols]; targets int64 [rows] (negative
 * values count from the end, like the reference's numpy one-hot indexing).
 * Writes loss[0] = -(1/total_rows) * sum_rows log_softmax(logits)[r, t_r] and
 * the per-row max, sum of exp(x - max) and -log p_target that the VJP reuses.
 * total_rows = rows on one GPU; with row sharding it is the global row count
 * (each shard's loss is its share of the global mean).  A target outside
 * [-cols, cols) is recorded in err_flag (int32[4], may be NULL) and gives a NaN
 * row; read it with oxc_check_error_flag. */
oxc_status oxc_cross_entropy_fwd(const float* logits, const int64_t* targets, float* loss,
                                 float* row_max, float* row_sum, float* row_nll, int64_t rows,
                                 int64_t cols, int64_t total_rows, int32_t* err_flag,
                                 void* stream);
/* dlogits = exp(x - max) * (g/M) / sum - onehot * g/M, g = *grad_loss (device
 * scalar; NULL = 1.0), M = total_rows. */
oxc_status oxc_cross_entropy_bwd(const float* logits, const int64_t* targets,
                                 const float* row_max, const float* row_sum,
                                 const float* grad_loss, float* dlogits, int64_t rows,
                                 int64_t cols, int64_t total_rows, void* stream);

/* ---- SiLU / SwiGLU: F.silu(g) [* u] ----------------------------------------
 * (python/oxitorch/nn/functional.py:202-204; sigmoid ops.rs:176).  gate and up
 * are 2-D views [rows, cols] with any strides (a transposed gate is read
 * along its contiguous dim); up == NULL computes F.silu(gate).  h, dgate, dup
 * are dense [rows, cols].  Forward optionally writes the dim-1 reductions of
 * h (row_sum, row_max, row_argmax as float indices; each may be NULL) with the
 * reference's f32::max / first-occurrence rules.  Backward optionally writes
 * sum(dgate^2) + sum(dup^2) in f64 to the device scalar `sumsq` (needs the
 * workspace oxc_swiglu_bwd_workspace_size reports). */
oxc_status oxc_swiglu_fwd(const oxc_view* gate, const oxc_view* up, float* h, float* row_sum,
                          float* row_max, float* row_argmax, void* stream);
size_t oxc_swiglu_bwd_workspace_size(int64_t rows, int64_t cols);
oxc_status oxc_swiglu_bwd(const oxc_view* gate, const oxc_view* up, const oxc_view* dh,
                          float* dgate, float* dup, double* sumsq, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ---- embedding: F.embedding = weight.index_select(0, ids) and its VJP -------
 * (python/oxitorch/nn/functional.py:245-247; crates/oxi-tensor/src/lib.rs:665-703;
 * VJP crates/oxi-autograd/src/ops.rs:741-769).  ids int64 [n] (negative ids
 * count from the end of the whole table); out / dout [n, cols].
 * The table on this GPU holds rows [vocab_offset, vocab_offset + rows) of a
 * vocab_total-row table (vocab_offset = 0, rows = vocab_total unsharded).
 * Forward: ids of other shards give zero rows.  Backward: dtable [rows, cols]
 * is written in full; row r is the left-to-right sum of dout over r's
 * occurrences in position order (bit-identical to the reference) when r
 * occurs at most 128 times, else the sum of 128-occurrence pieces.  Ids out
 * of range of the whole table are recorded in err_flag (int32[4]). */
oxc_status oxc_embedding_fwd(const float* table, const int64_t* ids, float* out, int64_t n,
                             int64_t vocab_total, int64_t vocab_offset, int64_t rows,
                             int64_t cols, int32_t* err_flag, void* stream);
size_t oxc_embedding_bwd_workspace_size(int64_t n, int64_t rows, int64_t cols);
oxc_status oxc_embedding_bwd(const float* dout, const int64_t* ids, float* dtable, int64_t n,
                             int64_t vocab_total, int64_t vocab_offset, int64_t rows,
                             int64_t cols, int32_t* err_flag, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ---- sparse exchange of a replicated table's gradient ------------------------
 * No counterpart in the reference (it has no distributed runtime): the
 * multi-GPU step of the embedding VJP when tokens are sharded across ranks and
 * the table is replicated.  oxc_embedding_bwd_compact is oxc_embedding_bwd
 * restricted to the rows that occur: out_ids int32 [min(n, rows)] receives the
 * occurring table rows (global ids, ascending), out_rows [min(n, rows), cols]
 * their gradients (the same sums as oxc_embedding_bwd), *count (device int64)
 * how many, and shard_counts (device int64 [shards], optional) how many fall in
 * each vocab shard of a `shards`-way balanced split of vocab_total rows
 * (shard s = rows [V*s/G, V*(s+1)/G)): the send counts of an all-to-all.
 * oxc_embedding_exchange_reduce is the owner's side after the all-to-all:
 * recv_ids / recv_rows hold the rows received from `sources` ranks, source s
 * at [src_offsets[s], src_offsets[s+1]) (device int64 [sources+1]); dshard
 * [shard_rows, cols] (rows shard_lo...) becomes, per row, the sum in source
 * order from 0.0 of the received rows (zeros where none arrived).  A received
 * id outside the shard is recorded in err_flag. */
size_t oxc_embedding_bwd_compact_workspace_size(int64_t n, int64_t rows, int64_t cols);
oxc_status oxc_embedding_bwd_compact(const float* dout, const int64_t* ids, int64_t n,
                                     int64_t vocab_total, int64_t vocab_offset, int64_t rows,
                                     int64_t cols, int32_t* out_ids, float* out_rows,
                                     int64_t* count, int32_t shards, int64_t* shard_counts,
                                     int32_t* err_flag, void* workspace, size_t workspace_bytes,
                                     void* stream);
/* The compact VJP in two calls, so the per-shard counts can cross ranks while
 * the sums run: _plan sorts the ids and writes out_ids, count and
 * shard_counts (a few microseconds of work); _sum then writes out_rows.  Both
 * take the same workspace, which carries the plan to the sums, and run in that
 * order (same stream, or ordered by an event). */
oxc_status oxc_embedding_bwd_compact_plan(const int64_t* ids, int64_t n, int64_t vocab_total,
                                          int64_t vocab_offset, int64_t rows, int64_t cols,
                                          int32_t* out_ids, int64_t* count, int32_t shards,
                                          int64_t* shard_counts, int32_t* err_flag,
                                          void* workspace, size_t workspace_bytes, void* stream);
oxc_status oxc_embedding_bwd_compact_sum(const float* dout, int64_t n, int64_t rows, int64_t cols,
                                         float* out_rows, void* workspace,
                                         size_t workspace_bytes, void* stream);
size_t oxc_embedding_exchange_reduce_workspace_size(int32_t sources, int64_t shard_rows);
oxc_status oxc_embedding_exchange_reduce(const int32_t* recv_ids, const float* recv_rows,
                                         const int64_t* src_offsets, int32_t sources,
                                         int64_t shard_lo, int64_t shard_rows, int64_t cols,
                                         float* dshard, int32_t* err_flag, void* workspace,
                                         size_t workspace_bytes, void* stream);

/* ---- multi-GPU collectives for a native host ---------------------------------
 * No counterpart in the reference (it has no distributed runtime; plan.md:325
 * lists one as a stretch goal).  The exchanges of the sharded layer path --
 * the all-reduce of weight-gradient and loss partials (f32) and of sums of
 * squares (f64), the reduce-scatter of a table gradient, and the variable
 * all-to-all of the sparse embedding exchange -- for a host that does not run
 * Python.  NCCL over NVLink / NVSwitch, loaded at run time from libnccl.so.2
 * (OXC_ERR_OTHER when it cannot be loaded).  One communicator per process and
 * GPU: rank 0 makes an id (oxc_comm_unique_id), the host hands its
 * OXC_COMM_ID_BYTES bytes to every rank out of band, and each rank calls
 * oxc_comm_init with its device current.  Every rank issues the same calls in
 * the same order; each call is asynchronous on `stream`.  oxc_comm_alltoallv
 * sends send_counts[p] elements of elem_bytes to rank p (consecutive in
 * `send`) and receives recv_counts[p] from it; both count arrays are on the
 * host. */
typedef struct oxc_comm oxc_comm;
#define OXC_COMM_ID_BYTES 128
oxc_status oxc_comm_unique_id(uint8_t* id);
oxc_status oxc_comm_init(oxc_comm** comm, const uint8_t* id, int32_t world, int32_t rank);
oxc_status oxc_comm_destroy(oxc_comm* comm);
oxc_status oxc_comm_allreduce_sum_f32(oxc_comm* comm, float* buf, int64_t n, void* stream);
oxc_status oxc_comm_allreduce_sum_f64(oxc_comm* comm, double* buf, int64_t n, void* stream);
oxc_status oxc_comm_reduce_scatter_f32(oxc_comm* comm, const float* in, float* out,
                                       int64_t count_per_rank, void* stream);
oxc_status oxc_comm_alltoallv(oxc_comm* comm, const void* send, const int64_t* send_counts,
                              void* recv, const int64_t* recv_counts, int64_t elem_bytes,
                              void* stream);

/* ---- the fused exchange over peer memory --------------------------------------
 * No counterpart in the reference.  The VJP of a replicated table with
 * token-sharded ids that delivers its rows itself: each occurring row's sum is
 * stored straight into the receive region of the rank that owns the row, over
 * NVLink (peer memory mapped with oxc_ipc_import), so the transfer overlaps
 * the sums and nothing waits on the host.  Ownership: cyclic = 0, owner p holds
 * table rows [lo[p], lo[p+1]); cyclic = 1, owner p holds rows p, p + world,
 * p + 2 world, ... (lo unused), which spreads Zipf-hot low ids over every
 * owner.  oxc_emb_push (device memory, built once by the host) names, for this
 * source rank, every owner's region: rows [cap][cols], ids [cap], and the
 * owner's count slot for this source; cap is at least the largest shard's row
 * count.  After every rank's oxc_embedding_bwd_push, a stream-ordered barrier
 * across the ranks (any collective: its completion on a rank implies every
 * rank's earlier kernels, whose peer stores are fenced at system scope, have
 * completed), then each owner runs oxc_embedding_exchange_reduce_regions over
 * its own regions (source s at [s * cap, s * cap + counts[s])) into its dense
 * shard: row v of it is table row shard_lo + v * shard_stride (contiguous:
 * shard_lo = lo[p], stride 1; cyclic: shard_lo = p, stride = world).  A row
 * beyond `cap` for one owner is recorded in err_flag and not sent. */
#define OXC_PUSH_MAX_RANKS 16
typedef struct oxc_emb_push {
  int32_t world;
  int32_t source;  /* this (source) rank: stores to its own region need no system-scope fence */
  int32_t cyclic;  /* 1: owner p holds rows p, p + world, ...; 0: rows [lo[p], lo[p+1]) */
  int32_t local;   /* 1: every region named here is in this GPU's own memory (the pull form) */
  int64_t cap;
  int64_t lo[OXC_PUSH_MAX_RANKS + 1];  /* contiguous ownership: owner p's first row, lo[world] = rows */
  float* rows[OXC_PUSH_MAX_RANKS];
  int32_t* ids[OXC_PUSH_MAX_RANKS];
  int64_t* count[OXC_PUSH_MAX_RANKS];
} oxc_emb_push;
oxc_status oxc_embedding_bwd_push(const float* dout, const int64_t* ids, int64_t n,
                                  int64_t vocab_total, int64_t cols, const oxc_emb_push* push,
                                  int32_t* err_flag, void* workspace, size_t workspace_bytes,
                                  void* stream);
oxc_status oxc_embedding_exchange_reduce_regions(const int32_t* recv_ids, const float* recv_rows,
                                                 const int64_t* counts, int32_t sources,
                                                 int64_t cap, int64_t shard_lo,
                                                 int64_t shard_stride, int64_t shard_rows,
                                                 int64_t cols, float* dshard, int32_t* err_flag,
                                                 void* workspace, size_t workspace_bytes,
                                                 void* stream);
/* The pull form of the same exchange.  Each source pushes into its OWN memory
 * (an oxc_emb_push table with local = 1 naming, for every owner p, its send
 * region p), so the VJP stores nothing over NVLink.  After the barrier, each
 * owner's oxc_embedding_exchange_pull reads, for every source s in rank order,
 * the region s holds for it -- peer memory mapped with oxc_ipc_import, or its
 * own for s = this rank -- and sums the rows in source order from 0.0 into its
 * dense shard (the same bits as oxc_embedding_exchange_reduce_regions), on a
 * communication stream that overlaps the next forward.  oxc_emb_pull (device
 * memory) lists the sources' regions for this owner; the workspace is
 * oxc_embedding_exchange_reduce_workspace_size(sources, shard_rows). */
typedef struct oxc_emb_pull {
  const float* rows[OXC_PUSH_MAX_RANKS];    /* source s's region for this owner: [cap][cols] */
  const int32_t* ids[OXC_PUSH_MAX_RANKS];   /* [cap] */
  const int64_t* count[OXC_PUSH_MAX_RANKS]; /* one count */
} oxc_emb_pull;
oxc_status oxc_embedding_exchange_pull(const oxc_emb_pull* pull, int32_t sources, int64_t cap,
                                       int64_t shard_lo, int64_t shard_stride,
                                       int64_t shard_rows, int64_t cols, float* dshard,
                                       int32_t* err_flag, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* Device memory shared between the processes of one node: oxc_ipc_export gives
 * the handle of the allocation holding dev_ptr and dev_ptr's byte offset in it;
 * oxc_ipc_import maps it into another process (peer access enabled) and
 * returns the exported address there; oxc_ipc_close unmaps it. */
#define OXC_IPC_HANDLE_BYTES 64
oxc_status oxc_ipc_export(const void* dev_ptr, uint8_t* handle, int64_t* offset);
oxc_status oxc_ipc_import(const uint8_t* handle, int64_t offset, void** dev_ptr);
oxc_status oxc_ipc_close(void* dev_ptr, int64_t offset);

/* ---- index_select along any dim, and its VJP --------------------------------
 * oxc_index_select replaces Tensor::index_select (crates/oxi-tensor/src/lib.rs:
 * 665-703) for any dim and any strides of x: out (dense row-major, x's shape
 * with dim -> n) = x[..., ids[k], ...].  ids int64 [n] on the device; negative
 * ids count from the end; an id out of range gives zeros and is recorded in
 * err_flag (int32[4]; oxc_check_error_flag then reports OutOfBounds with the
 * reference's "index i out of range for dim d of size len").
 * oxc_gather_dim0 replaces Tensor::gather_dim0 (lib.rs:857-886): index_select
 * on dim 0, InvalidArgument for a 0-D x.
 * oxc_index_select_bwd replaces scatter_index_select, the VJP of
 * ops::index_select (crates/oxi-autograd/src/ops.rs:498-517, 741-769): gx
 * (dense, `shape`, ndim dims) is zero except gx[o, ids[k], i] = sum of
 * g[o, k, i] over the occurrences k of each index, in position order from 0.0.
 * Slices of fewer than 128 floats (inner dims) are summed sequentially per
 * element, bit-identical to the reference; wider slices use the embedding VJP's
 * pipeline (bit-identical for indices occurring at most 128 times, else summed
 * in 128-occurrence pieces). */
oxc_status oxc_index_select(const oxc_view* x, int64_t dim, const int64_t* ids, int64_t n,
                            float* out, int32_t* err_flag, void* stream);
oxc_status oxc_gather_dim0(const oxc_view* x, const int64_t* ids, int64_t n, float* out,
                           int32_t* err_flag, void* stream);
size_t oxc_index_select_bwd_workspace_size(const int64_t* shape, int32_t ndim, int64_t dim,
                                           int64_t n);
oxc_status oxc_index_select_bwd(const float* g, const int64_t* ids, int64_t n,
                                const int64_t* shape, int32_t ndim, int64_t dim, float* gx,
                                int32_t* err_flag, void* workspace, size_t workspace_bytes,
                                void* stream);

/* ---- dim-0 scatter and its VJP: row selection ------------------------------
 * Replaces the host loops of Tensor::scatter_dim0 (crates/oxi-tensor/src/lib.rs:
 * 895-933, Python Tensor.scatter) and of the ops::scatter_dim0 VJP
 * (crates/oxi-autograd/src/ops.rs:531-598).  out[i] (rows of `inner` floats,
 * i < n) = a[map[i]] when map[i] >= 0, else b[i] when b is not null, else
 * zeros.  The caller resolves last-write-wins into `map` (int64, on the
 * device): forward map[r] = last writer of r or -1 with a = values, b = base;
 * d/dbase map[r] = r for unwritten rows, -1 for written ones, a = g, b = null;
 * d/dvalues map[p] = row of p for last writers, -1 for overwritten slots,
 * a = g, b = null.  The same call gives the ops::narrow_dim0 VJP
 * (crates/oxi-autograd/src/ops.rs:427-455, concat_rows of zero blocks around
 * g): map[r] = r - lo for the kept rows, -1 elsewhere, a = g, b = null.
 * map[i] >= a_rows is recorded in err_flag (int32[4]) and
 * that row is skipped.  Bit-exact (copies). */
oxc_status oxc_select_rows(const float* a, int64_t a_rows, const int64_t* map, int64_t n,
                           const float* b, float* out, int64_t inner, int32_t* err_flag,
                           void* stream);

/* ---- masked_select: boolean-mask indexing and its VJP -------------------------
 * Replaces Tensor::masked_select (crates/oxi-tensor/src/lib.rs:939-960) and the
 * host walk of the ops::masked_select VJP (crates/oxi-autograd/src/ops.rs:
 * 610-665).  x and mask are views of the broadcast grid's shape (broadcast
 * dims with stride 0); picks follow the grid's row-major order.
 * oxc_masked_select_count: per-chunk pick counts turned into offsets in the
 *   workspace (int64), the total at index ceil(n / 4096) (n = grid points).
 *   by_mask = 0: the forward's picks (mask != 0 and x not NaN: the
 *   reference's NaN sentinel drops picked NaNs); by_mask = 1: the VJP's
 *   (mask != 0; x may be null).
 * oxc_masked_select_fwd: out[total] = the picked x values (after a by_mask = 0
 *   count).
 * oxc_masked_select_bwd: gfull (dense, grid-shaped) = g[rank] at every point
 *   the mask picks, 0 elsewhere (after a by_mask = 1 count); ranks >= ng
 *   give 0.
 * oxc_broadcast_fold: gx[x_shape] = the sum of gfull over the grid dims where
 *   x has size 1, each x element folded in grid order from +0.0 in f32 (the
 *   reference's accumulation order for elements picked more than once). */
size_t oxc_masked_select_workspace_size(int64_t n);
oxc_status oxc_masked_select_count(const oxc_view* x, const oxc_view* mask, int32_t by_mask,
                                   void* workspace, size_t workspace_bytes, void* stream);
oxc_status oxc_masked_select_fwd(const oxc_view* x, const oxc_view* mask, const void* workspace,
                                 float* out, void* stream);
oxc_status oxc_masked_select_bwd(const float* g, int64_t ng, const oxc_view* mask,
                                 const void* workspace, float* gfull, void* stream);
oxc_status oxc_broadcast_fold(const float* gfull, const int64_t* grid_shape, const int64_t* x_shape,
                              int32_t ndim, float* gx, void* stream);

/* ---- LayerNorm backward without a caller workspace ------------------------
 * No counterpart in the reference: an addition for callers that cannot call
 * cudaMalloc (a host that owns all device memory through its own pool, or a
 * latency-critical step that cannot afford cudaMalloc's implicit device
 * synchronisation).  Same arguments and results as oxc_layer_norm_bwd minus
 * the workspace: the scratch is a fixed device array of
 * OXC_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that loads
 * the library holds until exit.  Sizes whose scratch
 * (oxc_layer_norm_bwd_workspace_size) exceeds it are rejected with
 * OXC_ERR_INVALID_ARGUMENT.  The first call on a device looks up the array's
 * device address (make it before any stream capture); all calls on a device
 * share the array, so calls that overlap on the GPU race and must be
 * serialised by the caller.  The looked-up address is cached per device for
 * the life of the process and does not survive cudaDeviceReset: a process
 * that resets a device must not call this entry point on it again.
 * Allocates nothing. */
#define OXC_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
oxc_status oxc_layer_norm_bwd_noalloc(const float* x, const float* w, const float* b,
                                      const float* mean, const float* rstd, const float* dy,
                                      float* dx, float* dw, float* db, int64_t rows, int64_t cols,
                                      int32_t act, int32_t grad_mode, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OXICUDA_H */
