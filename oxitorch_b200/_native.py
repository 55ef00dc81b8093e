"""ctypes binding of liboxicuda.so (the C ABI declared in include/oxicuda.h).

The library is loaded from this package directory.  There is no fallback:
if the shared library is missing or no CUDA device is visible, every entry
point raises, so a device tensor can never silently run on the CPU.

Status codes map onto Python exceptions the way the reference maps
OxitorchError (crates/oxi-bindings/src/error.rs:22-32): InvalidArgument and
ShapeMismatch -> ValueError, NotImplemented -> NotImplementedError, the rest
-> RuntimeError.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboxicuda.so")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_SHAPE_MISMATCH = 2
ERR_NOT_IMPLEMENTED = 3
ERR_OUT_OF_BOUNDS = 4
ERR_OTHER = 5
ERR_TIMEOUT = 6

GRAD_REF = 0
GRAD_EXACT = 1
ACT_NONE = 0
ACT_GELU_TANH = 1

MAX_DIMS = 8


class View(ctypes.Structure):
    """struct oxc_view: data pointer, ndim, shape[8], strides[8] (elements)."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("strides", ctypes.c_int64 * MAX_DIMS),
    ]


PUSH_MAX_RANKS = 16


class EmbPush(ctypes.Structure):
    """struct oxc_emb_push: where one source rank's VJP rows go on every owner."""

    _fields_ = [
        ("world", ctypes.c_int32),
        ("source", ctypes.c_int32),
        ("cyclic", ctypes.c_int32),
        ("local", ctypes.c_int32),
        ("cap", ctypes.c_int64),
        ("lo", ctypes.c_int64 * (PUSH_MAX_RANKS + 1)),
        ("rows", ctypes.c_void_p * PUSH_MAX_RANKS),
        ("ids", ctypes.c_void_p * PUSH_MAX_RANKS),
        ("count", ctypes.c_void_p * PUSH_MAX_RANKS),
    ]


class EmbPull(ctypes.Structure):
    """struct oxc_emb_pull: every source's region for one owner (the pull form)."""

    _fields_ = [
        ("rows", ctypes.c_void_p * PUSH_MAX_RANKS),
        ("ids", ctypes.c_void_p * PUSH_MAX_RANKS),
        ("count", ctypes.c_void_p * PUSH_MAX_RANKS),
    ]


class GatherColumn(ctypes.Structure):
    """struct oxc_gather_column: source rows, destination rows, bytes per row."""

    _fields_ = [("src", ctypes.c_void_p), ("dst", ctypes.c_void_p), ("row_bytes", ctypes.c_int64)]


class PlaneMap(ctypes.Structure):
    """struct oxc_plane_map: where one output image plane reads its pixels."""

    _fields_ = [
        ("src_offset", ctypes.c_int64),
        ("row_offset", ctypes.c_int32),
        ("col_base", ctypes.c_int32),
        ("col_step", ctypes.c_int32),
        ("channel", ctypes.c_int32),
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F32 = ctypes.c_float
_SZ = ctypes.c_size_t
_VP = ctypes.POINTER(View)
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64

# name -> (restype, argtypes); one line per entry point of include/oxicuda.h
SIGNATURES = {
    "oxc_abi_version": (_I32, []),
    "oxc_last_error": (ctypes.c_char_p, []),
    "oxc_device_count": (_I32, []),
    "oxc_stream_sync": (_I32, [_P, _I64]),
    "oxc_check_error_flag": (_I32, [_P, _P, _I64]),
    "oxc_kernel_error": (_I32, [ctypes.POINTER(ctypes.c_uint32), _I32]),
    "oxc_binary_op_id": (_I32, [ctypes.c_char_p]),
    "oxc_cmp_op_id": (_I32, [ctypes.c_char_p]),
    "oxc_unary_op_id": (_I32, [ctypes.c_char_p]),
    "oxc_reduce_kind_id": (_I32, [ctypes.c_char_p]),
    "oxc_binary": (_I32, [_I32, _VP, _VP, _VP, _P]),
    "oxc_cmp": (_I32, [_I32, _VP, _VP, _VP, _P]),
    "oxc_unary": (_I32, [_I32, _VP, _VP, _P]),
    "oxc_binary_scalar": (_I32, [_I32, _VP, _F32, _I32, _VP, _P]),
    "oxc_contiguous": (_I32, [_VP, _VP, _P]),
    "oxc_reduce_workspace_size": (_SZ, [_I32, _VP, _I64]),
    "oxc_reduce": (_I32, [_I32, _VP, _I64, _I32, _VP, _P, _SZ, _P]),
    "oxc_reduce_bwd_workspace_size": (_SZ, [_I32, _VP, _I64]),
    "oxc_reduce_bwd": (_I32, [_I32, _VP, _I64, _P, _P, _P, _SZ, _P]),
    "oxc_reduce_all_workspace_size": (_SZ, [_I64]),
    "oxc_reduce_all": (_I32, [_I32, _VP, _P, _P, _P, _SZ, _P]),
    "oxc_sum_squares_workspace_size": (_SZ, [_VP, _I32]),
    "oxc_sum_squares": (_I32, [_VP, _I32, _P, _P, _SZ, _P]),
    "oxc_rms_norm_fwd": (_I32, [_P, _P, _P, _P, _I64, _I64, _F32, _P]),
    "oxc_rms_norm_bwd_workspace_size": (_SZ, [_I64, _I64]),
    "oxc_rms_norm_bwd": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _P, _SZ, _P]),
    "oxc_layer_norm_fwd": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _F32, _I32, _P]),
    "oxc_layer_norm_bwd_workspace_size": (_SZ, [_I64, _I64]),
    "oxc_layer_norm_bwd": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _I32,
                                  _P, _SZ, _P]),
    "oxc_gelu_fwd": (_I32, [_P, _P, _I64, _P]),
    "oxc_gelu_bwd": (_I32, [_P, _P, _P, _I64, _P]),
    "oxc_softmax_fwd": (_I32, [_P, _P, _I64, _I64, _I32, _P]),
    "oxc_softmax_bwd": (_I32, [_P, _P, _P, _I64, _I64, _I32, _P]),
    "oxc_softmax_dim_fwd": (_I32, [_VP, _I64, _I32, _P, _P]),
    "oxc_softmax_dim_bwd": (_I32, [_P, _VP, _I64, _I32, _P, _P]),
    "oxc_cross_entropy_fwd": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P]),
    "oxc_cross_entropy_bwd": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "oxc_swiglu_fwd": (_I32, [_VP, _VP, _P, _P, _P, _P, _P]),
    "oxc_swiglu_bwd_workspace_size": (_SZ, [_I64, _I64]),
    "oxc_swiglu_bwd": (_I32, [_VP, _VP, _VP, _P, _P, _P, _P, _SZ, _P]),
    "oxc_embedding_fwd": (_I32, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P]),
    "oxc_embedding_bwd_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "oxc_embedding_bwd": (_I32, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _SZ, _P]),
    "oxc_embedding_bwd_compact_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "oxc_embedding_bwd_compact": (_I32, [_P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _I32,
                                         _P, _P, _P, _SZ, _P]),
    "oxc_embedding_bwd_compact_plan": (_I32, [_P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I32, _P,
                                              _P, _P, _SZ, _P]),
    "oxc_embedding_bwd_compact_sum": (_I32, [_P, _I64, _I64, _I64, _P, _P, _SZ, _P]),
    "oxc_embedding_exchange_reduce_workspace_size": (_SZ, [_I32, _I64]),
    "oxc_embedding_exchange_reduce": (_I32, [_P, _P, _P, _I32, _I64, _I64, _I64, _P, _P, _P, _SZ,
                                             _P]),
    "oxc_comm_unique_id": (_I32, [_P]),
    "oxc_comm_init": (_I32, [ctypes.POINTER(_P), _P, _I32, _I32]),
    "oxc_comm_destroy": (_I32, [_P]),
    "oxc_comm_allreduce_sum_f32": (_I32, [_P, _P, _I64, _P]),
    "oxc_comm_allreduce_sum_f64": (_I32, [_P, _P, _I64, _P]),
    "oxc_comm_reduce_scatter_f32": (_I32, [_P, _P, _P, _I64, _P]),
    "oxc_comm_alltoallv": (_I32, [_P, _P, _P, _P, _P, _I64, _P]),
    "oxc_embedding_bwd_push": (_I32, [_P, _P, _I64, _I64, _I64, _P, _P, _P, _SZ, _P]),
    "oxc_embedding_exchange_reduce_regions": (_I32, [_P, _P, _P, _I32, _I64, _I64, _I64, _I64,
                                                     _I64, _P, _P, _P, _SZ, _P]),
    "oxc_embedding_exchange_pull": (_I32, [_P, _I32, _I64, _I64, _I64, _I64, _I64, _P, _P, _P,
                                           _SZ, _P]),
    "oxc_ipc_export": (_I32, [_P, _P, ctypes.POINTER(_I64)]),
    "oxc_ipc_import": (_I32, [_P, _I64, ctypes.POINTER(_P)]),
    "oxc_ipc_close": (_I32, [_P, _I64]),
    "oxc_index_select": (_I32, [_VP, _I64, _P, _I64, _P, _P, _P]),
    "oxc_gather_dim0": (_I32, [_VP, _P, _I64, _P, _P, _P]),
    "oxc_index_select_bwd_workspace_size": (_SZ, [_P, _I32, _I64, _I64]),
    "oxc_index_select_bwd": (_I32, [_P, _P, _I64, _P, _I32, _I64, _P, _P, _P, _SZ, _P]),
    "oxc_select_rows": (_I32, [_P, _I64, _P, _I64, _P, _P, _I64, _P, _P]),
    "oxc_masked_select_workspace_size": (_SZ, [_I64]),
    "oxc_masked_select_count": (_I32, [_VP, _VP, _I32, _P, _SZ, _P]),
    "oxc_masked_select_fwd": (_I32, [_VP, _VP, _P, _P, _P]),
    "oxc_masked_select_bwd": (_I32, [_P, _I64, _VP, _P, _P, _P]),
    "oxc_broadcast_fold": (_I32, [_P, _P, _P, _I32, _P, _P]),
    "oxc_layer_norm_bwd_noalloc": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32,
                                          _I32, _P]),
    "oxc_sgd_step": (_I32, [_P, _P, _P, _I64, _F32, _F32, _I32, _P]),
    "oxc_adamw_step": (_I32, [_P, _P, _P, _P, _I64, _F32, _F32, _F32, _F32, _F32, _I32, _I64, _P]),
    "oxc_clip_grad_value": (_I32, [_P, _I64, _F32, _P]),
    "oxc_gather_rows": (_I32, [ctypes.POINTER(GatherColumn), _I32, _P, _I64, _I64, _P, _P]),
    "oxc_image_epoch": (_I32, [_P, _I64, _P, _I64, _I64, _P, _I64, _I32, _I32, _I32, _I32, _P, _I32,
                               _I32, _P, _P, _P]),
    "oxc_epoch_seed": (_U64, [_U64, _U64]),
    "oxc_batch_seed": (_U64, [_U64, _P, _I64]),
    "oxc_permutation": (_I32, [_U32, _I64, _P]),
    "oxc_epoch_transform_plan": (_I32, [_P, _I64, _I64, _U64, _P, _P, _P, _I32, _I32, _P, _P, _I64,
                                        _P]),
    "oxc_upload": (_I32, [_P, _P, _I64, _P]),
    "oxc_download": (_I32, [_P, _P, _I64, _P]),
}

NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024

_lib = None


def load(require_device: bool = True):
    """Loads the library (once).  Raises if it is missing; with
    ``require_device`` also raises when no CUDA device is visible."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"oxitorch_b200: {LIB_PATH} is not built; run `python -c "
                "'import __graft_entry__ as g; g.build()'` (there is no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    if require_device and _lib.oxc_device_count() <= 0:
        raise RuntimeError("oxitorch_b200: no CUDA device is visible (there is no CPU fallback)")
    return _lib


def last_error() -> str:
    msg = load(False).oxc_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str = "") -> None:
    """Raises the reference's exception type for a failing status."""
    if status == OK:
        return
    msg = last_error() or f"{what}: status {status}"
    if status in (ERR_INVALID_ARGUMENT, ERR_SHAPE_MISMATCH):
        raise ValueError(msg)
    if status == ERR_NOT_IMPLEMENTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def kernel_error_bits(clear: bool = True) -> int:
    """Device-side error bits recorded by kernels (synchronises nothing: call
    after the stream drained)."""
    v = ctypes.c_uint32(0)
    check(load().oxc_kernel_error(ctypes.byref(v), int(clear)), "oxc_kernel_error")
    return v.value


def make_view(t) -> View:
    """oxc_view of a torch CUDA float32 tensor (any strides, offset applied)."""
    if t.dim() > MAX_DIMS:
        raise NotImplementedError(f"not implemented: tensors of rank {t.dim()} > {MAX_DIMS}")
    v = View()
    v.data = t.data_ptr()
    v.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        v.shape[i] = s
        v.strides[i] = st
    return v
