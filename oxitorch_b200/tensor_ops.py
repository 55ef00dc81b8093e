"""Device-side mirror of oxi-tensor's ``Tensor`` registry methods.

Same names, argument meaning and errors as ``crates/oxi-tensor/src/lib.rs``:
``binary_op(name, a, b)``, ``cmp_op``, ``unary_op``, ``reduce(kind, x, dim,
keepdim)``, the whole-tensor ``sum_all``/``mean_all``/``reduce_all``, plus
``clip_grad_norm_`` (python/oxitorch/optim.py:242-263) over device
gradients.  Inputs are torch CUDA float32 tensors with any strides (views:
transposes, slices, zero-stride broadcasts); outputs are dense, like the
reference's ``from_results``.  Every op is one call into liboxicuda.so.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N
from .functional import _require_cuda_f32, _stream, _workspace

BINARY_OPS = ["add", "sub", "mul", "div", "pow", "min", "max"]
CMP_OPS = ["eq", "ne", "lt", "le", "gt", "ge"]
UNARY_OPS = ["neg", "abs", "sqrt", "rsqrt", "exp", "log", "log2", "log10", "sin", "cos", "tanh",
             "relu", "sigmoid", "floor", "ceil", "round", "sign", "square", "reciprocal"]
REDUCE_KINDS = ["sum", "mean", "max", "min", "argmax", "argmin", "norm"]


def _broadcast_shape(a, b):
    """layout::broadcast_shapes (layout.rs:67-88)."""
    rank = max(len(a), len(b))
    out = []
    for i in range(rank):
        ia, ib = len(a) - rank + i, len(b) - rank + i
        da = a[ia] if ia >= 0 else 1
        db = b[ib] if ib >= 0 else 1
        if da != db and da != 1 and db != 1:
            raise ValueError(f"shape mismatch: {list(a)} vs {list(b)}")
        out.append(max(da, db))
    return out


def _op_id(table, name, what):
    if name not in table:
        raise ValueError(f'invalid argument: unknown {what} op "{name}"')
    return table.index(name)


def _scalar(x):
    return isinstance(x, (int, float))


def binary_op(name, a, b):
    """Tensor::binary_op (lib.rs:332-336); a Python number on either side is a
    kernel argument (the value the reference's full-shape constant holds)."""
    op = _op_id(BINARY_OPS, name, "binary")
    if _scalar(a) and _scalar(b):
        raise TypeError("at least one operand must be a tensor")
    if _scalar(b) or _scalar(a):
        t, c, first = (a, b, 0) if _scalar(b) else (b, a, 1)
        _require_cuda_f32("operand", t)
        out = torch.empty(t.shape, dtype=torch.float32, device=t.device)
        N.check(N.load().oxc_binary_scalar(op, ctypes.byref(N.make_view(t)), float(c), first,
                                           ctypes.byref(N.make_view(out)), _stream()), name)
        return out
    _require_cuda_f32("a", a)
    _require_cuda_f32("b", b)
    out = torch.empty(_broadcast_shape(list(a.shape), list(b.shape)), dtype=torch.float32,
                      device=a.device)
    N.check(N.load().oxc_binary(op, ctypes.byref(N.make_view(a)), ctypes.byref(N.make_view(b)),
                                ctypes.byref(N.make_view(out)), _stream()), name)
    return out


def cmp_op(name, a, b):
    """Tensor::cmp_op (lib.rs:342-347): 1.0 where true, 0.0 elsewhere."""
    op = _op_id(CMP_OPS, name, "comparison")
    _require_cuda_f32("a", a)
    _require_cuda_f32("b", b)
    out = torch.empty(_broadcast_shape(list(a.shape), list(b.shape)), dtype=torch.float32,
                      device=a.device)
    N.check(N.load().oxc_cmp(op, ctypes.byref(N.make_view(a)), ctypes.byref(N.make_view(b)),
                             ctypes.byref(N.make_view(out)), _stream()), name)
    return out


def unary_op(name, a):
    """Tensor::unary_op (lib.rs:353-357)."""
    op = _op_id(UNARY_OPS, name, "unary")
    _require_cuda_f32("a", a)
    out = torch.empty(a.shape, dtype=torch.float32, device=a.device)
    N.check(N.load().oxc_unary(op, ctypes.byref(N.make_view(a)), ctypes.byref(N.make_view(out)),
                               _stream()), name)
    return out


def reduce(kind, x, dim, keepdim=False):
    """Tensor::reduce (lib.rs:519-576); argmax/argmin come back as float
    indices like the reference's f32 carrier."""
    k = _op_id(REDUCE_KINDS, kind, "reduction")
    _require_cuda_f32("x", x)
    nd = x.dim()
    d = dim + nd if dim < 0 else dim
    if not 0 <= d < nd:
        raise ValueError(f"invalid argument: dim {dim} out of range for {nd}-D tensor")
    shape = list(x.shape)
    if keepdim:
        shape[d] = 1
    else:
        shape.pop(d)
    out = torch.empty(shape, dtype=torch.float32, device=x.device)
    L = N.load()
    xv = N.make_view(x)
    ws = _workspace(L.oxc_reduce_workspace_size(k, ctypes.byref(xv), d), x.device)
    N.check(L.oxc_reduce(k, ctypes.byref(xv), d, int(keepdim), ctypes.byref(N.make_view(out)),
                         ws.data_ptr(), ws.numel(), _stream()), kind)
    return out


def reduce_all(kind, x, f64=False):
    """reduce_strip over every element (bindings lib.rs:126-143): a 0-d f32
    tensor (and the f64 value when f64=True)."""
    k = _op_id(REDUCE_KINDS, kind, "reduction")
    _require_cuda_f32("x", x)
    L = N.load()
    out = torch.empty((), dtype=torch.float32, device=x.device)
    out64 = torch.empty((), dtype=torch.float64, device=x.device)
    ws = _workspace(L.oxc_reduce_all_workspace_size(x.numel()), x.device)
    N.check(L.oxc_reduce_all(k, ctypes.byref(N.make_view(x)), out.data_ptr(), out64.data_ptr(),
                             ws.data_ptr(), ws.numel(), _stream()), kind)
    return (out, out64) if f64 else out


def sum_all(x):
    return reduce_all("sum", x)


def mean_all(x):
    return reduce_all("mean", x)


def sum_squares(tensors):
    """sum over tensors of sum(v*v) in f64, one device pass (0-d f64 tensor)."""
    tensors = list(tensors)
    if not 1 <= len(tensors) <= 16:
        raise ValueError("invalid argument: sum_squares takes 1..16 tensors")
    for t in tensors:
        _require_cuda_f32("tensor", t)
    views = (N.View * len(tensors))(*[N.make_view(t) for t in tensors])
    L = N.load()
    out = torch.empty((), dtype=torch.float64, device=tensors[0].device)
    ws = _workspace(L.oxc_sum_squares_workspace_size(views, len(tensors)), tensors[0].device)
    N.check(L.oxc_sum_squares(views, len(tensors), out.data_ptr(), ws.data_ptr(), ws.numel(),
                              _stream()), "sum_squares")
    return out


def clip_grad_norm_(grads, max_norm, norm_type=2.0):
    """clip_grad_norm_ (python/oxitorch/optim.py:242-263) for norm_type 2 over
    device gradients, in place: total = sqrt(sum of squares); if
    max_norm / (total + 1e-6) < 1 every gradient is scaled by it.  Returns
    the pre-clip total norm as a Python float, like the reference."""
    if norm_type != 2.0:
        raise NotImplementedError("not implemented: clip_grad_norm_ with norm_type != 2 on device")
    grads = [g for g in grads if g is not None]
    if not grads:
        return 0.0
    total = 0.0
    for i in range(0, len(grads), 16):
        total += float(sum_squares(grads[i:i + 16]).item())
    total = total ** 0.5
    scale = max_norm / (total + 1e-6)
    if scale < 1.0:
        for g in grads:
            scale_(g, scale)
    return total


def scale_(g, scale):
    """g *= scale in place (the registry's mul with a scalar operand)."""
    _require_cuda_f32("tensor", g)
    v = N.make_view(g)
    N.check(N.load().oxc_binary_scalar(2, ctypes.byref(v), float(scale), 0, ctypes.byref(v),
                                       _stream()), "scale_")
    return g
