"""Device-side mirror of oxi-tensor's ``Tensor`` registry methods.

Same names, argument meaning and errors as ``crates/oxi-tensor/src/lib.rs``:
``binary_op(name, a, b)``, ``cmp_op``, ``unary_op``, ``reduce(kind, x, dim,
keepdim)`` with its VJP ``reduce_backward`` and the autograd helper
``unbroadcast`` (graph.rs:274-313), the whole-tensor
``sum_all``/``mean_all``/``reduce_all``, plus
``clip_grad_norm_`` and ``clip_grad_value_`` (python/oxitorch/optim.py:242-272)
over device gradients.  Inputs are torch CUDA float32 tensors with any strides (views:
transposes, slices, zero-stride broadcasts); outputs are dense, like the
reference's ``from_results``.  Every op is one call into liboxicuda.so.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N
from .functional import _require_cuda_f32, _stream, _workspace, dense

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
    indices like the reference's f32 carrier.  Differentiable (for every kind
    but argmax/argmin) through the reference's reduce VJP, reduce_backward."""
    if x.requires_grad and torch.is_grad_enabled() and kind not in ("argmax", "argmin"):
        return _Reduce.apply(x, kind, dim, keepdim)
    return _reduce_fwd(kind, x, dim, keepdim)


def _reduce_fwd(kind, x, dim, keepdim):
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


def reduce_backward(kind, x, dim, g):
    """VJP of reduce(kind, x, dim, keepdim) (crates/oxi-autograd/src/ops.rs:
    327-388) for upstream gradient g (the forward output's shape, keepdim or
    not): sum broadcasts g, mean scales it by f32(1/len), max/min send it to
    each strip's first argmax/argmin, norm multiplies by x / (norm + 1e-12).
    argmax/argmin raise NotImplementedError, as in the reference."""
    k = _op_id(REDUCE_KINDS, kind, "reduction")
    _require_cuda_f32("x", x)
    _require_cuda_f32("g", g)
    nd = x.dim()
    d = dim + nd if dim < 0 else dim
    if not 0 <= d < nd:
        raise ValueError(f"invalid argument: dim {dim} out of range for {nd}-D tensor")
    kshape = list(x.shape)
    kshape[d] = 1
    if g.numel() != x.numel() // max(x.shape[d], 1) or list(g.shape) not in (
            kshape, kshape[:d] + kshape[d + 1:]):
        raise ValueError(f"shape mismatch: gradient {list(g.shape)} for reduce output of "
                         f"{list(x.shape)} over dim {d}")
    g = dense(g)
    dx = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    L = N.load()
    xv = N.make_view(x)
    ws = _workspace(L.oxc_reduce_bwd_workspace_size(k, ctypes.byref(xv), d), x.device)
    N.check(L.oxc_reduce_bwd(k, ctypes.byref(xv), d, g.data_ptr(), dx.data_ptr(), ws.data_ptr(),
                             ws.numel(), _stream()), f"{kind} backward")
    return dx


class _Reduce(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, kind, dim, keepdim):
        ctx.save_for_backward(x)
        ctx.kind, ctx.dim = kind, dim
        return _reduce_fwd(kind, x, dim, keepdim)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        return reduce_backward(ctx.kind, x, ctx.dim, g), None, None, None


def unbroadcast(g, shape):
    """graph.rs:274-313: sums g over the axes a forward broadcast expanded to
    bring it back to `shape` -- the prepended axes first (each a keepdim sum
    over the leading axis), then the size-1 target axes -- and reshapes.  Each
    step is one device reduction, in the reference's order."""
    _require_cuda_f32("g", g)
    shape = [int(s) for s in shape]
    gs = list(g.shape)
    if len(gs) < len(shape):
        raise ValueError(f"shape mismatch: {gs} vs {shape}")
    extra = len(gs) - len(shape)
    for i, s in enumerate(shape):
        if gs[extra + i] != s and s != 1:
            raise ValueError(f"shape mismatch: {gs} vs {shape}")
    t = g
    for i in range(extra):
        t = _reduce_fwd("sum", t, i, True)
    # the reference indexes t.shape by the target position here, so with
    # prepended axes it looks at (and sums) the leading axes; kept as is
    for i, s in enumerate(shape):
        if s == 1 and t.shape[i] != 1:
            t = _reduce_fwd("sum", t, i, True)
    if list(t.shape) != shape:
        n = 1
        for s in shape:
            n *= s
        if t.numel() != n:  # Tensor::reshape's element-count check
            raise ValueError(f"shape mismatch: {list(t.shape)} vs {shape}")
        t = t.reshape(shape)
    return t


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
    """clip_grad_norm_ (python/oxitorch/optim.py:242-263) over device
    gradients, in place; returns the pre-clip total norm as a Python float.

    * norm_type 2: sqrt of the f64 sum of squares (one multi-tensor pass);
    * inf: the largest |g| of each gradient (a gradient holding a NaN gives
      NaN, as np.max does), combined in list order with Python's ``max``
      like the reference, so a NaN counts only when it comes first;
    * any other p: (sum over gradients of sum |g|**p) ** (1/p), |g|**p in
      f32 through the registry's pow, each gradient's sum in f64.

    If max_norm / (total + 1e-6) < 1, every gradient is scaled by it (an f32
    multiply, as NumPy's f32 * Python float)."""
    grads = [g for g in grads if g is not None]
    if not grads:
        return 0.0
    if norm_type == float("inf"):
        total = None
        for g in grads:
            m = float(reduce_all("max", unary_op("abs", g)).item())
            if float(reduce_all("max", cmp_op("ne", g, g)).item()) > 0.0:
                m = float("nan")
            if total is None or m > total:
                total = m
    elif norm_type == 2.0:
        total = 0.0
        for i in range(0, len(grads), 16):
            total += float(sum_squares(grads[i:i + 16]).item())
        total = total ** 0.5
    else:
        p = float(norm_type)
        acc = 0.0
        for g in grads:
            powed = binary_op("pow", unary_op("abs", g), p)
            acc += float(reduce_all("sum", powed, f64=True)[1].item())
        total = acc ** (1.0 / p)
    scale = max_norm / (total + 1e-6)
    if scale < 1.0:
        for g in grads:
            scale_(g, scale)
    return total


def clip_grad_value_(grads, clip_value):
    """clip_grad_value_ (python/oxitorch/optim.py:266-272): every gradient
    clamped in place to [-clip_value, clip_value] with np.clip's NaN rules."""
    clip_value = float(clip_value)
    if clip_value <= 0:
        raise ValueError("clip_value must be positive")
    L = N.load()
    for g in grads:
        if g is None:
            continue
        _require_cuda_f32("grad", g)
        if not g.is_contiguous():
            raise ValueError("invalid argument: clip_grad_value_ clips gradients in place, "
                             "which needs dense storage")
        N.check(L.oxc_clip_grad_value(g.data_ptr(), g.numel(), clip_value, _stream()),
                "clip_grad_value_")


def scale_(g, scale):
    """g *= scale in place (the registry's mul with a scalar operand)."""
    _require_cuda_f32("tensor", g)
    v = N.make_view(g)
    N.check(N.load().oxc_binary_scalar(2, ctypes.byref(v), float(scale), 0, ctypes.byref(v),
                                       _stream()), "scale_")
    return g


# ---- dim-0 scatter (Tensor::scatter_dim0) and its VJP ------------------------------------------

def scatter_dim0_maps(rows, indices):
    """Row maps of one scatter (host work, no device access).

    The reference resolves last-write-wins with host loops over the index
    list (crates/oxi-autograd/src/ops.rs:531-559); the same resolution here
    yields the three ``oxc_select_rows`` maps:
    ``fwd[r]`` = last writer of row r or -1 (keep ``base``);
    ``keep[r]`` = r for unwritten rows, -1 for written ones (d/dbase);
    ``win[p]`` = row of slot p when p is that row's last write, else -1
    (d/dvalues).  Indices are validated first with the reference's message
    (lib.rs:911-919); negative ids count from the end."""
    import numpy as np
    ids = [int(i) for i in indices]
    for i in ids:
        r = rows + i if i < 0 else i
        if r < 0 or r >= rows:
            raise RuntimeError(f"out of bounds: index {i} out of range for dim 0 of size {rows}")
    resolved = np.array([rows + i if i < 0 else i for i in ids], dtype=np.int64)
    fwd = np.full(rows, -1, dtype=np.int64)
    np.maximum.at(fwd, resolved, np.arange(len(ids), dtype=np.int64))  # the last slot of a row wins
    keep = np.where(fwd < 0, np.arange(rows, dtype=np.int64), -1)
    win = np.where(fwd[resolved] == np.arange(len(ids)), resolved, -1) if ids else resolved
    return fwd, keep, win


def _select_rows(a, a_rows, dmap, b, inner, device):
    """One oxc_select_rows launch over the device map ``dmap``.  The maps come
    from scatter_dim0_maps, which validated every index on the host, so no
    error flag is read back (the call stays asynchronous)."""
    n = dmap.numel()
    out = torch.empty((n, inner), dtype=torch.float32, device=device)
    N.check(N.load().oxc_select_rows(a.data_ptr() if a is not None else None, a_rows,
                                     dmap.data_ptr(), n, b.data_ptr() if b is not None else None,
                                     out.data_ptr(), inner, None, _stream()), "select_rows")
    return out


class _ScatterDim0(torch.autograd.Function):
    @staticmethod
    def forward(ctx, base, values, maps):
        import numpy as np
        rows, inner = base.shape[0], base[0].numel() if base.shape[0] else 0
        # the three maps cross to the device in one copy; the VJP reuses them
        dmaps = torch.as_tensor(np.concatenate(maps)).to(base.device)
        fwd, keep, win = dmaps[:rows], dmaps[rows:2 * rows], dmaps[2 * rows:]
        out = _select_rows(dense(values), values.shape[0], fwd, dense(base), inner,
                           base.device)
        ctx.maps, ctx.rows, ctx.inner = (keep, win), rows, inner
        ctx.base_shape, ctx.values_shape = base.shape, values.shape
        return out.reshape(base.shape)

    @staticmethod
    def backward(ctx, g):
        keep, win = ctx.maps
        g = dense(g)
        gb = gv = None
        if ctx.needs_input_grad[0]:
            gb = _select_rows(g, ctx.rows, keep, None, ctx.inner, g.device).reshape(ctx.base_shape)
        if ctx.needs_input_grad[1]:
            gv = _select_rows(g, ctx.rows, win, None, ctx.inner, g.device).reshape(ctx.values_shape)
        return gb, gv, None


def scatter_dim0(base, indices, values):
    """Tensor::scatter_dim0 (crates/oxi-tensor/src/lib.rs:895-933; Python
    ``Tensor.scatter``): a copy of ``base`` whose rows ``indices[p]`` take
    ``values[p]``, the last write winning on repeated rows.  Its VJP is the
    reference's (crates/oxi-autograd/src/ops.rs:531-598): ``base`` gets the
    upstream grad with written rows zeroed, ``values`` gets the grad of the row
    each slot finally wrote and zero for overwritten slots.  One
    ``oxc_select_rows`` launch per result."""
    _require_cuda_f32("base", base)
    _require_cuda_f32("values", values)
    if base.dim() == 0:
        raise ValueError("invalid argument: scatter_dim0 requires at least a 1-D tensor")
    want = (len(indices),) + tuple(base.shape[1:])
    if tuple(values.shape) != want:
        raise ValueError(f"shape mismatch: {list(values.shape)} vs {list(want)}")
    maps = scatter_dim0_maps(base.shape[0], indices)
    return _ScatterDim0.apply(base, values, maps)


# ---- narrow along dim 0 (Python slicing) and its zero-padding VJP ----------------------------

def _slice_bounds(rows, lo, hi):
    """layout::normalize_slice for step 1 (crates/oxi-tensor/src/layout.rs:123-145):
    negative bounds count from the end and saturate at 0, others clamp to
    ``rows``; ``hi`` is raised to ``lo`` at least."""
    def resolve(v):
        return max(0, rows + v) if v < 0 else min(v, rows)
    lo = resolve(int(lo))
    return lo, max(resolve(int(hi)), lo)


def narrow_dim0_map(rows, offset, length):
    """Row map of the narrow VJP: gx[r] = g[r - lo] for the rows the slice
    kept, -1 (zero) elsewhere.  The reference builds the same rows with
    ``concat_rows`` of zero blocks around g (crates/oxi-autograd/src/ops.rs:431-455)."""
    import numpy as np
    lo, hi = _slice_bounds(rows, offset, offset + length)
    r = np.arange(rows, dtype=np.int64)
    return np.where((r >= lo) & (r < hi), r - lo, -1), lo, hi


class _NarrowDim0(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, offset, length):
        m, lo, hi = narrow_dim0_map(x.shape[0], offset, length)
        ctx.map, ctx.kept, ctx.shape = m, hi - lo, x.shape
        # a view, as Tensor::narrow returns (lib.rs:620-636)
        return x.narrow(0, lo, hi - lo)

    @staticmethod
    def backward(ctx, g):
        inner = 1
        for d in ctx.shape[1:]:
            inner *= d
        dmap = torch.as_tensor(ctx.map).to(g.device)
        gx = _select_rows(dense(g), ctx.kept, dmap, None, inner, g.device)
        return gx.reshape(ctx.shape), None, None


def narrow_dim0(x, offset, length):
    """ops::narrow_dim0 (crates/oxi-autograd/src/ops.rs:427-442), the op behind
    integer and slice indexing on dim 0 (crates/oxi-bindings/src/lib.rs:575-620):
    rows [offset, offset + length) as a view; the VJP writes the upstream grad
    back at those rows and zeros elsewhere, one ``oxc_select_rows`` launch."""
    _require_cuda_f32("x", x)
    if x.dim() == 0:
        raise ValueError("invalid argument: dim 0 out of range for 0-D tensor")
    return _NarrowDim0.apply(x, int(offset), int(length))


# ---- index_select along any dim, gather -------------------------------------------------

def _index_list(indices, length, dim, device, flat=False):
    """Validates host indices like Tensor::index_select (lib.rs:665-675):
    negative indices count from the end, any other out-of-range index raises
    OutOfBounds (RuntimeError) before anything is copied.  Device tensors of
    indices are checked by the kernels (error flag)."""
    if isinstance(indices, torch.Tensor):
        return indices.to(device=device, dtype=torch.int64).reshape(-1).contiguous(), False
    ids = [int(i) for i in indices]
    for i in ids:
        idx = length + i if i < 0 else i
        if idx < 0 or idx >= length:
            if flat:
                raise RuntimeError(f"out of bounds: flat index {i} out of range for "
                                   f"{length} elements")
            raise RuntimeError(f"out of bounds: index {i} out of range for dim {dim} "
                               f"of size {length}")
    return torch.tensor(ids, dtype=torch.int64, device=device), True


def _norm_dim(dim, nd):
    if nd == 0:
        raise ValueError(f"invalid argument: dim {dim} out of range for 0-D tensor")
    d = dim + nd if dim < 0 else dim
    if not 0 <= d < nd:
        raise ValueError(f"invalid argument: dim {dim} out of range for {nd}-D tensor")
    return d


def _check_flag(flag):
    N.check(N.load().oxc_check_error_flag(flag.data_ptr(), _stream(), -1), "index_select")


def index_select_fwd(x, dim, ids, checked=True):
    """out (dense) = x.index_select(dim, ids) for a device int64 ids tensor;
    one oxc_index_select launch over x's strides."""
    d = _norm_dim(dim, x.dim())
    shape = list(x.shape)
    shape[d] = ids.numel()
    out = torch.empty(shape, dtype=torch.float32, device=x.device)
    flag = torch.zeros(4, dtype=torch.int32, device=x.device)
    N.check(N.load().oxc_index_select(ctypes.byref(N.make_view(x)), d, ids.data_ptr(),
                                      ids.numel(), out.data_ptr(), flag.data_ptr(), _stream()),
            "index_select")
    if not checked:
        _check_flag(flag)
    return out


def index_select_bwd(g, ids, shape, dim):
    """scatter_index_select (crates/oxi-autograd/src/ops.rs:741-769): the
    gradient of x (dense, `shape`) from g, summing duplicate indices in
    position order."""
    d = _norm_dim(dim, len(shape))
    g = dense(g)
    gx = torch.empty(tuple(shape), dtype=torch.float32, device=g.device)
    dims = (ctypes.c_int64 * max(len(shape), 1))(*[int(v) for v in shape])
    flag = torch.zeros(4, dtype=torch.int32, device=g.device)
    L = N.load()
    ws = _workspace(L.oxc_index_select_bwd_workspace_size(dims, len(shape), d, ids.numel()),
                    g.device)
    N.check(L.oxc_index_select_bwd(g.data_ptr(), ids.data_ptr(), ids.numel(), dims, len(shape), d,
                                   gx.data_ptr(), flag.data_ptr(), ws.data_ptr(), ws.numel(),
                                   _stream()), "index_select backward")
    return gx


class _IndexSelect(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim, ids, checked):
        ctx.save_for_backward(ids)
        ctx.dim, ctx.shape = dim, tuple(x.shape)
        return index_select_fwd(x, dim, ids, checked)

    @staticmethod
    def backward(ctx, g):
        (ids,) = ctx.saved_tensors
        return index_select_bwd(g, ids, ctx.shape, ctx.dim), None, None, None


def index_select(x, dim, indices):
    """Tensor.index_select(dim, indices) (crates/oxi-bindings/src/lib.rs, the
    ops::index_select node of crates/oxi-autograd/src/ops.rs:498-517): any
    dim, any strides of x; indices a list of ints (validated here, like the
    reference) or a device int64 tensor (validated by the kernel's error
    flag).  Differentiable: duplicate indices accumulate."""
    _require_cuda_f32("x", x)
    d = _norm_dim(dim, x.dim())
    ids, checked = _index_list(indices, x.shape[d], d, x.device)
    return _IndexSelect.apply(x, d, ids, checked)


def gather(x, indices):
    """Tensor.gather(indices) (crates/oxi-bindings/src/lib.rs:645-648): the
    differentiable index_select along dim 0."""
    return index_select(x, 0, indices)


def gather_dim0(x, indices):
    """Tensor::gather_dim0 (crates/oxi-tensor/src/lib.rs:857-886): rows
    x[indices[i], ...] (no graph node); a 0-D x is InvalidArgument."""
    _require_cuda_f32("x", x)
    if x.dim() == 0:
        raise ValueError("invalid argument: gather_dim0 requires at least a 1-D tensor")
    ids, checked = _index_list(indices, x.shape[0], 0, x.device)
    shape = [ids.numel()] + list(x.shape[1:])
    out = torch.empty(shape, dtype=torch.float32, device=x.device)
    flag = torch.zeros(4, dtype=torch.int32, device=x.device)
    N.check(N.load().oxc_gather_dim0(ctypes.byref(N.make_view(x)), ids.data_ptr(), ids.numel(),
                                     out.data_ptr(), flag.data_ptr(), _stream()), "gather_dim0")
    if not checked:
        _check_flag(flag)
    return out


def gather_flat(x, indices):
    """Tensor::gather_flat (crates/oxi-tensor/src/lib.rs:834-850): elements at
    flat row-major indices of x, as a 1-D tensor (no graph node)."""
    _require_cuda_f32("x", x)
    flat = dense(x).reshape(-1)
    ids, checked = _index_list(indices, flat.numel(), 0, x.device, flat=True)
    return index_select_fwd(flat, 0, ids, checked)


# ---- masked_select (boolean-mask indexing) and its VJP ---------------------------------------

_MS_CHUNK = 4096  # grid points per count chunk of oxc_masked_select_count


def _ms_count(xv, mv, n, by_mask, device):
    """Pick offsets per chunk in a workspace; returns (workspace, total picks).
    Reading the total waits for the device: the output's length depends on it."""
    L = N.load()
    ws = torch.empty(max(1, L.oxc_masked_select_workspace_size(n) // 8), dtype=torch.int64,
                     device=device)
    N.check(L.oxc_masked_select_count(None if xv is None else ctypes.byref(xv), ctypes.byref(mv),
                                      by_mask, ws.data_ptr(), ws.numel() * 8, _stream()),
            "masked_select")
    return ws, int(ws[(n + _MS_CHUNK - 1) // _MS_CHUNK].item())


class _MaskedSelect(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, mask, shape):
        xe, me = x.expand(shape), mask.expand(shape)
        n = xe.numel()
        xv, mv = N.make_view(xe), N.make_view(me)
        ws, total = _ms_count(xv, mv, n, 0, x.device)
        out = torch.empty(total, dtype=torch.float32, device=x.device)
        if total:
            N.check(N.load().oxc_masked_select_fwd(ctypes.byref(xv), ctypes.byref(mv),
                                                   ws.data_ptr(), out.data_ptr(), _stream()),
                    "masked_select")
        ctx.save_for_backward(mask)
        ctx.shape, ctx.x_shape = tuple(shape), tuple(x.shape)
        return out

    @staticmethod
    def backward(ctx, g):
        (mask,) = ctx.saved_tensors
        shape, x_shape = ctx.shape, ctx.x_shape
        me = mask.expand(shape)
        mv = N.make_view(me)
        n = me.numel()
        ws, picks = _ms_count(None, mv, n, 1, g.device)
        g = dense(g)
        if picks != g.numel():
            # the reference reads past the end of g here (a picked NaN of x
            # left the forward shorter than the mask's picks)
            raise RuntimeError(f"out of bounds: masked_select grad has {g.numel()} elements "
                               f"for {picks} picks")
        gfull = torch.empty(shape, dtype=torch.float32, device=g.device)
        if n:
            N.check(N.load().oxc_masked_select_bwd(g.data_ptr() if g.numel() else None, g.numel(),
                                                   ctypes.byref(mv), ws.data_ptr(), gfull.data_ptr(),
                                                   _stream()), "masked_select backward")
        aligned = (1,) * (len(shape) - len(x_shape)) + x_shape
        if aligned == shape:
            return gfull.reshape(x_shape), None, None
        gx = torch.empty(x_shape, dtype=torch.float32, device=g.device)
        gs = (ctypes.c_int64 * max(1, len(shape)))(*shape)
        xs = (ctypes.c_int64 * max(1, len(shape)))(*aligned)
        N.check(N.load().oxc_broadcast_fold(gfull.data_ptr(), gs, xs, len(shape), gx.data_ptr(),
                                            _stream()), "masked_select backward")
        return gx, None, None


def masked_select(x, mask):
    """Tensor::masked_select (crates/oxi-tensor/src/lib.rs:939-960): the
    elements of ``x`` where the broadcast ``mask`` is nonzero, as a 1-D tensor
    in row-major order of the broadcast grid (a picked NaN of ``x`` is
    dropped, as the reference's NaN sentinel drops it).  The VJP is the
    reference's (crates/oxi-autograd/src/ops.rs:610-665): each grad element goes
    back to the x element it was picked from, elements picked more than once
    through broadcasting accumulating in grid order.  The mask is not
    differentiated."""
    _require_cuda_f32("x", x)
    _require_cuda_f32("mask", mask)
    shape = _broadcast_shape(tuple(x.shape), tuple(mask.shape))
    if len(shape) > N.MAX_DIMS:
        raise NotImplementedError(f"not implemented: tensors of rank {len(shape)} > {N.MAX_DIMS}")
    return _MaskedSelect.apply(x, mask.detach(), shape)


# The Python surface's name for the dim-0 scatter (``Tensor.scatter(indices,
# values)``, crates/oxi-bindings/src/lib.rs:650), with the base tensor first.
scatter = scatter_dim0
