"""Device-side mirror of oxitorch's ``F.*`` layer functions.

Same names, argument meaning and error behaviour as
``python/oxitorch/nn/functional.py`` for the memory-bound layers; each call is
one fused CUDA kernel through liboxicuda.so, and its VJP is one fused kernel
(plus a deterministic column-sum finisher for weight gradients).  Tensors are
torch CUDA float32 tensors: torch supplies device memory, the stream and the
autograd graph bookkeeping (``torch.autograd.Function``); all arithmetic on
the path is ours.

``grad_mode`` selects the backward semantics of the norms:
``"ref"`` (default) reproduces the reference graph, where ``rsqrt`` is
detached (crates/oxi-bindings/src/lib.rs:682-697); ``"exact"`` is the full
mathematical gradient.
"""

from __future__ import annotations

import torch

import ctypes

from . import _native as N

_MODES = {"ref": N.GRAD_REF, "exact": N.GRAD_EXACT}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda_f32(name, t):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch CUDA tensor")
    if not t.is_cuda:
        raise ValueError(f"invalid argument: {name} must live on a CUDA device "
                         "(oxitorch_b200 has no CPU path)")
    if t.dtype != torch.float32:
        raise ValueError(f"invalid argument: {name} must be float32, got {t.dtype}")


def _rows_cols(x):
    if x.dim() == 0:
        raise ValueError("invalid argument: dim -1 out of range for 0-D tensor")
    cols = x.shape[-1]
    rows = x.numel() // cols if cols else 0
    return rows, cols


def dense(t):
    """t itself when it is dense row-major, else a dense copy made on the
    device by oxc_contiguous (the reference's Tensor::contiguous,
    crates/oxi-tensor/src/lib.rs:220-240): strided and transposed views reach
    the fused row kernels through one copy kernel of this library."""
    if t.is_contiguous():
        return t
    _require_cuda_f32("tensor", t)
    out = torch.empty(t.shape, dtype=torch.float32, device=t.device)
    N.check(N.load().oxc_contiguous(ctypes.byref(N.make_view(t)), ctypes.byref(N.make_view(out)),
                                    _stream()), "contiguous")
    return out


def _row_major(name, t):
    """The fused row kernels read dense rows: a strided view is copied first
    (the reference's compositions accept any view and produce dense results)."""
    return dense(t)


def _vector(name, t, cols):
    """A [cols] parameter; a broadcast view with zero row strides is accepted
    and read through its first row (no copy)."""
    if t.dim() >= 1 and t.shape[-1] == cols and all(s == 0 for s in t.stride()[:-1]):
        t = t.reshape(-1)[:cols] if t.dim() == 1 else t.select(0, 0) if t.dim() == 2 else t
    if t.dim() != 1 or t.shape[0] != cols:
        raise ValueError(f"shape mismatch: {list(t.shape)} vs [{cols}]")
    if t.stride(0) != 1:
        raise ValueError(f"invalid argument: {name} must be contiguous")
    return t


def _workspace(nbytes, device):
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


# ---- RMSNorm ---------------------------------------------------------------------

def rms_norm_fwd(x, weight, eps=1e-6):
    """Returns (y, rstd) for x [..., cols]."""
    _require_cuda_f32("x", x)
    _require_cuda_f32("weight", weight)
    x = _row_major("x", x)
    rows, cols = _rows_cols(x)
    weight = _vector("weight", weight, cols)
    y = torch.empty_like(x)
    rstd = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    L = N.load()
    N.check(L.oxc_rms_norm_fwd(x.data_ptr(), weight.data_ptr(), y.data_ptr(), rstd.data_ptr(),
                               rows, cols, float(eps), _stream()), "rms_norm")
    return y, rstd


def rms_norm_bwd(x, weight, rstd, dy, grad_mode="ref"):
    """Returns (dx, dweight)."""
    x = _row_major("x", x)
    rows, cols = _rows_cols(x)
    weight = _vector("weight", weight, cols)
    dy = _row_major("dy", dy)
    dx = torch.empty_like(x)
    dw = torch.empty(cols, dtype=torch.float32, device=x.device)
    L = N.load()
    ws_bytes = L.oxc_rms_norm_bwd_workspace_size(rows, cols)
    ws = _workspace(ws_bytes, x.device)
    N.check(L.oxc_rms_norm_bwd(x.data_ptr(), weight.data_ptr(), rstd.data_ptr(), dy.data_ptr(),
                               dx.data_ptr(), dw.data_ptr(), rows, cols, _MODES[grad_mode],
                               ws.data_ptr(), ws.numel(), _stream()), "rms_norm backward")
    return dx, dw


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps, grad_mode):
        x = dense(x)
        y, rstd = rms_norm_fwd(x, weight, eps)
        ctx.save_for_backward(x, weight, rstd)
        ctx.grad_mode = grad_mode
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, rstd = ctx.saved_tensors
        dx, dw = rms_norm_bwd(x, weight, rstd, dense(dy), ctx.grad_mode)
        return dx, dw.reshape(weight.shape), None, None


def rms_norm(x, weight, eps=1e-6, grad_mode="ref"):
    """F.rms_norm (python/oxitorch/nn/functional.py:236-240): x / rms(x) * weight."""
    return _RMSNorm.apply(x, weight, eps, grad_mode)


# ---- LayerNorm (+ GELU) --------------------------------------------------------------

def layer_norm_fwd(x, weight, bias, eps=1e-5, act=N.ACT_NONE):
    """Returns (y, mean, rstd); y = act(layer_norm(x))."""
    _require_cuda_f32("x", x)
    _require_cuda_f32("weight", weight)
    _require_cuda_f32("bias", bias)
    x = _row_major("x", x)
    rows, cols = _rows_cols(x)
    weight = _vector("weight", weight, cols)
    bias = _vector("bias", bias, cols)
    y = torch.empty_like(x)
    mean = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    rstd = torch.empty_like(mean)
    L = N.load()
    N.check(L.oxc_layer_norm_fwd(x.data_ptr(), weight.data_ptr(), bias.data_ptr(), y.data_ptr(),
                                 mean.data_ptr(), rstd.data_ptr(), rows, cols, float(eps), act,
                                 _stream()), "layer_norm")
    return y, mean, rstd


def layer_norm_bwd(x, weight, bias, mean, rstd, dy, act=N.ACT_NONE, grad_mode="ref"):
    """Returns (dx, dweight, dbias)."""
    x = _row_major("x", x)
    rows, cols = _rows_cols(x)
    weight = _vector("weight", weight, cols)
    bias = _vector("bias", bias, cols)
    dy = _row_major("dy", dy)
    dx = torch.empty_like(x)
    dw = torch.empty(cols, dtype=torch.float32, device=x.device)
    db = torch.empty_like(dw)
    L = N.load()
    ws = _workspace(L.oxc_layer_norm_bwd_workspace_size(rows, cols), x.device)
    N.check(L.oxc_layer_norm_bwd(x.data_ptr(), weight.data_ptr(), bias.data_ptr(), mean.data_ptr(),
                                 rstd.data_ptr(), dy.data_ptr(), dx.data_ptr(), dw.data_ptr(),
                                 db.data_ptr(), rows, cols, act, _MODES[grad_mode], ws.data_ptr(),
                                 ws.numel(), _stream()), "layer_norm backward")
    return dx, dw, db


class _LayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps, act, grad_mode):
        x = dense(x)
        y, mean, rstd = layer_norm_fwd(x, weight, bias, eps, act)
        ctx.save_for_backward(x, weight, bias, mean, rstd)
        ctx.act, ctx.grad_mode = act, grad_mode
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, bias, mean, rstd = ctx.saved_tensors
        dx, dw, db = layer_norm_bwd(x, weight, bias, mean, rstd, dense(dy), ctx.act,
                                    ctx.grad_mode)
        return dx, dw.reshape(weight.shape), db.reshape(bias.shape), None, None, None


def layer_norm(x, weight, bias, eps=1e-5, grad_mode="ref"):
    """F.layer_norm (functional.py:227-233) over the last dim with affine weight/bias."""
    return _LayerNorm.apply(x, weight, bias, eps, N.ACT_NONE, grad_mode)


def layer_norm_gelu(x, weight, bias, eps=1e-5, grad_mode="ref"):
    """F.gelu(F.layer_norm(x, weight, bias, eps)) as one fused kernel each way
    (functional.py:227-233 then 194-199)."""
    return _LayerNorm.apply(x, weight, bias, eps, N.ACT_GELU_TANH, grad_mode)


# ---- GELU ------------------------------------------------------------------------------

def gelu_fwd(x):
    """y = gelu(x) (dense, x's shape) for any view x."""
    _require_cuda_f32("x", x)
    x = dense(x)
    y = torch.empty_like(x)
    N.check(N.load().oxc_gelu_fwd(x.data_ptr(), y.data_ptr(), x.numel(), _stream()), "gelu")
    return y


def gelu_bwd(x, dy):
    """dx = dy * gelu'(x), dense."""
    x, dy = dense(x), dense(dy)
    if dy.shape != x.shape:
        raise ValueError(f"shape mismatch: {list(dy.shape)} vs {list(x.shape)}")
    dx = torch.empty_like(x)
    N.check(N.load().oxc_gelu_bwd(x.data_ptr(), dy.data_ptr(), dx.data_ptr(), x.numel(),
                                  _stream()), "gelu backward")
    return dx


class _Gelu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        x = dense(x)
        ctx.save_for_backward(x)
        return gelu_fwd(x)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        return gelu_bwd(x, dy)


def gelu(x):
    """F.gelu (functional.py:194-199): 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))),
    one fused kernel each way.  After a LayerNorm, ``layer_norm_gelu`` fuses both."""
    return _Gelu.apply(x)


# ---- softmax / log_softmax ----------------------------------------------------------

def _softmax_dim(dim, x):
    if x.dim() == 0:
        raise ValueError(f"invalid argument: dim {dim} out of range for 0-D tensor")
    d = dim + x.dim() if dim < 0 else dim
    if not 0 <= d < x.dim():
        raise ValueError(f"invalid argument: dim {dim} out of range for {x.dim()}-D tensor")
    return d


def softmax_fwd(x, log=False, dim=-1):
    """y (dense, x's shape) = softmax or log_softmax of x over `dim`; x may be
    any strided view.  Dense rows along the last dim run the row kernels,
    other layouts the strided-row or column kernels (oxc_softmax_dim_fwd)."""
    _require_cuda_f32("x", x)
    d = _softmax_dim(dim, x)
    y = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    N.check(N.load().oxc_softmax_dim_fwd(ctypes.byref(N.make_view(x)), d, int(log), y.data_ptr(),
                                         _stream()), "softmax")
    return y


def softmax_bwd(y, dy, log=False, dim=-1):
    """dx (dense) from the forward output y (dense) and dy (any view)."""
    d = _softmax_dim(dim, y)
    dx = torch.empty(y.shape, dtype=torch.float32, device=y.device)
    N.check(N.load().oxc_softmax_dim_bwd(y.data_ptr(), ctypes.byref(N.make_view(dy)), d, int(log),
                                         dx.data_ptr(), _stream()), "softmax backward")
    return dx


class _Softmax(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, log, dim):
        y = softmax_fwd(x, log, dim)
        ctx.save_for_backward(y)
        ctx.log, ctx.dim = log, dim
        return y

    @staticmethod
    def backward(ctx, dy):
        (y,) = ctx.saved_tensors
        return softmax_bwd(y, dy, ctx.log, ctx.dim), None, None


def softmax(x, dim=-1):
    """F.softmax (functional.py:211-215), numerically stable, over any dim."""
    return _Softmax.apply(x, False, dim)


def log_softmax(x, dim=-1):
    """F.log_softmax (functional.py:218-222) over any dim."""
    return _Softmax.apply(x, True, dim)


# ---- cross-entropy ----------------------------------------------------------------------

def _targets_tensor(targets, n, classes, device):
    """The reference takes a Python list and indexes a numpy one-hot with it
    (functional.py:285-289): the same length check and numpy's index rules."""
    if isinstance(targets, torch.Tensor):
        t = targets.to(device=device, dtype=torch.int64).reshape(-1)
        if t.numel() != n:
            raise ValueError(f"{t.numel()} targets for batch of {n}")
        return t.contiguous()
    if len(targets) != n:
        raise ValueError(f"{len(targets)} targets for batch of {n}")
    for v in targets:
        if not -classes <= int(v) < classes:
            raise IndexError(f"index {int(v)} is out of bounds for axis 1 with size {classes}")
    return torch.tensor([int(v) for v in targets], dtype=torch.int64, device=device)


def cross_entropy_fwd(logits, targets, total_rows=None):
    """Returns (loss[1], row_max, row_sum, row_nll)."""
    _require_cuda_f32("logits", logits)
    logits = _row_major("logits", logits)
    if logits.dim() != 2:
        raise ValueError(f"invalid argument: cross_entropy expects [n, classes] logits, got {list(logits.shape)}")
    n, classes = logits.shape
    t = _targets_tensor(targets, n, classes, logits.device)
    loss = torch.empty(1, dtype=torch.float32, device=logits.device)
    row_max = torch.empty(n, dtype=torch.float32, device=logits.device)
    row_sum = torch.empty_like(row_max)
    row_nll = torch.empty_like(row_max)
    flag = torch.zeros(4, dtype=torch.int32, device=logits.device)
    L = N.load()
    N.check(L.oxc_cross_entropy_fwd(logits.data_ptr(), t.data_ptr(), loss.data_ptr(),
                                    row_max.data_ptr(), row_sum.data_ptr(), row_nll.data_ptr(), n,
                                    classes, int(total_rows or n), flag.data_ptr(), _stream()),
            "cross_entropy")
    return loss, row_max, row_sum, row_nll, t, flag


def cross_entropy_bwd(logits, t, row_max, row_sum, grad_loss=None, total_rows=None):
    n, classes = logits.shape
    dlogits = torch.empty_like(logits)
    N.check(N.load().oxc_cross_entropy_bwd(
        logits.data_ptr(), t.data_ptr(), row_max.data_ptr(), row_sum.data_ptr(),
        None if grad_loss is None else grad_loss.data_ptr(), dlogits.data_ptr(), n, classes,
        int(total_rows or n), _stream()), "cross_entropy backward")
    return dlogits


class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets):
        loss, row_max, row_sum, _, t, _ = cross_entropy_fwd(logits, targets)
        ctx.save_for_backward(logits, t, row_max, row_sum)
        return loss.reshape(())

    @staticmethod
    def backward(ctx, g):
        logits, t, row_max, row_sum = ctx.saved_tensors
        g = g.reshape(1).to(torch.float32).contiguous()
        return cross_entropy_bwd(logits, t, row_max, row_sum, g), None


def cross_entropy(logits, targets):
    """F.cross_entropy (functional.py:277-293): mean over the batch of
    -log_softmax(logits)[i, targets[i]]."""
    return _CrossEntropy.apply(logits, targets)


# ---- embedding ----------------------------------------------------------------------------

def _ids_tensor(indices, vocab, device):
    """The reference validates every id before copying (lib.rs:665-675):
    negative ids count from the end, anything else out of range raises."""
    if isinstance(indices, torch.Tensor):
        return indices.to(device=device, dtype=torch.int64).reshape(-1).contiguous()
    ids = [int(i) for i in indices]
    for i in ids:
        idx = vocab + i if i < 0 else i
        if idx < 0 or idx >= vocab:
            raise RuntimeError(f"out of bounds: index {i} out of range for dim 0 of size {vocab}")
    return torch.tensor(ids, dtype=torch.int64, device=device)


def embedding_fwd(ids, weight, vocab_offset=0, vocab_total=None):
    """out [n, cols] = weight[ids]; weight may be a vocab shard."""
    _require_cuda_f32("weight", weight)
    weight = _row_major("weight", weight)
    rows, cols = weight.shape
    total = int(vocab_total or rows)
    out = torch.empty(ids.numel(), cols, dtype=torch.float32, device=weight.device)
    flag = torch.zeros(4, dtype=torch.int32, device=weight.device)
    N.check(N.load().oxc_embedding_fwd(weight.data_ptr(), ids.data_ptr(), out.data_ptr(),
                                       ids.numel(), total, int(vocab_offset), rows, cols,
                                       flag.data_ptr(), _stream()), "embedding")
    return out, flag


def embedding_bwd(ids, dout, rows, vocab_offset=0, vocab_total=None):
    """dtable [rows, cols] for dout [n, cols]."""
    dout = _row_major("dout", dout)
    n, cols = ids.numel(), dout.shape[-1]
    total = int(vocab_total or rows)
    dtable = torch.empty(rows, cols, dtype=torch.float32, device=dout.device)
    flag = torch.zeros(4, dtype=torch.int32, device=dout.device)
    L = N.load()
    ws = _workspace(L.oxc_embedding_bwd_workspace_size(n, rows, cols), dout.device)
    N.check(L.oxc_embedding_bwd(dout.data_ptr(), ids.data_ptr(), dtable.data_ptr(), n, total,
                                int(vocab_offset), rows, cols, flag.data_ptr(), ws.data_ptr(),
                                ws.numel(), _stream()), "embedding backward")
    return dtable, flag


class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight):
        out, _ = embedding_fwd(ids, weight)
        ctx.save_for_backward(ids)
        ctx.rows = weight.shape[0]
        return out

    @staticmethod
    def backward(ctx, dout):
        (ids,) = ctx.saved_tensors
        dtable, _ = embedding_bwd(ids, dense(dout), ctx.rows)
        return None, dtable


def embedding(indices, weight):
    """F.embedding (functional.py:245-247): weight.index_select(0, indices);
    indices is a flat list of ints (or an int tensor); the output is
    [len(indices), dim]."""
    _require_cuda_f32("weight", weight)
    ids = _ids_tensor(indices, weight.shape[0], weight.device)
    return _Embedding.apply(ids, weight)


# ---- SiLU / SwiGLU -----------------------------------------------------------------------

def _as2d(name, t):
    _require_cuda_f32(name, t)
    if t.dim() == 1:
        return t.reshape(1, -1)
    if t.dim() != 2:
        t = t.reshape(-1, t.shape[-1])
    return t


def swiglu_fwd(gate, up=None, row_stats=False):
    """h = silu(gate) * up (silu(gate) if up is None) for 2-D views of any
    strides; with row_stats also the dim-1 sum, max and argmax of h."""
    g = _as2d("gate", gate)
    u = None if up is None else _as2d("up", up)
    R, C = g.shape
    h = torch.empty(R, C, dtype=torch.float32, device=g.device)
    stats = [torch.empty(R, dtype=torch.float32, device=g.device) for _ in range(3)] if row_stats else [None] * 3
    N.check(N.load().oxc_swiglu_fwd(ctypes.byref(N.make_view(g)),
                                    None if u is None else ctypes.byref(N.make_view(u)),
                                    h.data_ptr(), *[None if t is None else t.data_ptr() for t in stats],
                                    _stream()), "swiglu")
    return (h, *stats) if row_stats else h


def swiglu_bwd(gate, up, dh, sumsq=False):
    """(dgate, dup[, sum of squares of both as a 0-d f64 tensor])."""
    g = _as2d("gate", gate)
    u = None if up is None else _as2d("up", up)
    d = _as2d("dh", dh)
    R, C = g.shape
    dg = torch.empty(R, C, dtype=torch.float32, device=g.device)
    du = None if u is None else torch.empty(R, C, dtype=torch.float32, device=g.device)
    L = N.load()
    sq = torch.empty((), dtype=torch.float64, device=g.device) if sumsq else None
    ws = _workspace(L.oxc_swiglu_bwd_workspace_size(R, C) if sumsq else 0, g.device)
    N.check(L.oxc_swiglu_bwd(ctypes.byref(N.make_view(g)),
                             None if u is None else ctypes.byref(N.make_view(u)),
                             ctypes.byref(N.make_view(d)), dg.data_ptr(),
                             None if du is None else du.data_ptr(),
                             None if sq is None else sq.data_ptr(), ws.data_ptr(), ws.numel(),
                             _stream()), "swiglu backward")
    return (dg, du, sq) if sumsq else (dg, du)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gate, up):
        ctx.save_for_backward(gate, up)
        ctx.shape = gate.shape
        h = swiglu_fwd(gate, up)
        return h.reshape(gate.shape)

    @staticmethod
    def backward(ctx, dh):
        gate, up = ctx.saved_tensors
        dg, du = swiglu_bwd(gate, up, dh)
        return dg.reshape(ctx.shape), du.reshape(ctx.shape)


class _SiLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.save_for_backward(x)
        return swiglu_fwd(x).reshape(x.shape)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        dg, _ = swiglu_bwd(x, None, dy)
        return dg.reshape(x.shape)


def silu(x):
    """F.silu (functional.py:202-204): x * sigmoid(x)."""
    return _SiLU.apply(x)


def swiglu(gate, up):
    """silu(gate) * up, the decoder-MLP gate (composed by callers of F.silu)."""
    return _SwiGLU.apply(gate, up)
