"""Softmax / log_softmax over any dim, the fused row layers on strided inputs,
and index_select along any dim with its duplicate-accumulating VJP, on the
device against the oracle.

Tolerances (tests/parity.py): softmax as in test_gpu_softmax_ce.py (rtol
1e-5 / atol 1e-6 plus the reference's summation-order and exp/log libm
budgets and the max node's exact-zero VJP term); index_select and its VJP
bit-exact, except table slices summed from more than 128 occurrences in the
wide-slice pipeline (rtol 1e-4, duplicate-id accumulation).
"""

import numpy as np
import pytest

from parity import ATOL, RTOL, RTOL_BIG, assert_bitexact, assert_close, max_vjp_budget, \
    reference_budget

pytestmark = pytest.mark.gpu


def _dev(a, grad=False):
    import torch
    return torch.from_numpy(np.array(a, order="C", copy=True)).cuda().requires_grad_(grad)


def _host(t):
    return t.detach().cpu().numpy()


def _layout(a, layout):
    """A device view with a's values in one of several memory layouts."""
    import torch
    if layout == "dense":
        return _dev(a)
    if layout == "transposed":  # reversed dim order in memory
        return _dev(np.ascontiguousarray(a.transpose(tuple(range(a.ndim))[::-1]))).permute(
            *range(a.ndim)[::-1])
    if layout == "padded":      # last dim padded in memory (rows of a wider buffer)
        buf = torch.zeros(a.shape[:-1] + (a.shape[-1] + 5,), device="cuda")
        buf[..., :a.shape[-1]] = _dev(a)
        return buf[..., :a.shape[-1]]
    raise ValueError(layout)


# ---- softmax / log_softmax over any dim ---------------------------------------------------

SOFTMAX_CASES = [
    ((64, 300), 0), ((64, 300), 1), ((6, 50, 40), 0), ((6, 50, 40), 1), ((6, 50, 40), -1),
    ((3000, 8), 0), ((2, 40000), 0), ((5, 1, 7), 1), ((1, 9), 0), ((33, 4, 2, 5), 2),
]


def _oracle_softmax(oracle, x, dy, dim, log):
    def run():
        xt = oracle.from_numpy(x, True)
        y = (oracle.log_softmax if log else oracle.softmax)(xt, dim)
        y.backward(dy)
        return y.numpy(), xt.grad.numpy()
    ref, budget = reference_budget(oracle, run, libm=("exp", "log"))
    mv = max_vjp_budget(oracle, run)
    return ref, [b + m for b, m in zip(budget, mv)]


@pytest.mark.parametrize("log", [False, True])
@pytest.mark.parametrize("shape,dim", SOFTMAX_CASES)
def test_softmax_any_dim_vs_oracle(oracle, shape, dim, log):
    """F.softmax / F.log_softmax(x, dim) (functional.py:211-222) for every dim
    of 2-, 3- and 4-D inputs: the forward and its VJP through autograd."""
    from oxitorch_b200 import functional as F
    rng = np.random.default_rng(sum(shape) + 7 * dim + log)
    x = (rng.standard_normal(shape, dtype=np.float32) * np.float32(2)).astype(np.float32)
    x[rng.random(shape) < 0.01] = 20.0
    dy = rng.standard_normal(shape, dtype=np.float32)
    (y_ref, dx_ref), (by, bdx) = _oracle_softmax(oracle, x, dy, dim, log)
    xg = _dev(x, True)
    fn = F.log_softmax if log else F.softmax
    y = fn(xg, dim)
    y.backward(_dev(dy))
    rtol = RTOL if shape[dim] < 32768 else RTOL_BIG
    assert_close(_host(y), y_ref, rtol=rtol, atol=ATOL + by, what="y")
    assert_close(_host(xg.grad), dx_ref, rtol=rtol, atol=ATOL + bdx, what="dx")


@pytest.mark.parametrize("layout", ["transposed", "padded"])
@pytest.mark.parametrize("dim", [0, 1, -1])
@pytest.mark.parametrize("log", [False, True])
def test_softmax_strided_views_match_dense(oracle, layout, dim, log):
    """Strided x and strided upstream grads give the dense results: the
    strided-row kernel (the reduced dim not dense in memory), the column kernel
    reading a transposed view, and padded rows; checked against the oracle."""
    from oxitorch_b200 import functional as F
    shape = (48, 6, 70)
    rng = np.random.default_rng(11 + dim + 2 * log)
    x = rng.standard_normal(shape, dtype=np.float32) * np.float32(3)
    dy = rng.standard_normal(shape, dtype=np.float32)
    (y_ref, dx_ref), (by, bdx) = _oracle_softmax(oracle, x, dy, dim, log)
    xv = _layout(x, layout).requires_grad_()
    assert not xv.is_contiguous()
    fn = F.log_softmax if log else F.softmax
    y = fn(xv, dim)
    y.backward(_layout(dy, layout))
    assert y.is_contiguous()
    assert_close(_host(y), y_ref, atol=ATOL + by, what=f"y ({layout})")
    assert_close(_host(xv.grad), dx_ref, atol=ATOL + bdx, what=f"dx ({layout})")
    xd = _dev(x, True)
    yd = fn(xd, dim)
    yd.backward(_dev(dy))
    if layout == "padded" and dim in (-1, 2):
        # padded rows along the last dim: the same row kernel as dense rows
        assert_bitexact(_host(y), _host(yd), "y vs dense")


def test_softmax_dim_errors_match_reference():
    import torch
    from oxitorch_b200 import functional as F
    x = torch.zeros(3, 4, device="cuda")
    with pytest.raises(ValueError, match="dim 2 out of range for 2-D tensor"):
        F.softmax(x, 2)
    with pytest.raises(ValueError, match="zero-length dim"):
        F.log_softmax(torch.zeros(3, 0, device="cuda"), 1)
    assert F.softmax(torch.zeros(0, 4, device="cuda"), 1).shape == (0, 4)


# ---- fused row layers on strided inputs --------------------------------------------------

@pytest.mark.parametrize("layout", ["transposed", "padded"])
def test_norms_accept_strided_x(oracle, layout):
    """F.rms_norm / F.layer_norm(+GELU) of a transposed or padded x: one
    device copy to dense rows (oxc_contiguous), then the fused kernels; the
    results are bit-identical to the dense input's and match the oracle."""
    import test_gpu_norms as TN
    from oxitorch_b200 import functional as F
    rng = np.random.default_rng(5)
    m, n = 96, 1024
    x = rng.standard_normal((m, n), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    b = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    dy = rng.standard_normal((m, n), dtype=np.float32)
    for kind in ("rms", "ln"):
        outs = []
        for lay in (layout, "dense"):
            xv = _layout(x, lay).requires_grad_()
            wv, bv = _dev(w, True), _dev(b, True)
            y = F.rms_norm(xv, wv, 1e-6) if kind == "rms" else F.layer_norm_gelu(xv, wv, bv, 1e-5)
            y.backward(_layout(dy, lay))
            outs.append([_host(y), _host(xv.grad), _host(wv.grad)] +
                        ([_host(bv.grad)] if kind == "ln" else []))
        for got, want, name in zip(outs[0], outs[1], ("y", "dx", "dw", "db")):
            assert_bitexact(got, want, f"{kind} {name} strided vs dense")
        if kind == "rms":
            ref = TN._oracle_rms(oracle, x, w, dy)
            y_, rstd = F.rms_norm_fwd(_dev(x), _dev(w), 1e-6)
            TN._check_rms(x, w, dy, outs[0][0], outs[0][1], outs[0][2], ref, _host(rstd))
        else:
            ref = TN._oracle_ln(oracle, x, w, b, dy, True)
            got = TN._ln_dev(x, w, b, dy, True)
            TN._check_ln(x, w, dy, (outs[0][0], outs[0][1], outs[0][2], outs[0][3]) + got[4:],
                         ref, True)


# ---- index_select along any dim ------------------------------------------------------------

INDEX_CASES = [
    ((5, 7), 0, [4, -1, 0, 4]),                 # rows, negative and repeated ids
    ((5, 7), 1, [6, -7, 3, 3, 3]),              # columns (inner 1)
    ((5, 7), -1, []),                           # no ids
    ((4, 6, 300), 1, "dup"),                    # wide slices (>= 128 floats), outer 4
    ((4, 6, 9), -1, "dup"),                     # last dim of a 3-D tensor
    ((3, 2000, 2), 1, "hot"),                   # narrow slices, ids occurring > 128 times
    ((2, 50, 256), 1, "hot"),                   # wide slices, hot ids in 128-position pieces
    ((64, 4096), 0, "dup"),                     # embedding-shaped, float4 copies
    ((9, 3, 4, 5), 2, [3, 0, -4, 3]),           # 4-D, middle dim
]


def _ids(spec, length, rng):
    if spec == "dup":
        return [int(i) for i in rng.integers(-length, length, 3 * length)]
    if spec == "hot":
        return [int(i) for i in np.minimum(rng.zipf(1.3, 4000) - 1, length - 1)] + [-1, 0]
    return list(spec)


@pytest.mark.parametrize("layout", ["dense", "transposed"])
@pytest.mark.parametrize("shape,dim,spec", INDEX_CASES)
def test_index_select_any_dim_and_vjp(oracle, shape, dim, spec, layout):
    """Tensor.index_select(dim, ids) (lib.rs:665-703) and its VJP
    scatter_index_select (autograd/ops.rs:741-769) against the oracle: the
    forward bit-exact; the gradient bit-exact (position-order sums from 0.0)
    except wide slices of ids occurring more than 128 times."""
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(sum(shape) + dim)
    d = dim % len(shape)
    ids = _ids(spec, shape[d], rng)
    x = rng.standard_normal(shape, dtype=np.float32)
    xv = _layout(x, layout).requires_grad_()
    out = T.index_select(xv, dim, ids)
    assert_bitexact(_host(out), oracle.t_index_select(x, dim, ids), "index_select")
    g = rng.standard_normal(tuple(out.shape), dtype=np.float32)
    out.backward(_dev(g))
    resolved = [i + shape[d] if i < 0 else i for i in ids]
    want = oracle.scatter_index_select(g, d, resolved, shape)
    got = _host(xv.grad)
    inner = int(np.prod(shape[d + 1:], dtype=np.int64))
    counts = np.bincount(np.asarray(resolved, np.int64), minlength=shape[d])
    if inner < 128 or counts.max(initial=0) <= 128:
        assert_bitexact(got, want, "index_select VJP")
    else:
        cold = np.moveaxis(got, d, 0)[counts <= 128]
        assert_bitexact(cold, np.moveaxis(want, d, 0)[counts <= 128], "VJP cold slices")
        scale = np.zeros(shape, np.float64)
        np.add.at(np.moveaxis(scale, d, 0), np.asarray(resolved),
                  np.abs(np.moveaxis(g.astype(np.float64), d, 0)))
        assert_close(got, want, rtol=RTOL_BIG, atol=ATOL * np.maximum(scale, 1.0),
                     what="VJP hot slices", strict_atol=ATOL * np.maximum(scale, 1.0))


def test_index_select_errors_match_reference():
    import torch
    from oxitorch_b200 import tensor_ops as T
    x = torch.zeros(5, 7, device="cuda")
    with pytest.raises(RuntimeError, match="index 9 out of range for dim 1 of size 7"):
        T.index_select(x, 1, [0, 9])
    with pytest.raises(RuntimeError, match="index -8 out of range for dim 1 of size 7"):
        T.index_select(x, -1, [-8])
    # device ids are checked by the kernel's error flag
    with pytest.raises(RuntimeError, match="index 7 out of range for dim 1 of size 7"):
        T.index_select(x, 1, torch.tensor([1, 7], device="cuda"))
    with pytest.raises(ValueError, match="dim 2 out of range for 2-D tensor"):
        T.index_select(x, 2, [0])


def test_gather_kats():
    """tensor/tests.rs:358-374 (gather_flat, gather_dim0) and
    test_indexing_grad.py:103-109 (gather accumulates duplicate grads)."""
    import torch
    from oxitorch_b200 import tensor_ops as T
    base = torch.arange(1, 7, dtype=torch.float32, device="cuda").reshape(2, 3)
    np.testing.assert_array_equal(_host(T.gather_flat(base, [0, 5, 1])), [1, 6, 2])
    with pytest.raises(RuntimeError, match="flat index 6 out of range for 6 elements"):
        T.gather_flat(base, [6])
    with pytest.raises(RuntimeError, match="flat index -7 out of range for 6 elements"):
        T.gather_flat(base, [-7])
    rows = T.gather_dim0(base, [1, 1, 0])
    np.testing.assert_array_equal(_host(rows), [[4, 5, 6], [4, 5, 6], [1, 2, 3]])
    with pytest.raises(RuntimeError, match="index 2 out of range for dim 0 of size 2"):
        T.gather_dim0(base, [2])
    with pytest.raises(ValueError, match="gather_dim0 requires at least a 1-D tensor"):
        T.gather_dim0(torch.tensor(1.0, device="cuda"), [0])
    t = torch.tensor([[1.0, 2.0], [3.0, 4.0]], device="cuda", requires_grad=True)
    out = T.gather(t, [1, 1])
    out.backward(torch.tensor([[5.0, 5.0], [6.0, 6.0]], device="cuda"))
    np.testing.assert_array_equal(_host(out), [[3, 4], [3, 4]])
    np.testing.assert_array_equal(_host(t.grad), [[0, 0], [11, 11]])
    # the same through the strided 'transposed' view of a 3 x 3 picked by rows
    a = np.arange(9, dtype=np.float32).reshape(3, 3)
    tt = _layout(a, "transposed").requires_grad_()
    picked = T.index_select(tt, 0, [2, 1, 1])
    picked.backward(torch.ones(3, 3, device="cuda"))
    np.testing.assert_array_equal(_host(picked), a[[2, 1, 1]])
    np.testing.assert_array_equal(_host(tt.grad), [[0, 0, 0], [2, 2, 2], [1, 1, 1]])
