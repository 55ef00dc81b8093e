"""Reduce VJPs (crates/oxi-autograd/src/ops.rs:327-388) and unbroadcast
(graph.rs:274-313) on the device vs the oracle's restatement.

sum / mean / max / min gradients are copies, one IEEE product, or a scatter to
the first argmax/argmin: bit-exact.  The norm gradient divides by the strip's
norm, which the kernels sum in tree order (row strips) where the reference
folds left to right: rtol 1e-5 plus the reference's own summation error.
unbroadcast sums over non-last axes fold left to right like the reference
(bit-exact); sums over the last axis use the tree (tolerance as above).
"""

import numpy as np
import pytest

from parity import ATOL, RTOL, assert_bitexact, assert_close, reference_budget

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    return t.detach().cpu().numpy()


def _oracle_vjp(oracle, x, kind, dim, keepdim, g):
    def run():
        xt = oracle.from_numpy(x, True)
        y = oracle.Tensor(oracle.a_reduce(xt._v, kind, dim, keepdim))
        y.backward(g)
        return (xt.grad.numpy(),)
    return reference_budget(oracle, run, libm=())


def _case(seed, shape):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape).astype(np.float32)
    # ties and NaNs along every axis: max/min must pick the first occurrence
    # and ignore NaN (f32::max), a NaN at index 0 keeps index 0 (argmax)
    x.reshape(-1)[::7] = np.float32(2.5)
    x.reshape(-1)[5::11] = np.nan
    return x


@pytest.mark.parametrize("kind", ["sum", "mean", "max", "min", "norm"])
@pytest.mark.parametrize("dim", [0, 1, -1])
@pytest.mark.parametrize("keepdim", [False, True])
def test_reduce_vjp_vs_oracle(oracle, kind, dim, keepdim):
    from oxitorch_b200 import tensor_ops as T
    shape = (7, 33, 40)
    x = _case(3 + dim, shape)
    if kind == "norm":
        x = np.nan_to_num(x)
    oshape = list(shape)
    d = dim % 3
    if keepdim:
        oshape[d] = 1
    else:
        oshape.pop(d)
    g = np.random.default_rng(9).standard_normal(oshape).astype(np.float32)
    (want,), (budget,) = _oracle_vjp(oracle, x, kind, dim, keepdim, g)
    got = _host(T.reduce_backward(kind, _dev(x), dim, _dev(g)))
    if kind == "norm":
        assert_close(got, want, rtol=RTOL, atol=ATOL + budget, what="norm vjp")
    else:
        assert_bitexact(got, want, f"{kind} vjp")


@pytest.mark.parametrize("kind", ["sum", "mean", "max", "norm"])
def test_reduce_vjp_strided_input(oracle, kind):
    """A transposed view as the forward input (strides [1, rows])."""
    from oxitorch_b200 import tensor_ops as T
    base = _case(11, (64, 300))
    if kind == "norm":
        base = np.nan_to_num(base)
    x = np.ascontiguousarray(base.T)               # [300, 64] values
    xv = _dev(base).t()                            # the same values, strides [1, 300]
    assert tuple(xv.stride()) == (1, 300)
    g = np.random.default_rng(1).standard_normal((300,)).astype(np.float32)
    (want,), (budget,) = _oracle_vjp(oracle, x, kind, 1, False, g)
    got = _host(T.reduce_backward(kind, xv, 1, _dev(g)))
    if kind == "norm":
        assert_close(got, want, rtol=RTOL, atol=ATOL + budget, what="norm vjp")
    else:
        assert_bitexact(got, want, f"{kind} vjp")


def test_reduce_autograd_and_errors():
    import torch
    from oxitorch_b200 import tensor_ops as T
    x = _case(5, (16, 50))
    xg = _dev(x).requires_grad_()
    y = T.reduce("max", xg, 1)
    y.backward(torch.ones_like(y))
    g = _host(xg.grad)
    assert g.sum() == 16.0 and ((g == 0) | (g == 1)).all()
    with pytest.raises(NotImplementedError, match="no gradient"):
        T.reduce_backward("argmax", _dev(x), 1, _dev(np.zeros(16, np.float32)))
    with pytest.raises(ValueError, match="out of range"):
        T.reduce_backward("sum", _dev(x), 2, _dev(np.zeros(16, np.float32)))
    with pytest.raises(ValueError, match="shape mismatch"):
        T.reduce_backward("sum", _dev(x), 1, _dev(np.zeros(15, np.float32)))


@pytest.mark.parametrize("gshape,target", [((4, 3, 5), (4, 1, 5)), ((4, 3, 5), (1, 3, 1)),
                                           ((6, 4, 3, 5), (4, 3, 5)), ((4, 3, 5), (4, 3, 1)),
                                           ((2, 9, 33), (9, 33)), ((4, 3, 5), (1, 5))])
def test_unbroadcast_vs_oracle(oracle, gshape, target):
    """Including a target the reference itself cannot reach: with prepended
    axes it sums by target position, so [4,3,5] -> [1,5] ends in a failed
    reshape; both sides raise the shape mismatch."""
    from oxitorch_b200 import tensor_ops as T
    g = np.random.default_rng(len(gshape) + sum(target)).standard_normal(gshape).astype(np.float32)
    try:
        want = oracle.unbroadcast(g, target)
    except Exception as e:  # the reference's ShapeMismatch (or numpy's reshape error)
        with pytest.raises(ValueError, match="shape mismatch"):
            T.unbroadcast(_dev(g), target)
        return
    got = _host(T.unbroadcast(_dev(g), target))
    assert got.shape == tuple(target)
    last_axis_summed = len(target) == len(gshape) and target[-1] == 1 and gshape[-1] != 1
    if last_axis_summed:
        assert_close(got, want, rtol=RTOL, atol=ATOL * np.abs(g).sum() / max(want.size, 1),
                     what="unbroadcast", strict_atol=ATOL * np.abs(g).sum() / max(want.size, 1))
    else:
        assert_bitexact(got, want, "unbroadcast")
