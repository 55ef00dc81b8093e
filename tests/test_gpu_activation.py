"""F.gelu on its own (the GELU that does not follow a LayerNorm), forward and
VJP, against the oracle's composition of the reference graph
(python/oxitorch/nn/functional.py:194-199) and against float64.

Tolerances (tests/parity.py): rtol 1e-5 / atol 1e-6 plus the reference's own
budget: its summation order (none here: no sums) and the effect of a 4-ulp
change of the tanh it calls (glibc) -- the kernels evaluate the tanh form
through its logistic identity, as the fused LayerNorm+GELU kernels do.
"""

import numpy as np
import pytest

from parity import ATOL, assert_bitexact, assert_close, reference_budget

pytestmark = pytest.mark.gpu


def _dev(a, grad=False):
    import torch
    return torch.from_numpy(np.array(a, order="C", copy=True)).cuda().requires_grad_(grad)


def _host(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("shape", [(64, 4096), (1000, 777), (7,), (3, 5, 11), (1, 1)])
def test_gelu_vs_oracle(oracle, shape):
    from oxitorch_b200 import functional as F
    rng = np.random.default_rng(sum(shape))
    x = (rng.standard_normal(shape, dtype=np.float32) * np.float32(3)).astype(np.float32)
    dy = rng.standard_normal(shape, dtype=np.float32)

    def run():
        xt = oracle.from_numpy(x, True)
        y = oracle.gelu(xt)
        y.backward(dy)
        return y.numpy(), xt.grad.numpy()
    (y_ref, dx_ref), (by, bdx) = reference_budget(oracle, run, libm=("tanh",))
    xg = _dev(x, True)
    y = F.gelu(xg)
    y.backward(_dev(dy))
    assert_close(_host(y), y_ref, atol=ATOL + by, what="gelu(x)")
    assert_close(_host(xg.grad), dx_ref, atol=ATOL + bdx, what="dx")
    # the standalone kernels agree with the autograd path bit for bit
    assert_bitexact(_host(F.gelu_fwd(_dev(x))), _host(y), "gelu_fwd")
    assert_bitexact(_host(F.gelu_bwd(_dev(x), _dev(dy))), _host(xg.grad), "gelu_bwd")


def test_gelu_strided_input_and_grad():
    """A transposed x and a non-contiguous upstream gradient: one dense copy each
    (oxc_contiguous), then the same kernels -- the dense results, bit for bit."""
    from oxitorch_b200 import functional as F
    rng = np.random.default_rng(3)
    x = rng.standard_normal((96, 130), dtype=np.float32)
    dy = rng.standard_normal((96, 130), dtype=np.float32)
    xt = _dev(np.ascontiguousarray(x.T)).t().requires_grad_()
    F.gelu(xt).backward(_dev(np.ascontiguousarray(dy.T)).t())
    xd = _dev(x, True)
    yd = F.gelu(xd)
    yd.backward(_dev(dy))
    assert_bitexact(_host(F.gelu(xt)), _host(yd), "y")
    assert_bitexact(_host(xt.grad), _host(xd.grad), "dx")


def test_gelu_vs_float64_at_exact_arguments():
    """gelu(x) and gelu'(x) at exactly representable x against float64.  Bound:
    a few ulp, plus 4 ulp of |2 c v| (v = x + k x^3), the conditioning of
    e^(-2 c v) in the rounded argument; values below 1e-36 may flush to zero."""
    from oxitorch_b200 import functional as F
    x = np.linspace(-10.0, 10.0, 4093).astype(np.float32)
    x[:12] = [0.0, 1e-20, -1e-20, 1e-3, -1e-3, -0.7517916, 30.0, -30.0, 45.0, -45.0, 5.5, -5.5]
    y = _host(F.gelu_fwd(_dev(x)))
    d = _host(F.gelu_bwd(_dev(x), _dev(np.ones_like(x))))
    c = np.float64(np.float32(np.sqrt(2.0 / np.pi)))
    k = np.float64(np.float32(0.044715))
    x64 = x.astype(np.float64)
    v = x64 + k * x64 ** 3
    with np.errstate(over="ignore"):
        s = 1.0 / (1.0 + np.exp(-2.0 * c * v))
    g64 = x64 * s
    d64 = s + 2.0 * x64 * s * (1.0 - s) * c * (1.0 + 3.0 * k * x64 ** 2)
    rel = 2.0 ** -24 * (8.0 + 4.0 * np.abs(2.0 * c * v))
    assert_close(y, g64, rtol=0, atol=rel * np.abs(g64) + 1e-36, what="gelu(x)")
    dscale = np.abs(s) + np.abs(2.0 * x64 * s * (1.0 - s) * c * (1.0 + 3.0 * k * x64 ** 2))
    assert_close(d, d64, rtol=0, atol=rel * dscale + 1e-36, what="gelu'(x)")


def test_gelu_errors():
    import torch
    from oxitorch_b200 import functional as F
    with pytest.raises(ValueError, match="CUDA device"):
        F.gelu(torch.zeros(3))
    with pytest.raises(ValueError, match="shape mismatch"):
        F.gelu_bwd(torch.zeros(3, device="cuda"), torch.zeros(4, device="cuda"))
    assert F.gelu(torch.zeros(0, 5, device="cuda")).shape == (0, 5)
