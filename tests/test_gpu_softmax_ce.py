"""softmax / log_softmax / cross-entropy kernels vs the oracle and fixtures.

Tolerances (tests/parity.py): rtol 1e-5 / atol 1e-6 plus the reference's own
summation-order error, a 4-ulp exp/log libm budget and, for gradients, the
max node's exact-zero VJP term the kernels leave out.  Cross-entropy
gradients are compared as M * dlogits (M = rows), i.e. in units of the
per-row gradient, so atol 1e-6 stays meaningful for every batch size.
"""

import numpy as np
import pytest

from parity import ATOL, RTOL, RTOL_BIG, assert_close, assert_bitexact, max_vjp_budget, \
    reference_budget

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    return t.detach().cpu().numpy()


def _logits(seed, m, n, spikes=True):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((m, n), dtype=np.float32) * np.float32(2.0)).astype(np.float32)
    if spikes:
        x[rng.random((m, n)) < 0.01] = 20.0
    dy = rng.standard_normal((m, n), dtype=np.float32)
    return x, dy


def _oracle_softmax(oracle, x, dy, log):
    def run():
        xt = oracle.from_numpy(x, True)
        y = (oracle.log_softmax if log else oracle.softmax)(xt, -1)
        y.backward(dy)
        return y.numpy(), xt.grad.numpy()
    ref, budget = reference_budget(oracle, run, libm=("exp", "log"))
    mv = max_vjp_budget(oracle, run)
    return ref, [b + m for b, m in zip(budget, mv)]


def _dev_softmax(x, dy, log):
    from oxitorch_b200 import functional as F
    y = F.softmax_fwd(_dev(x), log)
    dx = F.softmax_bwd(y, _dev(dy), log)
    return _host(y), _host(dx)


def _check_softmax(got, ref, budget, n):
    rtol = RTOL if n < 32768 else RTOL_BIG
    (y, dx), (y_ref, dx_ref), (by, bdx) = got, ref, budget
    assert_close(y, y_ref, rtol=rtol, atol=ATOL + by, what="y")
    assert_close(dx, dx_ref, rtol=rtol, atol=ATOL + bdx, what="dx")


@pytest.mark.parametrize("name,log", [("softmax_4x3000", False), ("logsoftmax_4x3000", True),
                                      ("logsoftmax_3x5", True)])
def test_softmax_golden(oracle, golden, name, log):
    g = {k.split(".", 1)[1]: v for k, v in golden.items() if k.startswith(name + ".")}
    _, budget = _oracle_softmax(oracle, g["x"], g["dy"], log)
    _check_softmax(_dev_softmax(g["x"], g["dy"], log), (g["y"], g["dx"]), budget, g["x"].shape[1])


@pytest.mark.parametrize("m,n,log", [(64, 32000, False), (64, 32000, True), (37, 1001, True),
                                     (300, 4096, False), (1, 1, True), (5, 7, False)])
def test_softmax_vs_oracle(oracle, m, n, log):
    x, dy = _logits(m * 3 + n, m, n)
    ref, budget = _oracle_softmax(oracle, x, dy, log)
    _check_softmax(_dev_softmax(x, dy, log), ref, budget, n)


def test_softmax_stability_large_inputs():
    """test_nn.py:40-48 on the device: finite log_softmax of [1000, 1001, 1002]."""
    y, _ = _dev_softmax(np.array([[1000.0, 1001.0, 1002.0]], np.float32),
                        np.ones((1, 3), np.float32), True)
    assert np.all(np.isfinite(y))
    want = np.exp(np.array([1000.0, 1001.0, 1002.0]) - 1002.0)
    assert np.allclose(np.exp(y) / np.exp(y).sum(), want / want.sum(), atol=1e-6)


def test_softmax_autograd_and_determinism():
    from oxitorch_b200 import functional as F
    x, dy = _logits(9, 128, 32000)
    outs = []
    for _ in range(2):
        xg = _dev(x).requires_grad_()
        F.log_softmax(xg).backward(_dev(dy))
        outs.append(_host(xg.grad))
    assert_bitexact(outs[0], outs[1], "dx run-to-run")


# ---- cross-entropy ----------------------------------------------------------------------

def _oracle_ce(oracle, x, t):
    def run():
        xt = oracle.from_numpy(x, True)
        loss = oracle.cross_entropy(xt, [int(v) for v in t])
        loss.backward()
        return np.array([loss.item()], np.float32), xt.grad.numpy()
    ref, budget = reference_budget(oracle, run, libm=("exp", "log"))
    mv = max_vjp_budget(oracle, run)
    return ref, [b + m for b, m in zip(budget, mv)]


def _dev_ce(x, t):
    from oxitorch_b200 import functional as F
    loss, rmax, rsum, _, tt, flag = F.cross_entropy_fwd(_dev(x), [int(v) for v in t])
    dx = F.cross_entropy_bwd(_dev(x), tt, rmax, rsum)
    assert int(flag.cpu()[0]) == 0
    return _host(loss), _host(dx)


def _check_ce(got, ref, budget, m):
    (loss, dx), (l_ref, dx_ref), (bl, bdx) = got, ref, budget
    rtol = RTOL if m < 32768 else RTOL_BIG
    assert_close(loss, l_ref, rtol=rtol, atol=ATOL + bl, what="loss")
    # gradients in units of the per-row gradient (M * dlogits)
    assert_close(dx * m, dx_ref * m, rtol=rtol, atol=ATOL + bdx * m, what="M * dlogits")


@pytest.mark.parametrize("name", ["ce_8x3200", "ce_5x7"])
def test_cross_entropy_golden(oracle, golden, name):
    g = {k.split(".", 1)[1]: v for k, v in golden.items() if k.startswith(name + ".")}
    _, budget = _oracle_ce(oracle, g["x"], g["targets"])
    _check_ce(_dev_ce(g["x"], g["targets"]), (g["loss"].reshape(1), g["dx"]), budget,
              g["x"].shape[0])


@pytest.mark.parametrize("m,n", [(64, 32000), (33, 1000), (1, 3), (7, 4097)])
def test_cross_entropy_vs_oracle(oracle, m, n):
    x, _ = _logits(m * 5 + n, m, n)
    t = np.random.default_rng(m + n).integers(0, n, m)
    t[0] = -1  # negative targets count from the end (numpy one-hot indexing)
    ref, budget = _oracle_ce(oracle, x, t)
    _check_ce(_dev_ce(x, t), ref, budget, m)


def test_cross_entropy_reference_values():
    """test_nn.py:111-122: loss and grad = (softmax - onehot) / n."""
    x = np.array([[1.0, 2.0, 3.0], [3.0, 1.0, 2.0]], np.float32)
    loss, dx = _dev_ce(x, [2, 0])
    m = x.max(-1, keepdims=True)
    ls = x - m - np.log(np.exp(x - m).sum(-1, keepdims=True))
    assert abs(float(loss[0]) - (-np.mean([ls[0, 2], ls[1, 0]]))) < 1e-5
    g = (np.exp(ls) - np.eye(3, dtype=np.float32)[[2, 0]]) / 2
    assert np.allclose(dx, g, rtol=1e-4, atol=1e-6)


def _nonfinite_rows(n, seed):
    """Rows with -inf / +inf / NaN placed the way the reference's edge cases
    differ: leading -inf then finite values (the online max starts at -inf),
    all -inf, NaN, -inf only at the target (+inf loss), -inf elsewhere too
    (NaN loss: the one-hot product 0 * -inf), +inf, a dominated row and a
    plain row.  Returns logits, targets, upstream gradient."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((8, n)).astype(np.float32)
    t = rng.integers(0, n, 8)
    x[0, :2] = -np.inf
    t[0] = n - 1
    x[1, :] = -np.inf
    x[2, n // 2] = np.nan
    t[3] = 1
    x[3, 1] = -np.inf
    t[4] = 0
    x[4, 0] = -np.inf
    x[4, n - 1] = -np.inf
    x[5, n // 3] = np.inf
    x[6, :] = -30.0
    x[6, t[6]] = 0.0
    dy = rng.standard_normal((8, n)).astype(np.float32)
    return x, t, dy


@pytest.mark.parametrize("n", [1000, 37])
@pytest.mark.parametrize("log", [False, True])
def test_softmax_nonfinite_rows(oracle, n, log):
    x, _, dy = _nonfinite_rows(n, n)
    ref, budget = _oracle_softmax(oracle, x, dy, log)
    _check_softmax(_dev_softmax(x, dy, log), ref, budget, n)


@pytest.mark.parametrize("n", [1000, 37])
def test_cross_entropy_nonfinite_rows(oracle, n):
    """Per-row values against the reference graph's picked sum (one-hot
    product), the mean, and a finite VJP on the rows the reference keeps
    finite."""
    from oxitorch_b200 import functional as F
    x, t, _ = _nonfinite_rows(n, n + 1)
    loss, rmax, rsum, nll, tt, flag = F.cross_entropy_fwd(_dev(x), [int(v) for v in t])
    assert int(flag.cpu()[0]) == 0
    onehot = np.zeros_like(x)
    onehot[np.arange(8), t] = 1.0
    ls = oracle.log_softmax(oracle.from_numpy(x), -1)
    picked = (oracle.from_numpy(onehot) * ls).sum(-1).numpy()
    want = -picked
    got = _host(nll)
    assert np.array_equal(np.isnan(got), np.isnan(want)), (got, want)
    assert np.array_equal(np.isposinf(got), np.isposinf(want)), (got, want)
    fin = np.isfinite(want)
    assert_close(got[fin], want[fin], rtol=RTOL, atol=1e-5, what="row nll")
    assert np.isnan(_host(loss)[0])
    (_, dref), (_, bdx) = _oracle_ce(oracle, x, t)
    dx = _host(F.cross_entropy_bwd(_dev(x), tt, rmax, rsum))
    assert_close(dx * 8, dref * 8, rtol=RTOL, atol=ATOL + bdx * 8, what="M * dlogits")


def test_cross_entropy_errors():
    import torch
    from oxitorch_b200 import functional as F
    logits = torch.zeros(2, 3, device="cuda")
    with pytest.raises(ValueError, match="targets"):
        F.cross_entropy(logits, [0, 1, 2])
    with pytest.raises(IndexError, match="out of bounds"):
        F.cross_entropy(logits, [0, 3])


def test_cross_entropy_autograd():
    from oxitorch_b200 import functional as F
    x, _ = _logits(17, 16, 512)
    t = np.random.default_rng(3).integers(0, 512, 16)
    xg = _dev(x).requires_grad_()
    F.cross_entropy(xg, [int(v) for v in t]).backward()
    _, dx = _dev_ce(x, t)
    assert_bitexact(_host(xg.grad), dx, "autograd dlogits")


def test_cross_entropy_config3_full_size(oracle):
    """BASELINE config 3 (bench.config_inputs(3), the benchmarked arrays):
    logits [32768, 32000] ~ N(0, 2^2), 1% of entries +20, targets uniform.  Loss vs an fp64 torch computation of the whole batch;
    dlogits of 64 sampled rows vs the oracle (its 64-row batch has 1/64 where
    the full batch has 1/32768; both are powers of two, so the oracle's
    gradients rescale exactly); run-to-run determinism."""
    import torch
    from oxitorch_b200 import functional as F
    import bench
    M, C = 32768, 32000
    inp = bench.config_inputs(3)  # the arrays the benchmark times
    x = torch.from_numpy(inp["logits"]).cuda()
    t = torch.from_numpy(inp["targets"]).cuda()
    del inp
    loss, rmax, rsum, _, tt, flag = F.cross_entropy_fwd(x, t)
    dx = F.cross_entropy_bwd(x, tt, rmax, rsum)
    assert int(flag.cpu()[0]) == 0
    lse = torch.cat([torch.logsumexp(x[i:i + 4096].double(), dim=1) for i in range(0, M, 4096)])
    want = (lse - x.gather(1, t[:, None])[:, 0].double()).mean().item()
    assert abs(loss.item() - want) <= 1e-5 * abs(want), (loss.item(), want)
    rows = np.random.default_rng(0).choice(M, 64, replace=False)
    xs = x[rows].cpu().numpy()
    ts = t[rows].cpu().numpy()
    (_, dref), (_, bdx) = _oracle_ce(oracle, xs, ts)
    scale = np.float32(64.0 / M)
    got = _host(dx[rows])
    assert_close(got * M, dref * scale * M, rtol=RTOL_BIG, atol=ATOL + bdx * 64, what="M * dlogits rows")
    row_sums = dx.sum(dim=1).abs().max().item()
    assert row_sums < 1e-9, row_sums
    dx2 = F.cross_entropy_bwd(x, tt, rmax, rsum)
    assert torch.equal(dx, dx2)
