"""RMSNorm and LayerNorm(+GELU) kernels vs the oracle and the golden fixtures.

Tolerances: see tests/parity.py.  dweight/dbias are column sums over rows, so
their absolute tolerance is 1e-6 * sum_rows |term| (the term each test names).
"""

import numpy as np
import pytest

from parity import RTOL, RTOL_BIG, ATOL, assert_close, assert_bitexact, reference_budget

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    return t.detach().cpu().numpy()


def _rms_case(seed, m, n):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, n), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    dy = rng.standard_normal((m, n), dtype=np.float32)
    return x, w, dy


def _oracle_rms(oracle, x, w, dy, eps=1e-6):
    """(y, dx, dw) of the composed reference path and their budgets (the
    reference's own summation-order error, tests/parity.py)."""
    def run():
        xt, wt = oracle.from_numpy(x, True), oracle.from_numpy(w, True)
        y = oracle.rms_norm(xt, wt, eps)
        y.backward(dy)
        return y.numpy(), xt.grad.numpy(), wt.grad.numpy()
    return reference_budget(oracle, run, libm=())


def _check_rms(x, w, dy, y, dx, dw, ref, rstd):
    (y_ref, dx_ref, dw_ref), (by, bdx, bdw) = ref
    assert_close(y, y_ref, atol=ATOL + by, what="y")
    assert_close(dx, dx_ref, atol=ATOL + bdx, what="dx")
    t1 = x * rstd[:, None]
    scale = np.abs(dy.astype(np.float64) * t1).sum(0)
    assert_close(dw, dw_ref, atol=ATOL * np.maximum(scale, 1.0) + bdw, what="dw",
                 strict_atol=ATOL * np.maximum(scale, 1.0))
    # f64 yardstick: the kernel's dw is within 1e-6 * sum|terms| of the exact value
    x64 = x.astype(np.float64)
    inv64 = 1.0 / np.sqrt((x64 * x64).mean(1) + 1e-6)
    dw64 = (dy.astype(np.float64) * x64 * inv64[:, None]).sum(0)
    assert_close(dw, dw64, rtol=RTOL, atol=ATOL * np.maximum(scale, 1.0), what="dw vs f64",
                 strict_atol=ATOL * np.maximum(scale, 1.0))


@pytest.mark.parametrize("name", ["rms_4x4096", "rms_7x1001", "rms_3x4"])
def test_rms_norm_golden(oracle, golden, name):
    from oxitorch_b200 import functional as F
    g = {k.split(".", 1)[1]: v for k, v in golden.items() if k.startswith(name + ".")}
    y, rstd = F.rms_norm_fwd(_dev(g["x"]), _dev(g["w"]), 1e-6)
    dx, dw = F.rms_norm_bwd(_dev(g["x"]), _dev(g["w"]), rstd, _dev(g["dy"]))
    _, budget = _oracle_rms(oracle, g["x"], g["w"], g["dy"])
    _check_rms(g["x"], g["w"], g["dy"], _host(y), _host(dx), _host(dw),
               ((g["y"], g["dx"], g["dw"]), budget), _host(rstd))


@pytest.mark.parametrize("m,n", [(256, 4096), (33, 4095), (5, 32768), (64, 11008), (1, 1), (2, 17)])
def test_rms_norm_vs_oracle(oracle, m, n):
    from oxitorch_b200 import functional as F
    x, w, dy = _rms_case(m * 7 + n, m, n)
    ref = _oracle_rms(oracle, x, w, dy)
    y, rstd = F.rms_norm_fwd(_dev(x), _dev(w), 1e-6)
    dx, dw = F.rms_norm_bwd(_dev(x), _dev(w), rstd, _dev(dy))
    _check_rms(x, w, dy, _host(y), _host(dx), _host(dw), ref, _host(rstd))


def test_rms_norm_config1_full_size(oracle):
    """x [4096, 4096] ~ N(0,1), w ~ U(0.5,1.5), eps 1e-6."""
    import bench
    from oxitorch_b200 import functional as F
    inp = bench.config_inputs(1)  # the arrays the benchmark times
    x, w, dy = inp["x"], inp["w"], inp["dy"]
    ref = _oracle_rms(oracle, x, w, dy)
    y, rstd = F.rms_norm_fwd(_dev(x), _dev(w), 1e-6)
    dx, dw = F.rms_norm_bwd(_dev(x), _dev(w), rstd, _dev(dy))
    _check_rms(x, w, dy, _host(y), _host(dx), _host(dw), ref, _host(rstd))


def test_rms_norm_exact_mode_vs_torch_autograd():
    """OXC_GRAD_EXACT is the full gradient: compare with torch fp64 autograd."""
    import torch
    from oxitorch_b200 import functional as F
    x, w, dy = _rms_case(9, 64, 1024)
    xd = torch.from_numpy(x).double().requires_grad_()
    wd = torch.from_numpy(w).double().requires_grad_()
    yd = xd * torch.rsqrt((xd * xd).mean(-1, keepdim=True) + 1e-6) * wd
    yd.backward(torch.from_numpy(dy).double())
    xg, wg = _dev(x).requires_grad_(), _dev(w).requires_grad_()
    y = F.rms_norm(xg, wg, 1e-6, grad_mode="exact")
    y.backward(_dev(dy))
    assert_close(_host(y), yd.detach().numpy(), what="y")
    assert_close(_host(xg.grad), xd.grad.numpy(), rtol=1e-4, atol=1e-5, what="dx exact")
    assert_close(_host(wg.grad), wd.grad.numpy(), rtol=1e-4, atol=1e-4, what="dw exact")


def test_rms_norm_autograd_and_determinism():
    from oxitorch_b200 import functional as F
    x, w, dy = _rms_case(11, 300, 4096)
    outs = []
    for _ in range(2):
        xg, wg = _dev(x).requires_grad_(), _dev(w).requires_grad_()
        F.rms_norm(xg, wg).backward(_dev(dy))
        outs.append((_host(xg.grad), _host(wg.grad)))
    assert_bitexact(outs[0][0], outs[1][0], "dx run-to-run")
    assert_bitexact(outs[0][1], outs[1][1], "dw run-to-run")


def _ln_case(seed, m, n):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, n), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    b = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    dy = rng.standard_normal((m, n), dtype=np.float32)
    return x, w, b, dy


def _oracle_ln(oracle, x, w, b, dy, gelu):
    """(outputs, budgets): y, dx, dw, db of the composed reference path and, per
    element, the reference's own summation-order error plus the effect of a
    4-ulp tanh difference (see tests/parity.py)."""
    def run():
        xt, wt, bt = (oracle.from_numpy(x, True), oracle.from_numpy(w, True),
                      oracle.from_numpy(b, True))
        y = oracle.layer_norm(xt, wt, bt, 1e-5)
        if gelu:
            y = oracle.gelu(y)
        y.backward(dy)
        return y.numpy(), xt.grad.numpy(), wt.grad.numpy(), bt.grad.numpy()
    return reference_budget(oracle, run, libm=("tanh",) if gelu else ())


def _ln_dev(x, w, b, dy, gelu, mode="ref"):
    from oxitorch_b200 import functional as F
    from oxitorch_b200 import _native as N
    act = N.ACT_GELU_TANH if gelu else N.ACT_NONE
    y, mean, rstd = F.layer_norm_fwd(_dev(x), _dev(w), _dev(b), 1e-5, act)
    dx, dw, db = F.layer_norm_bwd(_dev(x), _dev(w), _dev(b), mean, rstd, _dev(dy), act, mode)
    return _host(y), _host(dx), _host(dw), _host(db), _host(mean), _host(rstd)


def _check_ln(x, w, dy, got, ref, gelu):
    y, dx, dw, db, mean, rstd = got
    (y_ref, dx_ref, dw_ref, db_ref), (by, bdx, bdw, bdb) = ref
    # Centering (x - mean) turns a rounding of the mean into an absolute error
    # of |mean| * 2^-24 * rstd * |w| in y: 4 ulp of the mean propagated
    # (negligible for rows centred near 0, dominant for large offsets).
    gf = 1.2 if gelu else 1.0  # |gelu'| <= ~1.13
    cen = 4 * 2.0 ** -24 * (np.abs(mean) * rstd)[:, None] * np.abs(w)[None, :] * gf
    assert_close(y, y_ref, atol=ATOL + by + cen, what="y")
    # with GELU the gradient through y sees the same shift
    cdx = cen * np.abs(dy) * np.abs(w)[None, :] * rstd[:, None] if gelu else 0.0
    assert_close(dx, dx_ref, atol=ATOL + bdx + cdx, what="dx")
    # dweight terms: g * xhat; dbias terms: g, with |g| <= ~1.2 |dy| for GELU
    t1 = (x - mean[:, None]) * rstd[:, None]
    g_scale = np.abs(dy.astype(np.float64)) * gf
    cdw = (g_scale * (4 * 2.0 ** -24 * np.abs(mean) * rstd)[:, None]).sum(0)
    sdw = ATOL * np.maximum((g_scale * np.abs(t1)).sum(0), 1.0)
    sdb = ATOL * np.maximum(g_scale.sum(0), 1.0)
    assert_close(dw, dw_ref, atol=sdw + bdw + cdw, what="dw", strict_atol=sdw)
    assert_close(db, db_ref, atol=sdb + bdb, what="db", strict_atol=sdb)
    return cen, cdx, cdw, sdw, sdb


@pytest.mark.parametrize("name,gelu", [("lngelu_4x4096", True), ("lngelu_5x777", True),
                                       ("ln_6x512", False)])
def test_layer_norm_golden(oracle, golden, name, gelu):
    g = {k.split(".", 1)[1]: v for k, v in golden.items() if k.startswith(name + ".")}
    got = _ln_dev(g["x"], g["w"], g["b"], g["dy"], gelu)
    _, budget = _oracle_ln(oracle, g["x"], g["w"], g["b"], g["dy"], gelu)
    _check_ln(g["x"], g["w"], g["dy"], got, ((g["y"], g["dx"], g["dw"], g["db"]), budget), gelu)


@pytest.mark.parametrize("m,n,gelu", [(128, 4096, True), (40, 4095, True), (3, 32768, True),
                                      (50, 11008, False), (1, 1, True), (9, 33, False)])
def test_layer_norm_vs_oracle(oracle, m, n, gelu):
    x, w, b, dy = _ln_case(m * 13 + n, m, n)
    ref = _oracle_ln(oracle, x, w, b, dy, gelu)
    _check_ln(x, w, dy, _ln_dev(x, w, b, dy, gelu), ref, gelu)


@pytest.mark.parametrize("m,n,gelu", [(600, 4096, False), (37, 1001, True), (37, 1001, False)])
def test_layer_norm_pilot_fallback_rows(oracle, m, n, gelu):
    """Rows that defeat the forward's one-pass statistics: the first 32
    elements far from the rest (the pilot misses the mean by many standard
    deviations, so the second, corrected pass must run), a large common offset
    (cancellation), a constant row (zero variance) and ordinary rows.  Covers
    the persistent register kernel (plain LayerNorm, 4096 wide, more rows than
    resident CTAs) and the one-row-per-CTA kernel (odd width)."""
    x, w, b, dy = _ln_case(m * 7 + n, m, n)
    x[0::4, :32] += np.float32(1000.0)
    x[1::4] += np.float32(3.0e4)
    x[2::8] = np.float32(2.5)
    x[3::4, 32:] -= np.float32(50.0)
    got = _ln_dev(x, w, b, dy, gelu)
    # forward vs float64 on every row: the kernel's own error is a few ulp of
    # the row mean propagated through the normalisation (the reference's
    # sequential mean of a row offset by 3e4 is itself off by ~1e-2 there)
    x64 = x.astype(np.float64)
    mu = x64.mean(1, keepdims=True)
    rs = 1.0 / np.sqrt(((x64 - mu) ** 2).mean(1, keepdims=True) + 1e-5)
    y64 = (x64 - mu) * rs * w + b
    if gelu:
        y64 = 0.5 * y64 * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (y64 + 0.044715 * y64 ** 3)))
    cen = 8 * 2.0 ** -24 * np.abs(mu) * rs * np.abs(w)[None, :] * 1.2
    assert_close(got[0], y64, rtol=RTOL, atol=ATOL + cen, what="y vs f64")
    assert_close(got[4], mu[:, 0], rtol=RTOL, atol=ATOL, what="mean vs f64")
    assert_close(got[5], rs[:, 0], rtol=1e-5, atol=0, what="rstd vs f64")
    # the whole graph vs the oracle on the rows whose reference is accurate
    keep = np.arange(m) % 4 != 1
    xk, dyk = x[keep], dy[keep]
    ref = _oracle_ln(oracle, xk, w, b, dyk, gelu)
    _check_ln(xk, w, dyk, _ln_dev(xk, w, b, dyk, gelu), ref, gelu)


def test_layer_norm_gelu_config2_full_size(oracle):
    """BASELINE config 2 at the size and on the arrays the benchmark times
    (bench.config_inputs(2): x [16384, 4096], numpy PCG64(2)): every row and
    column, so the VJP's persistent geometry (about 111 rows per CTA and its
    dweight/dbias partials) is the benchmarked one.  Besides the pass/fail
    check, the elements beyond the bare tolerance (rtol 1e-5, atol 1e-6;
    1e-6 x Sigma|terms| for dweight/dbias) are attributed to the budget that
    admits them: the reference's own summation order, then the libm (tanh)
    ulps, then the centring term."""
    import bench
    from parity import reference_budget_parts, strict_breakdown
    inp = bench.config_inputs(2)
    x, w, b, dy = inp["x"], inp["w"], inp["b"], inp["dy"]
    assert x.shape == (16384, 4096)

    def run():
        xt, wt, bt = (oracle.from_numpy(x, True), oracle.from_numpy(w, True),
                      oracle.from_numpy(b, True))
        y = oracle.gelu(oracle.layer_norm(xt, wt, bt, 1e-5))
        y.backward(dy)
        return y.numpy(), xt.grad.numpy(), wt.grad.numpy(), bt.grad.numpy()
    base, sums, libm = reference_budget_parts(oracle, run, ("tanh",))
    got = _ln_dev(x, w, b, dy, True)
    budget = [a + c for a, c in zip(sums, libm)]
    cen, cdx, cdw, sdw, sdb = _check_ln(x, w, dy, got, (base, budget), True)
    for i, (name, strict, centre) in enumerate((("y", ATOL, cen), ("dx", ATOL, cdx),
                                                ("dw", sdw, cdw), ("db", sdb, 0.0))):
        strict_breakdown(got[i], base[i], RTOL, strict,
                         [("summation_order", sums[i]), ("libm_tanh", libm[i]),
                          ("centring", centre)], what=f"config 2 {name}")


@pytest.mark.parametrize("n", [4096, 4094])
def test_gelu_evaluation_vs_f64(n):
    """The kernels' GELU and its derivative at exactly known arguments, against
    float64.  A row of alternating +1/-1 has mean 0 and variance 1 exactly, so
    with weight 0 the affine output is fma(xhat, 0, b) = b: y = gelu(b).  With
    one row and dy = 1, dbias = gelu'(b).  n = 4096 runs the pipelined kernels,
    n = 4094 (not a multiple of 4) the register kernels.

    Bound: a few ulp, plus 4 ulp of the exponent's size |2 c v| (v = b + k b^3):
    the rounding of v moves e^(-2 c v) by that much in relative terms, which is
    the formula's own conditioning far into the negative tail.  Results below
    1e-36 in magnitude may flush to zero (ex2/rcp run flush-to-zero)."""
    x = np.tile(np.array([1.0, -1.0], np.float32), (1, n // 2))
    b = np.linspace(-10.0, 10.0, n).astype(np.float32)
    b[:12] = [0.0, 1e-20, -1e-20, 1e-3, -1e-3, -0.7517916, 30.0, -30.0, 45.0, -45.0, 5.5, -5.5]
    w = np.zeros(n, np.float32)
    dy = np.ones((1, n), np.float32)
    y, _, _, db, mean, rstd = _ln_dev(x, w, b, dy, True)
    assert mean[0] == 0.0 and rstd[0] == np.float32(1.0 / np.sqrt(np.float32(1.0) + np.float32(1e-5)))
    c = np.float64(np.float32(np.sqrt(2.0 / np.pi)))
    k = np.float64(np.float32(0.044715))
    b64 = b.astype(np.float64)
    v = b64 + k * b64 ** 3
    with np.errstate(over="ignore"):
        s = 1.0 / (1.0 + np.exp(-2.0 * c * v))
    g64 = b64 * s
    d64 = s + 2.0 * b64 * s * (1.0 - s) * c * (1.0 + 3.0 * k * b64 ** 2)
    rel = 2.0 ** -24 * (8.0 + 4.0 * np.abs(2.0 * c * v))
    assert_close(y[0], g64, rtol=0, atol=rel * np.abs(g64) + 1e-36, what="gelu(b)")
    dscale = np.abs(s) + np.abs(2.0 * b64 * s * (1.0 - s) * c * (1.0 + 3.0 * k * b64 ** 2))
    assert_close(db, d64, rtol=0, atol=rel * dscale + 1e-36, what="gelu'(b)")


def test_layer_norm_exact_mode_vs_torch_autograd():
    import torch
    x, w, b, dy = _ln_case(21, 64, 1024)
    xd = torch.from_numpy(x).double().requires_grad_()
    wd = torch.from_numpy(w).double().requires_grad_()
    bd = torch.from_numpy(b).double().requires_grad_()
    yd = torch.nn.functional.gelu(
        torch.nn.functional.layer_norm(xd, (1024,), wd, bd, 1e-5), approximate="tanh")
    yd.backward(torch.from_numpy(dy).double())
    y, dx, dw, db, _, _ = _ln_dev(x, w, b, dy, True, mode="exact")
    assert_close(y, yd.detach().numpy(), rtol=1e-5, atol=1e-6, what="y")
    assert_close(dx, xd.grad.numpy(), rtol=1e-4, atol=1e-5, what="dx exact")
    assert_close(dw, wd.grad.numpy(), rtol=1e-4, atol=1e-4, what="dw exact")
    assert_close(db, bd.grad.numpy(), rtol=1e-4, atol=1e-4, what="db exact")


def test_layer_norm_autograd_function():
    from oxitorch_b200 import functional as F
    x, w, b, dy = _ln_case(5, 32, 4096)
    xg, wg, bg = _dev(x).requires_grad_(), _dev(w).requires_grad_(), _dev(b).requires_grad_()
    F.layer_norm_gelu(xg, wg, bg).backward(_dev(dy))
    got = _ln_dev(x, w, b, dy, True)
    assert_bitexact(_host(xg.grad), got[1], "dx")
    assert_bitexact(_host(wg.grad), got[2], "dw")
    assert_bitexact(_host(bg.grad), got[3], "db")


def test_workspace_too_small_is_a_value_error():
    import torch
    from oxitorch_b200 import _native as N
    L = N.load()
    x = torch.zeros(64, 256, device="cuda")
    w = torch.ones(256, device="cuda")
    rstd = torch.ones(64, device="cuda")
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    st = L.oxc_rms_norm_bwd(x.data_ptr(), w.data_ptr(), rstd.data_ptr(), x.data_ptr(),
                            x.data_ptr(), w.data_ptr(), 64, 256, 0, ws.data_ptr(), 16,
                            torch.cuda.current_stream().cuda_stream)
    with pytest.raises(ValueError, match="workspace"):
        N.check(st)
