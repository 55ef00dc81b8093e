"""SiLU / SwiGLU kernels and the BASELINE config 5 decoder-MLP block.

Elementwise results follow the reference's rounding sequence step by step;
differences come only from exp (CUDA vs glibc, a 4-ulp budget measured on the
oracle) -- tolerance rtol 1e-5 / atol 1e-6 plus that budget.  Row sums carry
the reference's own summation-order error too (tests/parity.py)."""

import numpy as np
import pytest

from parity import ATOL, RTOL, RTOL_BIG, assert_bitexact, assert_close, reference_budget

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    return t.detach().cpu().numpy()


def _oracle_swiglu(oracle, g, u, dh):
    def run():
        gt = oracle.from_numpy(g, True)
        if u is None:
            h = oracle.silu(gt)
            h.backward(dh)
            return h.numpy(), gt.grad.numpy()
        ut = oracle.from_numpy(u, True)
        h = oracle.silu(gt) * ut
        h.backward(dh)
        return h.numpy(), gt.grad.numpy(), ut.grad.numpy()
    return reference_budget(oracle, run, libm=("exp", "sigmoid"))


@pytest.mark.parametrize("name", ["silu_4x1000", "swiglu_4x1100"])
def test_swiglu_golden(oracle, golden, name):
    from oxitorch_b200 import functional as F
    g = {k.split(".", 1)[1]: v for k, v in golden.items() if k.startswith(name + ".")}
    if name.startswith("silu"):
        (h_ref, dg_ref), (bh, bdg) = _oracle_swiglu(oracle, g["x"], None, g["dy"])
        h = F.swiglu_fwd(_dev(g["x"]))
        dg, _ = F.swiglu_bwd(_dev(g["x"]), None, _dev(g["dy"]))
        assert_close(_host(h), g["y"], atol=ATOL + bh, what="silu y")
        assert_close(_host(dg), g["dx"], atol=ATOL + bdg, what="silu dx")
    else:
        (_, _, _), (bh, bdg, bdu) = _oracle_swiglu(oracle, g["g"], g["u"], g["dh"])
        h = F.swiglu_fwd(_dev(g["g"]), _dev(g["u"]))
        dg, du = F.swiglu_bwd(_dev(g["g"]), _dev(g["u"]), _dev(g["dh"]))
        assert_close(_host(h), g["h"], atol=ATOL + bh, what="h")
        assert_close(_host(dg), g["dg"], atol=ATOL + bdg, what="dg")
        assert_close(_host(du), g["du"], atol=ATOL + bdu, what="du")


@pytest.mark.parametrize("transposed_gate", [False, True])
@pytest.mark.parametrize("m,n", [(300, 1100), (33, 47), (1, 5)])
def test_swiglu_vs_oracle_layouts(oracle, m, n, transposed_gate):
    from oxitorch_b200 import functional as F
    rng = np.random.default_rng(m + n)
    g = rng.standard_normal((m, n), dtype=np.float32) * np.float32(3)
    u = rng.standard_normal((m, n), dtype=np.float32)
    dh = rng.standard_normal((m, n), dtype=np.float32)
    (h_ref, dg_ref, du_ref), (bh, bdg, bdu) = _oracle_swiglu(oracle, g, u, dh)
    gd = _dev(np.ascontiguousarray(g.T)).t() if transposed_gate else _dev(g)
    h, s, mx, am = F.swiglu_fwd(gd, _dev(u), row_stats=True)
    dg, du, sq = F.swiglu_bwd(gd, _dev(u), _dev(dh), sumsq=True)
    assert_close(_host(h), h_ref, atol=ATOL + bh, what="h")
    assert_close(_host(dg), dg_ref, atol=ATOL + bdg, what="dg")
    assert_close(_host(du), du_ref, atol=ATOL + bdu, what="du")
    # dim-1 reductions of the kernel's own h: max/argmax exact, sum in tree order
    hh = _host(h)
    assert_bitexact(_host(mx), oracle.t_reduce("max", hh, 1, False), "row max")
    assert_bitexact(_host(am), oracle.t_reduce("argmax", hh, 1, False), "row argmax")
    want_s = oracle.t_reduce("sum", hh, 1, False)
    assert_close(_host(s), want_s, atol=ATOL * np.abs(hh).sum(1) + 1e-6, what="row sum",
                 strict_atol=ATOL * np.abs(hh).sum(1) + 1e-6)
    want_sq = float((_host(dg).astype(np.float64) ** 2).sum() + (_host(du).astype(np.float64) ** 2).sum())
    assert abs(float(_host(sq)) - want_sq) <= 1e-12 * want_sq + 1e-30


def _gate_view(g, layout):
    """Device view of g [m, n] in one of the layouts the kernels dispatch on."""
    import torch
    m, n = g.shape
    if layout == "row_strided":      # rows of a wider buffer: row stride n + 12
        buf = torch.zeros(m, n + 12, device="cuda")
        buf[:, :n] = _dev(g)
        return buf[:, :n]
    if layout == "col_strided":      # transposed view of a taller buffer: stride m + 4
        buf = torch.zeros(n, m + 4, device="cuda")
        buf[:, :m] = _dev(np.ascontiguousarray(g.T))
        return buf[:, :m].t()
    if layout == "misaligned":       # base 4 bytes past a 16-byte boundary
        buf = torch.zeros(m * n + 1, device="cuda")
        buf[1:] = _dev(g.reshape(-1))
        return buf[1:].view(m, n)
    raise ValueError(layout)


@pytest.mark.parametrize("with_up", [True, False])
@pytest.mark.parametrize("layout", ["row_strided", "col_strided", "misaligned"])
def test_swiglu_gate_layouts_many_strips(oracle, layout, with_up):
    """More 32-token strips than SMs (CTAs loop), a feature count that is not a
    multiple of the 128-feature tile, strided and misaligned gates, silu-only,
    and NaNs: h[0, 0] NaN (argmax 0, max ignores it) and a NaN mid-row."""
    from oxitorch_b200 import functional as F
    rng = np.random.default_rng(31)
    m, n = 4800, 260
    g = rng.standard_normal((m, n), dtype=np.float32) * np.float32(3)
    g[0, 0] = np.nan
    g[7, 100] = np.nan
    u = rng.standard_normal((m, n), dtype=np.float32) if with_up else None
    dh = rng.standard_normal((m, n), dtype=np.float32)
    outs, budgets = _oracle_swiglu(oracle, g, u, dh)
    gd = _gate_view(g, layout)
    ud = _dev(u) if with_up else None
    h, s, mx, am = F.swiglu_fwd(gd, ud, row_stats=True)
    res = F.swiglu_bwd(gd, ud, _dev(dh), sumsq=True)
    assert_close(_host(h), outs[0], atol=ATOL + budgets[0], what="h")
    assert_close(_host(res[0]), outs[1], atol=ATOL + budgets[1], what="dg")
    if with_up:
        assert_close(_host(res[1]), outs[2], atol=ATOL + budgets[2], what="du")
    hh = _host(h)
    assert_bitexact(_host(mx), oracle.t_reduce("max", hh, 1, False), "row max")
    assert_bitexact(_host(am), oracle.t_reduce("argmax", hh, 1, False), "row argmax")
    assert _host(am)[0] == 0
    fin = np.isfinite(hh).all(1)
    want_s = oracle.t_reduce("sum", hh, 1, False)
    assert np.isnan(_host(s)[~fin]).all()
    assert_close(_host(s)[fin], want_s[fin], atol=ATOL * np.abs(hh[fin]).sum(1) + 1e-6,
                 what="row sum", strict_atol=ATOL * np.abs(hh[fin]).sum(1) + 1e-6)
    parts = [_host(res[0])] + ([_host(res[1])] if with_up else [])
    want_sq = sum(float(np.nansum(p.astype(np.float64) ** 2)) for p in parts)
    got_sq = float(_host(res[-1]))
    assert np.isnan(got_sq) or abs(got_sq - want_sq) <= 1e-12 * want_sq


def test_silu_autograd():
    from oxitorch_b200 import functional as F
    rng = np.random.default_rng(4)
    x = rng.standard_normal((64, 200), dtype=np.float32)
    xg = _dev(x).requires_grad_()
    F.silu(xg).backward(_dev(np.ones_like(x)))
    dg, _ = F.swiglu_bwd(_dev(x), None, _dev(np.ones_like(x)))
    assert_bitexact(_host(xg.grad), _host(dg), "silu autograd")


def test_decoder_mlp_block_config5(oracle):
    """BASELINE config 5 at full size: x [65536, 4096]; RMSNorm weight given as
    a broadcast_to([65536, 4096]) view of [1, 4096]; gate a transposed view of
    a contiguous [11008, 65536] buffer; up [65536, 11008]; upstream dy, dh.
    Outputs y, h, dim-1 sum/max/argmax of h, dx, dweight, dg, du and the
    whole-tensor L2 over {dx, dg, du}.  Checked on 64 sampled rows against the
    oracle, dweight and the L2 against float64 torch over everything."""
    import torch
    from oxitorch_b200 import functional as F
    from oxitorch_b200 import tensor_ops as T
    import bench
    M, D, H = 65536, 4096, 11008
    inp = {k: torch.from_numpy(v).cuda() for k, v in bench.config_inputs(5).items()}
    x, up, dy, dh = inp["x"], inp["up"], inp["dy"], inp["dh"]
    w = inp["w"].broadcast_to(M, D)
    gate = inp["gate_buf"].t()                             # strides [1, 65536]
    assert gate.stride() == (1, M) and w.stride() == (0, 1)

    y, rstd = F.rms_norm_fwd(x, w, 1e-6)
    h, hs, hm, ha = F.swiglu_fwd(gate, up, row_stats=True)
    dx, dw = F.rms_norm_bwd(x, w, rstd, dy)
    dg, du, sq_gu = F.swiglu_bwd(gate, up, dh, sumsq=True)
    total = float(T.sum_squares([dx]).item()) + float(sq_gu.item())
    l2 = total ** 0.5

    rows = np.sort(np.random.default_rng(1).choice(M, 64, replace=False))
    xs, ws_ = x[rows].cpu().numpy(), w[0].cpu().numpy()
    gs, us = gate[rows].cpu().numpy(), up[rows].cpu().numpy()
    dys, dhs = dy[rows].cpu().numpy(), dh[rows].cpu().numpy()

    def rms_run():
        xt, wt = oracle.from_numpy(xs, True), oracle.from_numpy(ws_, True)
        yy = oracle.rms_norm(xt, wt, 1e-6)
        yy.backward(dys)
        return yy.numpy(), xt.grad.numpy()
    (y_ref, dx_ref), (by, bdx) = reference_budget(oracle, rms_run, libm=())
    assert_close(_host(y[rows]), y_ref, atol=ATOL + by, what="y rows")
    assert_close(_host(dx[rows]), dx_ref, atol=ATOL + bdx, what="dx rows")

    (h_ref, dg_ref, du_ref), (bh, bdg, bdu) = _oracle_swiglu(oracle, gs, us, dhs)
    assert_close(_host(h[rows]), h_ref, atol=ATOL + bh, what="h rows")
    assert_close(_host(dg[rows]), dg_ref, atol=ATOL + bdg, what="dg rows")
    assert_close(_host(du[rows]), du_ref, atol=ATOL + bdu, what="du rows")
    hr = _host(h[rows])
    assert_bitexact(_host(hm[rows]), oracle.t_reduce("max", hr, 1, False), "row max")
    assert_bitexact(_host(ha[rows]), oracle.t_reduce("argmax", hr, 1, False), "row argmax")
    assert_close(_host(hs[rows]), oracle.t_reduce("sum", hr, 1, False),
                 atol=ATOL * np.abs(hr).sum(1) + 1e-6, what="row sum",
                 strict_atol=ATOL * np.abs(hr).sum(1) + 1e-6)

    # dweight over all rows vs float64 (REF semantics: sum dy * x * inv)
    dw64 = torch.zeros(D, dtype=torch.float64, device="cuda")
    absw = torch.zeros(D, dtype=torch.float64, device="cuda")
    for i in range(0, M, 8192):
        xx = x[i:i + 8192].double()
        inv = torch.rsqrt((xx * xx).mean(1, keepdim=True) + 1e-6)
        t = dy[i:i + 8192].double() * xx * inv
        dw64 += t.sum(0)
        absw += t.abs().sum(0)
    assert_close(_host(dw), dw64.cpu().numpy(), rtol=RTOL_BIG,
                 atol=ATOL * np.maximum(absw.cpu().numpy(), 1.0), what="dweight vs f64",
                 strict_atol=ATOL * np.maximum(absw.cpu().numpy(), 1.0))
    # L2 over {dx, dg, du} vs float64 torch
    want = sum(float((t.double() ** 2).sum().item()) for t in (dx, dg, du)) ** 0.5
    assert abs(l2 - want) <= 1e-6 * want, (l2, want)
