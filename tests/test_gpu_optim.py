"""The optimizer step on the device (oxc_sgd_step / oxc_adamw_step and the
oxitorch_b200.optim classes) against the oracle restatement of
crates/oxi-autograd/src/optim.rs.

Every update is a sequence of individually rounded f32 operations in the
reference's order, so results must be bit-identical to the oracle, on both
the 128-bit path and the scalar path (a parameter 4 bytes off 16-byte
alignment, and sizes that are not multiples of 4), over several steps.  The
reference's own optimizer test scenarios (optim.rs:314-447) run through the
Python classes, with the reference's errors."""

import numpy as np
import pytest

from parity import assert_bitexact

pytestmark = pytest.mark.gpu


def _buf(a, misalign):
    """Device copy of a; with misalign the data starts 4 bytes past a
    16-byte boundary (the scalar path)."""
    import torch
    off = 1 if misalign else 0
    t = torch.zeros(a.size + off + 3, dtype=torch.float32, device="cuda")
    v = t[off:off + a.size]
    v.copy_(torch.from_numpy(np.ascontiguousarray(a)))
    return v


def _host(t):
    return t.detach().cpu().numpy()


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("n,misalign", [(1000003, False), (4096, True), (5, False), (1, True)])
@pytest.mark.parametrize("momentum,nesterov", [(0.0, False), (0.9, False), (0.9, True)])
def test_sgd_kernel_bitexact(oracle, n, misalign, momentum, nesterov):
    from oxitorch_b200 import _native as N
    L = N.load()
    rng = np.random.default_rng(n + int(10 * momentum) + nesterov)
    p = rng.standard_normal(n).astype(np.float32)
    dp, dv = _buf(p, misalign), _buf(np.zeros(n, np.float32), misalign)
    buf = None
    for step in range(3):
        g = rng.standard_normal(n).astype(np.float32)
        dg = _buf(g, misalign)
        N.check(L.oxc_sgd_step(dp.data_ptr(), dg.data_ptr(), dv.data_ptr() if momentum else None,
                               n, 0.1, momentum, int(nesterov), _stream()), "sgd")
        p, buf = oracle.sgd_step(p, g, buf, 0.1, momentum, nesterov)
        assert_bitexact(_host(dp), p, f"param step {step}")
        if momentum:
            assert_bitexact(_host(dv), buf, f"velocity step {step}")


@pytest.mark.parametrize("n,misalign", [(1000003, False), (4096, True), (7, False)])
@pytest.mark.parametrize("decoupled,wd", [(True, 0.01), (True, 0.0), (False, 0.01), (False, 0.0)])
def test_adam_kernel_bitexact(oracle, n, misalign, decoupled, wd):
    from oxitorch_b200 import _native as N
    L = N.load()
    rng = np.random.default_rng(n + int(decoupled) + int(wd * 100))
    p = rng.standard_normal(n).astype(np.float32)
    dp = _buf(p, misalign)
    dm, dv = _buf(np.zeros(n, np.float32), misalign), _buf(np.zeros(n, np.float32), misalign)
    m = v = None
    for t in (1, 2, 3):
        g = (rng.standard_normal(n) * 0.1).astype(np.float32)
        dg = _buf(g, misalign)
        N.check(L.oxc_adamw_step(dp.data_ptr(), dg.data_ptr(), dm.data_ptr(), dv.data_ptr(), n,
                                 1e-3, 0.9, 0.999, 1e-8, wd, int(decoupled), t, _stream()), "adam")
        p, m, v = oracle.adamw_step(p, g, m, v, 1e-3, 0.9, 0.999, 1e-8, wd, decoupled, t)
        assert_bitexact(_host(dp), p, f"param t={t}")
        assert_bitexact(_host(dm), m, f"m t={t}")
        assert_bitexact(_host(dv), v, f"v t={t}")


def test_kernel_argument_errors():
    from oxitorch_b200 import _native as N
    L = N.load()
    d = _buf(np.ones(8, np.float32), False)
    assert L.oxc_sgd_step(d.data_ptr(), d.data_ptr(), None, 8, 0.1, 0.0, 1, _stream()) == 1
    assert "nesterov momentum requires momentum > 0" in N.last_error()
    assert L.oxc_adamw_step(d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), 8, 0.1, 0.9,
                            0.999, 1e-8, 0.0, 1, 0, _stream()) == 1
    assert L.oxc_sgd_step(None, None, None, 0, 0.1, 0.0, 0, _stream()) == 0  # empty: no-op


# ---- the Python classes: the reference's optimizer test scenarios ---------------------------

def _param(vals, grad=None):
    import torch
    p = torch.tensor(vals, dtype=torch.float32, device="cuda", requires_grad=True)
    if grad is not None:
        p.grad = torch.tensor(grad, dtype=torch.float32, device="cuda")
    return p


def test_sgd_momentum_matches_reference():
    from oxitorch_b200 import optim
    p = _param([1.0])
    opt = optim.Sgd([p], lr=0.1, momentum=0.9)
    for want in (1.0 - 0.05, 0.95 - 0.095, 0.855 - 0.1355):
        p.grad = _param([0.5]).detach()
        opt.step()
        assert abs(float(p.detach().cpu()[0]) - want) < 1e-6


def test_sgd_nesterov_and_its_error():
    from oxitorch_b200 import optim
    p = _param([1.0], [0.5])
    optim.Sgd([p], lr=0.1, momentum=0.9, nesterov=True).step()
    assert abs(float(p.detach().cpu()[0]) - (1.0 - 0.1 * 0.95)) < 1e-6
    with pytest.raises(ValueError, match="nesterov momentum requires momentum > 0"):
        optim.Sgd([p], lr=0.1, momentum=0.0, nesterov=True)


def test_skipped_params_keep_state_and_counters(oracle):
    """SGD: a parameter without a gradient gets no stale velocity.  AdamW: a
    parameter that skipped a step starts its bias correction at t = 1."""
    import torch
    from oxitorch_b200 import optim
    a, b = _param([1.0], [0.5]), _param([1.0])
    opt = optim.Sgd([a, b], lr=0.1, momentum=0.9)
    opt.step()                         # b has no gradient yet
    a.grad = torch.full_like(a, 0.5)
    b.grad = torch.full_like(b, 0.5)
    opt.step()
    assert abs(float(b.detach().cpu()[0]) - 0.95) < 1e-6
    assert abs(float(a.detach().cpu()[0]) - (0.95 - 0.095)) < 1e-6
    a, b = _param([1.0], [0.5]), _param([1.0])
    opt = optim.AdamW([a, b], lr=0.1, weight_decay=0.0)
    opt.step()
    b.grad = torch.full_like(b, 0.5)
    a.grad = None
    opt.step()
    want, _, _ = oracle.adamw_step(np.ones(1, np.float32), np.full(1, 0.5, np.float32), None, None,
                                   0.1, 0.9, 0.999, 1e-8, 0.0, True, 1)
    assert_bitexact(_host(b), want, "second parameter's first step uses t = 1")


def test_adamw_and_adam_multi_param_bitexact(oracle):
    """A parameter list (a matrix, a vector, and one left with the zero gradient
    zero_grad gives it, which still counts as a step) over three steps,
    against the oracle."""
    import torch
    from oxitorch_b200 import optim
    rng = np.random.default_rng(5)
    for cls, decoupled in ((optim.AdamW, True), (optim.Adam, False)):
        vals = [rng.standard_normal((33, 17)).astype(np.float32),
                rng.standard_normal(101).astype(np.float32),
                rng.standard_normal(3).astype(np.float32)]
        ps = [_param(v.tolist()) for v in vals]
        opt = cls(ps, lr=3e-3, weight_decay=0.05)
        ref = [(v.reshape(-1), None, None, 0) for v in vals]
        for step in range(3):
            opt.zero_grad()
            for i in (0, 1):  # parameter 2 keeps a zero gradient
                g = rng.standard_normal(vals[i].shape).astype(np.float32)
                ps[i].grad = torch.from_numpy(g).cuda()
            for i in range(3):
                g = _host(ps[i].grad).reshape(-1)
                pv, m, v, t = ref[i]
                pv, m, v = oracle.adamw_step(pv, g, m, v, opt.lr, 0.9, 0.999, 1e-8, 0.05,
                                             decoupled, t + 1)
                ref[i] = (pv, m, v, t + 1)
            opt.step()
            for i in range(3):
                assert_bitexact(_host(ps[i]).reshape(-1), ref[i][0], f"{cls.__name__} p{i} s{step}")


def test_lr_is_f32_and_state_size_mismatch_raises():
    import torch
    from oxitorch_b200 import optim
    p = _param([1.0, 2.0], [0.5, 0.5])
    opt = optim.Sgd([p], lr=0.1, momentum=0.9)
    assert opt.lr == float(np.float32(0.1))
    opt.lr = 0.3
    assert opt.lr == float(np.float32(0.3))
    opt.step()
    q = _param([1.0, 2.0, 3.0], [0.5, 0.5, 0.5])
    opt.params = [q]
    with pytest.raises(ValueError, match="the parameter set changed mid-run"):
        opt.step()
    cpu = torch.ones(2, requires_grad=True)
    cpu.grad = torch.ones(2)
    with pytest.raises(ValueError, match="CUDA"):
        optim.Sgd([cpu]).step()
