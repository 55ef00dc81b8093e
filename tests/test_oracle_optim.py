"""The oracle's optimizer step against the reference's own optimizer tests
(crates/oxi-autograd/src/optim.rs, tests module, lines 314-447), at the
tolerances those tests use.  Scenario by scenario: SGD momentum over three
steps, Nesterov look-ahead, a parameter skipped on a step keeping no stale
velocity, AdamW against its closed form over two steps, classic Adam folding
decay into the gradient, and per-parameter step counters across a skip."""

import math

import numpy as np

from oracle import oxiref as O


def _s(x):
    return np.array([x], np.float32)


def test_sgd_momentum_matches_reference():
    val, buf = _s(1.0), None
    for want in (1.0 - 0.05, 0.95 - 0.095, 0.855 - 0.1355):
        val, buf = O.sgd_step(val, _s(0.5), buf, 0.1, 0.9, False)
        assert abs(float(val[0]) - want) < 1e-6


def test_sgd_nesterov_uses_lookahead():
    val, _ = O.sgd_step(_s(1.0), _s(0.5), None, 0.1, 0.9, True)
    assert abs(float(val[0]) - (1.0 - 0.1 * 0.95)) < 1e-6


def test_sgd_skipped_param_keeps_velocity():
    # step 1: only the first parameter has a gradient; step 2: both do, and
    # the second starts from a fresh (zero) velocity
    p0, b0 = O.sgd_step(_s(1.0), _s(0.5), None, 0.1, 0.9, False)
    p0, b0 = O.sgd_step(_s(0.95), _s(0.5), b0, 0.1, 0.9, False)
    p1, _ = O.sgd_step(_s(1.0), _s(0.5), None, 0.1, 0.9, False)
    assert abs(float(p1[0]) - 0.95) < 1e-6
    assert abs(float(p0[0]) - (0.95 - 0.095)) < 1e-6


def test_adamw_two_steps_match_closed_form():
    lr, b1, b2, eps, wd, grad = 0.1, 0.9, 0.999, 1e-8, 0.1, 0.5
    val, moment, vel = 1.0, 0.0, 0.0
    p, m, v = _s(1.0), None, None
    for step in (1, 2):
        moment = b1 * moment + (1.0 - b1) * grad
        vel = b2 * vel + (1.0 - b2) * grad * grad
        m_hat = moment / (1.0 - b1 ** step)
        v_hat = vel / (1.0 - b2 ** step)
        want = val - lr * m_hat / (math.sqrt(v_hat) + eps) - lr * wd * val
        p, m, v = O.adamw_step(np.float32(val) * np.ones(1, np.float32), _s(grad), m, v,
                               lr, b1, b2, eps, wd, True, step)
        assert abs(float(p[0]) - want) < 1e-5, (step, float(p[0]), want)
        val = want


def test_adam_classic_decay_folds_into_gradient():
    start, grad, wd = np.float32(1.0), np.float32(0.5), np.float32(0.1)
    g_eff = grad + wd * start
    moment = np.float32(1.0 - 0.9) * g_eff
    vel = np.float32(1.0 - 0.999) * g_eff * g_eff
    m_hat = moment / np.float32(1.0 - 0.9)
    v_hat = vel / np.float32(1.0 - 0.999)
    want = start - np.float32(0.1) * m_hat / (np.sqrt(v_hat) + np.float32(1e-8))
    p, _, _ = O.adamw_step(_s(1.0), _s(0.5), None, None, 0.1, 0.9, 0.999, 1e-8, 0.1, False, 1)
    assert abs(float(p[0]) - float(want)) < 1e-5


def test_per_param_step_counters_track_skips():
    # the second parameter skipped step 1; its first real step uses t = 1
    p, _, _ = O.adamw_step(_s(1.0), _s(0.5), None, None, 0.1, 0.9, 0.999, 1e-8, 0.0, True, 1)
    grad = 0.5
    moment, vel = 0.1 * grad, 0.001 * grad * grad
    want = 1.0 - 0.1 * (moment / 0.1) / (math.sqrt(vel / 0.001) + 1e-8)
    assert abs(float(p[0]) - want) < 1e-5


def test_bias_correction_uses_powf_per_step():
    """The bias corrections 1 - beta^t come from C powf at each step's t."""
    for t in (1, 2, 7, 1000):
        assert abs(float(O._powf(0.9, t)) - float(np.float32(0.9)) ** t) < 1e-6 * 0.9 ** t + 1e-30
