"""The CPU oracle against the reference's own known answers.

Literal cases live in tests/golden/reference_kats.json (each cites the
reference test it comes from); formula cases restate the assertions of the
reference's python/tests/test_nn.py and test_smoke.py.
"""

import json
import os

import numpy as np
import pytest

from parity import assert_close

HERE = os.path.dirname(os.path.abspath(__file__))
KATS = json.load(open(os.path.join(HERE, "golden", "reference_kats.json")))


def _arr(v, shape=None):
    a = np.asarray(v, dtype=np.float32)
    return a.reshape(shape) if shape is not None else a


@pytest.mark.parametrize("case", KATS["reduce_strip"], ids=lambda c: c["src"])
def test_reduce_strip(oracle, case):
    data = _arr(case["data"])
    for kind, want in case.get("want", {}).items():
        assert oracle.t_reduce_strip_all(kind, data) == np.float32(want)
    for kind, err in case.get("error", {}).items():
        with pytest.raises(oracle.InvalidArgument):
            oracle.t_reduce_strip_all(kind, data)


@pytest.mark.parametrize("case", KATS["registry_scalar"], ids=lambda c: c["src"])
def test_registry_scalar(oracle, case):
    a = _arr([case["a"]])
    if case["kind"] == "unary":
        got = oracle.t_unary(case["op"], a)
    elif case["kind"] == "binary":
        got = oracle.t_binary(case["op"], a, _arr([case["b"]]))
    else:
        got = oracle.t_cmp(case["op"], a, _arr([case["b"]]))
    assert got[0] == np.float32(case["want"])


@pytest.mark.parametrize("case", KATS["binary"], ids=lambda c: c["src"])
def test_binary(oracle, case):
    a = _arr(case["a"], case["a_shape"])
    b = _arr(case["b"], case["b_shape"])
    if "error" in case:
        with pytest.raises(oracle.ShapeMismatch):
            oracle.t_binary(case["op"], a, b)
        return
    got = oracle.t_binary(case["op"], a, b)
    assert list(got.shape) == case["out_shape"]
    np.testing.assert_array_equal(got.reshape(-1), _arr(case["want"]))


def test_unknown_ops(oracle):
    for case in KATS["unknown_op"]:
        assert case["op"] not in oracle.BINARY_OPS
    with pytest.raises(oracle.InvalidArgument):
        oracle.t_unary("frobnicate", _arr([1.0]))


def test_cmp(oracle):
    for case in KATS["cmp"]:
        for op, want in case["want"].items():
            got = oracle.t_cmp(op, _arr(case["a"]), _arr(case["b"]))
            np.testing.assert_array_equal(got, _arr(want))


@pytest.mark.parametrize("case", KATS["reduce"], ids=lambda c: c["src"])
def test_reduce(oracle, case):
    a = _arr(case["data"], case["shape"])
    if "error" in case:
        with pytest.raises(oracle.InvalidArgument):
            oracle.t_reduce(case["kind"], a, case["dim"], case["keepdim"])
        return
    got = oracle.t_reduce(case["kind"], a, case["dim"], case["keepdim"])
    assert list(got.shape) == case["out_shape"]
    if "atol" in case:
        assert_close(got.reshape(-1), _arr(case["want"]), rtol=0, atol=case["atol"])
    else:
        np.testing.assert_array_equal(got.reshape(-1), _arr(case["want"]))


def test_reduce_all(oracle):
    for case in KATS["reduce_all"]:
        t = oracle.from_numpy(_arr(case["data"], case["shape"]))
        assert t.mean().item() == case["want"]["mean"]
        assert t.sum().item() == case["want"]["sum"]


@pytest.mark.parametrize("case", KATS["index_select"], ids=lambda c: c["src"])
def test_index_select(oracle, case):
    a = _arr(case["data"], case["shape"])
    if "error" in case:
        with pytest.raises(oracle.OutOfBounds, match="out of range for dim 0 of size"):
            oracle.t_index_select(a, case["dim"], case["ids"])
        return
    got = oracle.t_index_select(a, case["dim"], case["ids"])
    assert list(got.shape) == case["out_shape"]
    np.testing.assert_array_equal(got.reshape(-1), _arr(case["want"]))


@pytest.mark.parametrize("case", KATS["embedding_grad"], ids=lambda c: c["src"])
def test_embedding_grad(oracle, case):
    table = oracle.from_numpy(_arr(case["table"], case["table_shape"]), True)
    out = table.index_select(0, case["ids"])
    if "want_out" in case:
        np.testing.assert_array_equal(out.numpy().reshape(-1), _arr(case["want_out"]))
    if case["seed"] == "ones":
        out.sum().backward()
    else:
        out.backward(_arr(case["seed"], out.shape))
    np.testing.assert_array_equal(table.grad.numpy().reshape(-1), _arr(case["want_grad"]))


# ---- formula known answers (python/tests/test_nn.py) ------------------------------

def _t(oracle, a, rg=False):
    return oracle.from_numpy(np.asarray(a, dtype=np.float32), rg)


def test_softmax_log_softmax_values(oracle):
    """test_nn.py:30-37."""
    x = _t(oracle, [[1.0, 2.0, 3.0], [3.0, 1.0, 2.0]])
    xr = x.numpy()
    ref = np.exp(xr) / np.exp(xr).sum(-1, keepdims=True)
    assert np.allclose(oracle.softmax(x, -1).numpy(), ref, atol=1e-6)
    ls = oracle.log_softmax(x, -1).numpy()
    assert np.allclose(np.exp(ls).sum(-1), 1.0, atol=1e-6)


def test_log_softmax_stability(oracle):
    """test_nn.py:40-48."""
    ls = oracle.log_softmax(_t(oracle, [[1000.0, 1001.0, 1002.0]]), -1).numpy()
    assert np.all(np.isfinite(ls))
    sm = np.exp(ls)
    sm = sm / sm.sum()
    want = np.exp(np.array([1000.0, 1001.0, 1002.0]) - 1002.0)
    assert np.allclose(sm, want / want.sum(), atol=1e-6)


def test_activation_values(oracle):
    """test_nn.py:51-60."""
    x = _t(oracle, [-1.0, 0.0, 1.0, 2.0])
    r = x.numpy()
    assert np.allclose(x.apply("relu").numpy(), np.maximum(r, 0), atol=1e-7)
    assert np.allclose(x.apply("sigmoid").numpy(), 1 / (1 + np.exp(-r)), atol=1e-6)
    assert np.allclose(x.apply("tanh").numpy(), np.tanh(r), atol=1e-6)
    assert np.allclose(oracle.silu(x).numpy(), r / (1 + np.exp(-r)), atol=1e-6)
    c = np.sqrt(2 / np.pi)
    assert np.allclose(oracle.gelu(x).numpy(), 0.5 * r * (1 + np.tanh(c * (r + 0.044715 * r**3))),
                       atol=1e-5)


def test_layer_norm_value_and_grad(oracle):
    """test_nn.py:63-78."""
    x = _t(oracle, [[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]], True)
    w = _t(oracle, [1.0, 1.0, 1.0], True)
    b = _t(oracle, [0.0, 0.0, 0.0], True)
    out = oracle.layer_norm(x, w, b)
    xr = x.numpy()
    mu = xr.mean(-1, keepdims=True)
    v = ((xr - mu) ** 2).mean(-1, keepdims=True)
    assert np.allclose(out.numpy(), (xr - mu) / np.sqrt(v + 1e-5), rtol=1e-4, atol=1e-5)
    coef = np.array([[1.0, -2.0, 0.5], [0.25, 1.0, -1.0]], dtype=np.float32)
    (out * _t(oracle, coef)).sum().backward()
    assert x.grad is not None and w.grad is not None and b.grad is not None
    assert np.abs(x.grad.numpy()).sum() > 1e-6


def test_rms_norm_value(oracle):
    """test_nn.py:81-87."""
    x = _t(oracle, [[1.0, -2.0, 3.0]])
    w = _t(oracle, [1.0, 2.0, 0.5])
    xr = x.numpy()
    ref = xr / np.sqrt((xr**2).mean(-1, keepdims=True) + 1e-6) * np.array([[1.0, 2.0, 0.5]])
    assert np.allclose(oracle.rms_norm(x, w).numpy(), ref, rtol=1e-4, atol=1e-5)


def test_cross_entropy_value_and_grad(oracle):
    """test_nn.py:111-122."""
    logits = _t(oracle, [[1.0, 2.0, 3.0], [3.0, 1.0, 2.0]], True)
    loss = oracle.cross_entropy(logits, [2, 0])
    lg = logits.numpy()
    m = lg.max(-1, keepdims=True)
    ls = lg - m - np.log(np.exp(lg - m).sum(-1, keepdims=True))
    assert abs(loss.item() - (-np.mean([ls[0, 2], ls[1, 0]]))) < 1e-5
    loss.backward()
    g = (np.exp(ls) - np.eye(3, dtype=np.float32)[[2, 0]]) / 2
    assert np.allclose(logits.grad.numpy(), g, rtol=1e-4, atol=1e-6)


def test_cross_entropy_rejects_wrong_batch(oracle):
    """test_nn.py:125-128."""
    with pytest.raises(ValueError, match="targets"):
        oracle.cross_entropy(_t(oracle, np.zeros((2, 3))), [0, 1, 2])


def test_reduction_parity_smoke(oracle):
    """test_smoke.py:107-121 (RTOL 1e-5, ATOL 1e-6 there)."""
    rng = np.random.default_rng(0x5EED)
    a = rng.standard_normal((3, 4, 5)).astype(np.float32)
    t = _t(oracle, a)
    np.testing.assert_allclose(t.sum(0).numpy(), a.sum(0), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(t.sum(-1).numpy(), a.sum(-1), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(t.mean(1).numpy(), a.mean(1), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(t.max(0).numpy(), a.max(0), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(t.min(2).numpy(), a.min(2), rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(t.argmax(-1).numpy(), a.argmax(-1))
    np.testing.assert_array_equal(t.argmin(1).numpy(), a.argmin(1))
    np.testing.assert_allclose(t.norm(-1, False).numpy(), np.linalg.norm(a, axis=-1), rtol=1e-5,
                               atol=1e-6)
    assert t.sum().item() == pytest.approx(float(a.sum()), rel=1e-5)


def test_sign_of_zero_is_one(oracle):
    """Rust f32::signum (crates/oxi-tensor/src/ops.rs:192) never returns 0."""
    got = oracle.t_unary("sign", np.array([0.0, -0.0, 2.0, -3.0], np.float32))
    np.testing.assert_array_equal(got, [1.0, -1.0, 1.0, -1.0])
