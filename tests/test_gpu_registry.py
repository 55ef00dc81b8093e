"""Elementwise registry ops and reductions on the device vs the oracle.

* IEEE-exact ops (+ - * / sqrt rsqrt square reciprocal neg abs relu floor ceil
  round sign min max) and all comparisons: bit-exact, NaN patterns included.
* libm ops (exp log log2 log10 sin cos tanh sigmoid pow): within a stated
  number of ulps of the oracle's glibc results (CUDA's documented maximum
  error plus glibc's).
* reductions: max/min/argmax/argmin bit-exact (NaN and tie rules of
  f32::max and first-occurrence argmax); column-mode sums/means/norms
  bit-exact (same left-to-right order as the reference); tree-order sums
  within rtol 1e-5 (1e-4 from 32k elements) plus the reference's own
  summation-order error, and on long rows 1e-6 x sum|terms| (a reordered sum
  of cancelling terms).
"""

import json
import os

import numpy as np
import pytest

from parity import ATOL, RTOL, RTOL_BIG, assert_bitexact, assert_close

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
EXACT_UNARY = ["neg", "abs", "sqrt", "rsqrt", "relu", "floor", "ceil", "round", "sign", "square",
               "reciprocal"]
LIBM_ULPS = {"exp": 3, "log": 2, "log2": 3, "log10": 3, "sin": 3, "cos": 3, "tanh": 4,
             "sigmoid": 4}


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    return t.detach().cpu().numpy()


def _ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7fffffff), a)
    b = np.where(b < 0, -(b & 0x7fffffff), b)
    return np.abs(a - b)


def _assert_ulps(got, want, ulps, what):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert (np.isnan(got) == np.isnan(want)).all(), f"{what}: NaN pattern"
    fin = ~np.isnan(want)
    assert (np.isinf(got[fin]) == np.isinf(want[fin])).all(), f"{what}: inf pattern"
    d = _ulps(got[fin], want[fin])
    assert d.max(initial=0) <= ulps, f"{what}: {d.max()} ulps (limit {ulps})"


def _values(seed, n):
    rng = np.random.default_rng(seed)
    v = np.concatenate([
        rng.standard_normal(n).astype(np.float32) * 3,
        rng.uniform(-100, 100, n // 4).astype(np.float32),
        np.exp(rng.uniform(-30, 30, n // 4)).astype(np.float32),
        np.array([0.0, -0.0, 1.0, -1.0, 0.5, -0.5, 1.5, -2.5, np.inf, -np.inf, np.nan,
                  1e-40, -1e-40, 3.4e38, 88.0, -104.0], np.float32)])
    return v.astype(np.float32)


@pytest.mark.parametrize("name", EXACT_UNARY + list(LIBM_ULPS))
def test_unary_ops(oracle, name):
    from oxitorch_b200 import tensor_ops as T
    x = _values(hash(name) % 1000, 4096)
    got = _host(T.unary_op(name, _dev(x)))
    want = oracle.t_unary(name, x)
    if name in EXACT_UNARY:
        if name == "relu":  # f32::max(-0.0, 0.0) may return either zero
            got, want = got + 0.0, want + 0.0
        assert_bitexact(got, want, name)
    else:
        _assert_ulps(got, want, LIBM_ULPS[name], name)


@pytest.mark.parametrize("name", ["add", "sub", "mul", "div", "min", "max", "pow"])
def test_binary_ops_broadcast_and_strided(oracle, name):
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(7)
    a = rng.standard_normal((37, 50), dtype=np.float32)
    b = rng.standard_normal((50,), dtype=np.float32)
    if name == "pow":
        a = np.abs(a) + np.float32(0.1)
    cases = [
        (a, b),                                   # row broadcast
        (a, b[:37].reshape(37, 1)),               # column broadcast
        (a, a.T.copy().T),                        # transposed (column-major) view
        (a[::2, 1::3], a[::2, ::3]),              # stepped slices
        (np.float32(1.5) * np.ones((), np.float32), a),  # 0-d operand
    ]
    for i, (x, y) in enumerate(cases):
        xd, yd = _dev(x), _dev(y)
        if i == 2:
            yd = _dev(np.ascontiguousarray(a.T)).t()   # a genuine strided view
        if i == 3:
            xd = _dev(a)[::2, 1::3]
            yd = _dev(a)[::2, ::3]
        got = _host(T.binary_op(name, xd, yd))
        want = oracle.t_binary(name, np.asarray(x, np.float32), np.asarray(y, np.float32))
        if name == "pow":
            _assert_ulps(got, want, 6, f"{name} case {i}")
        else:
            assert_bitexact(got, want, f"{name} case {i}")


@pytest.mark.parametrize("name", ["add", "sub", "mul", "div"])
def test_binary_scalar_both_sides(oracle, name):
    from oxitorch_b200 import tensor_ops as T
    x = _values(3, 1000)[:1003]
    xd = _dev(x.reshape(17, 59))
    xt = _dev(np.ascontiguousarray(x.reshape(17, 59).T)).t()
    for t in (xd, xt):
        got = _host(T.binary_op(name, t, 2.5))
        assert_bitexact(got, oracle.t_binary(name, x.reshape(17, 59), np.float32(2.5)), name)
        got = _host(T.binary_op(name, 2.5, t))
        assert_bitexact(got, oracle.t_binary(name, np.float32(2.5), x.reshape(17, 59)), name)


def _transposed(x, pad=0):
    """Device view of x [R, C] that is column-major: the transpose of a
    [C, R + pad] buffer (column stride R + pad)."""
    import torch
    r, c = x.shape
    buf = torch.zeros(c, r + pad, device="cuda")
    buf[:, :r] = _dev(np.ascontiguousarray(x.T))
    return buf[:, :r].t()


@pytest.mark.parametrize("shape", [(300, 1100), (33, 196), (1000, 388)])
def test_transposed_operand_paths(oracle, shape):
    """One column-major input with 16-byte aligned columns takes the tile
    pipeline (TMA boxes for the transposed input); a misaligned column stride
    takes the 32x32 tiles.  Every result must match the oracle on the dense
    values: unary ops, both operand orders of non-commutative binaries, and
    scalars on either side."""
    from oxitorch_b200 import tensor_ops as T
    r, c = shape
    x = _values(r + c, r * c)[: r * c].reshape(r, c)
    y = np.random.default_rng(c).standard_normal((r, c)).astype(np.float32)
    for pad in (0, 1):  # pad 1: column stride r + 1, not a multiple of 4
        xt = _transposed(x, pad)
        assert xt.stride() == (1, r + pad)
        for name in ("neg", "sqrt", "reciprocal", "sigmoid", "exp"):
            got = _host(T.unary_op(name, xt))
            want = oracle.t_unary(name, x)
            if name in EXACT_UNARY:
                assert_bitexact(got, want, f"{name} pad {pad}")
            else:
                _assert_ulps(got, want, LIBM_ULPS[name], f"{name} pad {pad}")
        for name in ("sub", "div", "max", "mul"):
            assert_bitexact(_host(T.binary_op(name, xt, _dev(y))), oracle.t_binary(name, x, y),
                            f"{name}(T, dense) pad {pad}")
            assert_bitexact(_host(T.binary_op(name, _dev(y), xt)), oracle.t_binary(name, y, x),
                            f"{name}(dense, T) pad {pad}")
            assert_bitexact(_host(T.binary_op(name, xt, 1.75)),
                            oracle.t_binary(name, x, np.float32(1.75)), f"{name}(T, s) pad {pad}")
            assert_bitexact(_host(T.binary_op(name, 1.75, xt)),
                            oracle.t_binary(name, np.float32(1.75), x), f"{name}(s, T) pad {pad}")
        got = _host(T.cmp_op("lt", xt, _dev(y)))
        assert_bitexact(got, oracle.t_cmp("lt", x, y), f"lt(T, dense) pad {pad}")


@pytest.mark.parametrize("pad", [0, 1])
def test_transposed_every_op(oracle, pad):
    """Every unary op, and every binary op with a scalar on either side, on a
    column-major view: pad 0 takes the tile pipeline, whose consumers select
    one op-specialised loop per tile; pad 1 the 32x32 tiles."""
    from oxitorch_b200 import tensor_ops as T
    r, c = 257, 392
    x = _values(5, r * c)[: r * c].reshape(r, c)
    xt = _transposed(x, pad)
    for name in EXACT_UNARY + list(LIBM_ULPS):
        got = _host(T.unary_op(name, xt))
        want = oracle.t_unary(name, x)
        if name in EXACT_UNARY:
            if name == "relu":  # f32::max(-0.0, 0.0) may return either zero
                got, want = got + 0.0, want + 0.0
            assert_bitexact(got, want, f"{name} pad {pad}")
        else:
            _assert_ulps(got, want, LIBM_ULPS[name], f"{name} pad {pad}")
    for name in ("add", "sub", "mul", "div", "min", "max", "pow"):
        for s, first in ((1.75, False), (-0.5, True)):
            got = _host(T.binary_op(name, s, xt) if first else T.binary_op(name, xt, s))
            want = (oracle.t_binary(name, np.float32(s), x) if first
                    else oracle.t_binary(name, x, np.float32(s)))
            if name == "pow":
                _assert_ulps(got, want, 6, f"pow pad {pad} scalar first {first}")
            else:
                assert_bitexact(got, want, f"{name} pad {pad} scalar first {first}")


def test_cmp_ops_bitexact(oracle):
    from oxitorch_b200 import tensor_ops as T
    x = _values(11, 2000)
    y = np.roll(x, 7)
    y[::5] = x[::5]  # equal pairs
    for name in T.CMP_OPS:
        got = _host(T.cmp_op(name, _dev(x), _dev(y)))
        assert_bitexact(got, oracle.t_cmp(name, x, y), name)


def test_registry_known_answers():
    from oxitorch_b200 import tensor_ops as T
    kats = json.load(open(os.path.join(HERE, "golden", "reference_kats.json")))
    for c in kats["binary"]:
        a = _dev(np.asarray(c["a"], np.float32).reshape(c["a_shape"]))
        b = _dev(np.asarray(c["b"], np.float32).reshape(c["b_shape"]))
        if "error" in c:
            with pytest.raises(ValueError, match="shape mismatch"):
                T.binary_op(c["op"], a, b)
            continue
        got = T.binary_op(c["op"], a, b)
        assert list(got.shape) == c["out_shape"], c["src"]
        np.testing.assert_array_equal(_host(got).reshape(-1), c["want"], err_msg=c["src"])
    for c in kats["cmp"]:
        for op, want in c["want"].items():
            got = _host(T.cmp_op(op, _dev(np.asarray(c["a"], np.float32)), _dev(np.asarray(c["b"], np.float32))))
            np.testing.assert_array_equal(got, want, err_msg=c["src"])
    for c in kats["registry_scalar"]:
        a = _dev(np.asarray([c["a"]], np.float32))
        if c["kind"] == "unary":
            got = T.unary_op(c["op"], a)
        elif c["kind"] == "binary":
            got = T.binary_op(c["op"], a, _dev(np.asarray([c["b"]], np.float32)))
        else:
            got = T.cmp_op(c["op"], a, _dev(np.asarray([c["b"]], np.float32)))
        assert float(_host(got)[0]) == c["want"], c["src"]
    with pytest.raises(ValueError, match="unknown binary op"):
        T.binary_op("frob", a, a)


# ---- reductions --------------------------------------------------------------------------

def _red_inputs():
    rng = np.random.default_rng(5)
    a = rng.standard_normal((6, 300, 70), dtype=np.float32)
    a[2, 5, :] = 3.0  # ties for argmax/argmin
    return a


@pytest.mark.parametrize("kind", ["sum", "mean", "max", "min", "argmax", "argmin", "norm"])
@pytest.mark.parametrize("dim", [0, 1, 2, -1])
@pytest.mark.parametrize("keepdim", [False, True])
def test_reduce_all_kinds_dims(oracle, kind, dim, keepdim):
    from oxitorch_b200 import tensor_ops as T
    a = _red_inputs()
    for view_name, host, dev in [("dense", a, _dev(a)),
                                 ("permuted", np.ascontiguousarray(a.transpose(2, 0, 1)),
                                  _dev(a).permute(2, 0, 1))]:
        got = _host(T.reduce(kind, dev, dim, keepdim))
        want = oracle.t_reduce(kind, host, dim, keepdim)
        assert got.shape == want.shape
        what = f"{kind} dim={dim} keepdim={keepdim} {view_name}"
        if kind in ("max", "min", "argmax", "argmin"):
            assert_bitexact(got, want, what)
        else:
            oracle.PRECISE_SUMS[0] = True
            exact = oracle.t_reduce(kind, host, dim, keepdim)
            oracle.PRECISE_SUMS[0] = False
            budget = np.abs(want.astype(np.float64) - exact)
            assert_close(got, want, rtol=RTOL, atol=ATOL + budget, what=what)


@pytest.mark.parametrize("shape", [(9600, 2100), (500, 4100)])
def test_reduce_long_rows_both_geometries(oracle, shape):
    """Rows of 2048+ elements over dim 1: with at least 64 outputs per SM
    (9600 rows on 148 SMs) a warp takes each output, with fewer (500 rows) a
    CTA.  Every kind against the oracle; ties and NaNs placed in some rows.
    The kernels sum in a tree, the reference left to right, so sums are held
    to 1e-6 x sum|terms| per row (the column-sum convention of tests/parity.py):
    a row of 2100 N(0,1) values can sum to ~1 with sum|x| ~ 1700."""
    import torch
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(shape[0])
    a = rng.standard_normal(shape, dtype=np.float32)
    a[3, 100:110] = 7.5      # ties: the first index wins
    a[7, 1999] = np.nan      # NaN ignored by max/argmax
    a[8, 0] = np.nan         # NaN at index 0: argmax keeps 0
    warps = shape[0] >= torch.cuda.get_device_properties(0).multi_processor_count * 64
    assert warps == (shape[0] == 9600)
    d = _dev(a)
    for kind in ("sum", "mean", "max", "min", "argmax", "argmin", "norm"):
        got = _host(T.reduce(kind, d, 1))
        want = oracle.t_reduce(kind, a, 1, False)
        what = f"{kind} {shape}"
        if kind in ("max", "min", "argmax", "argmin"):
            assert_bitexact(got, want, what)
        else:
            oracle.PRECISE_SUMS[0] = True
            exact = oracle.t_reduce(kind, a, 1, False)
            oracle.PRECISE_SUMS[0] = False
            budget = np.abs(want.astype(np.float64) - exact)
            terms = np.abs(a.astype(np.float64))
            scale = {"sum": terms.sum(1), "mean": terms.mean(1),
                     "norm": np.sqrt((terms * terms).sum(1))}[kind]
            assert_close(got, want, rtol=RTOL, atol=ATOL * np.maximum(scale, 1.0) + budget,
                         what=what, strict_atol=ATOL * np.maximum(scale, 1.0))


def test_reduce_column_mode_is_the_reference_order(oracle):
    """A non-contiguous strip per output is folded left to right: sums over
    dim 0 match the reference bit for bit."""
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(6)
    a = rng.standard_normal((400, 3000), dtype=np.float32)
    for kind in ("sum", "mean", "norm"):
        assert_bitexact(_host(T.reduce(kind, _dev(a), 0, False)), oracle.t_reduce(kind, a, 0, False), kind)


def test_reduce_long_columns_split(oracle):
    """Long strips over few outputs are folded in ordered segments."""
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(7)
    a = rng.standard_normal((40000, 64), dtype=np.float32)
    for kind in ("sum", "max", "argmin", "norm"):
        got = _host(T.reduce(kind, _dev(a), 0, True))
        want = oracle.t_reduce(kind, a, 0, True)
        if kind in ("max", "argmin"):
            assert_bitexact(got, want, kind)
        else:
            oracle.PRECISE_SUMS[0] = True
            exact = oracle.t_reduce(kind, a, 0, True)
            oracle.PRECISE_SUMS[0] = False
            budget = np.abs(want.astype(np.float64) - exact)
            assert_close(got, want, rtol=RTOL_BIG, atol=ATOL + budget, what=kind)


def test_reduce_nan_and_tie_rules(oracle):
    from oxitorch_b200 import tensor_ops as T
    a = np.array([[np.nan, 1.0, 5.0, 5.0],
                  [2.0, np.nan, 7.0, 7.0],
                  [np.nan, np.nan, np.nan, np.nan],
                  [-np.inf, -np.inf, -np.inf, -np.inf],
                  [0.0, -0.0, 0.0, -1.0]], np.float32)
    for kind in ("max", "min", "argmax", "argmin"):
        for d in (0, 1):
            got = _host(T.reduce(kind, _dev(a), d))
            want = oracle.t_reduce(kind, a, d, False)
            assert_bitexact(got + 0.0, want + 0.0, f"{kind} dim {d}")


def test_reduce_known_answers_and_errors():
    from oxitorch_b200 import tensor_ops as T
    kats = json.load(open(os.path.join(HERE, "golden", "reference_kats.json")))
    for c in kats["reduce"]:
        a = _dev(np.asarray(c["data"], np.float32).reshape(c["shape"]))
        if "error" in c:
            with pytest.raises(ValueError):
                T.reduce(c["kind"], a, c["dim"], c["keepdim"])
            continue
        got = T.reduce(c["kind"], a, c["dim"], c["keepdim"])
        assert list(got.shape) == c["out_shape"], c["src"]
        np.testing.assert_allclose(_host(got).reshape(-1), c["want"], rtol=0,
                                   atol=c.get("atol", 0), err_msg=c["src"])
    for c in kats["reduce_all"]:
        a = _dev(np.asarray(c["data"], np.float32).reshape(c["shape"]))
        assert float(_host(T.mean_all(a))) == c["want"]["mean"]
        assert float(_host(T.sum_all(a))) == c["want"]["sum"]


def test_reduce_all_whole_tensor(oracle):
    """Whole-tensor reductions vs f64 (rtol 1e-4 from 32k elements) and exact
    max/argmax, on a dense and a transposed 1M-element tensor."""
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(12)
    a = rng.standard_normal((1024, 1024), dtype=np.float32)
    for t, h in [(_dev(a), a), (_dev(np.ascontiguousarray(a.T)).t(), a)]:
        s, s64 = T.reduce_all("sum", t, f64=True)
        assert abs(float(_host(s64)) - oracle.sum_all_f64(h)) <= 1e-9 * np.abs(h).sum()
        assert_close(_host(s), np.float32(oracle.sum_all_f64(h)), rtol=RTOL_BIG, atol=1e-3, what="sum")
        n, n64 = T.reduce_all("norm", t, f64=True)
        assert abs(float(_host(n64)) - np.sqrt(oracle.sumsq_all_f64(h))) < 1e-9 * 1024
        assert float(_host(T.reduce_all("max", t))) == h.max()
        assert float(_host(T.reduce_all("argmax", t))) == float(np.argmax(h))
        assert float(_host(T.reduce_all("argmin", t))) == float(np.argmin(h))


def test_clip_grad_norm(oracle):
    """optim.py:242-263: total = (sum over grads of sum |g|^2)^(1/2); grads
    scaled by max_norm / (total + 1e-6) when that is < 1."""
    import torch
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(13)
    gs = [rng.standard_normal(s, dtype=np.float32) for s in [(300, 70), (5000,), (64, 64, 3)]]
    want_total = float(sum(float(np.sum(np.abs(g) ** 2.0)) for g in gs)) ** 0.5
    dev = [_dev(g) for g in gs]
    total = T.clip_grad_norm_(dev, 1.0)
    assert abs(total - want_total) <= 1e-5 * want_total
    scale = 1.0 / (want_total + 1e-6)
    for g, d in zip(gs, dev):
        assert_close(_host(d), g * np.float32(scale), rtol=1e-5, atol=1e-7, what="clipped grad")


@pytest.mark.parametrize("norm_type", [1.0, 3.0, float("inf")])
def test_clip_grad_norm_other_norms(oracle, norm_type):
    """optim.py:242-263 for p = 1, 3 and inf: the inf total is exact; finite p
    within the f32 pairwise-sum and powf budget of the reference's numpy."""
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(int(norm_type) if norm_type != float("inf") else 99)
    gs = [rng.standard_normal(s, dtype=np.float32) for s in [(300, 70), (5001,), (64, 64, 3)]]
    want_total, want = oracle.clip_grad_norm_np(gs, 1.0, norm_type)
    dev = [_dev(g) for g in gs]
    total = T.clip_grad_norm_(dev, 1.0, norm_type)
    if norm_type == float("inf"):
        assert total == want_total
    else:
        assert abs(total - want_total) <= 1e-5 * want_total
    for w, d in zip(want, dev):
        assert_close(_host(d), w, rtol=1e-5, atol=1e-7, what="clipped grad")
    # reference cases (python/tests/test_phase4_training.py:211-223)
    g = _dev(np.array([[3.0, -4.0]], np.float32))
    assert T.clip_grad_norm_([g], 1.0, float("inf")) == 4.0
    assert np.allclose(_host(g), [[0.75, -1.0]], rtol=1e-5)
    nan_first = [_dev(np.array([np.nan, 1.0], np.float32)), _dev(np.array([5.0], np.float32))]
    assert np.isnan(T.clip_grad_norm_(nan_first, 1.0, float("inf")))


def test_clip_grad_value_matches_np_clip(oracle):
    """optim.py:266-272: np.clip, NaN kept, -0.0 kept, both vector and scalar
    paths (a gradient 4 bytes off alignment and an odd length)."""
    import torch
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(21)
    g = (rng.standard_normal(100003) * 3).astype(np.float32)
    g[:6] = [np.nan, np.inf, -np.inf, -0.0, 0.0, 2.0]
    buf = torch.zeros(g.size + 1, dtype=torch.float32, device="cuda")
    mis = buf[1:]
    mis.copy_(torch.from_numpy(g))
    dense = _dev(g)
    T.clip_grad_value_([dense, None, mis], 2.0)
    (want,) = oracle.clip_grad_value_np([g], 2.0)
    for d in (dense, mis):
        assert np.array_equal(_host(d).view(np.uint32), want.view(np.uint32))
    with pytest.raises(ValueError, match="clip_value must be positive"):
        T.clip_grad_value_([dense], 0.0)
