"""Comparison helpers for the parity tests.

Tolerances (from the project's parity contract):
* integer, index and copy results: bit-exact;
* fp32 results: |got - want| <= atol + rtol * |want| with rtol 1e-5, atol 1e-6;
* reductions over >= 32k elements and duplicate-id gradient accumulation:
  rtol 1e-4;
* outputs that are sums (column sums such as dweight/dbias, row sums): the
  reference folds left to right in f32 while the kernels use fixed-order
  trees, so the absolute term is scaled by the sum's condition number:
  atol = 1e-6 * sum(|terms|) (each test states the terms); 1e-5 * sum(|terms|)
  when the terms themselves depend on a row reduction over >= 32k elements;
* outputs computed from a centred value (x - mean, LayerNorm) also allow 4 ulp
  of |mean| propagated through the normalisation: the kernel's own rounding of
  a large row mean, which the reference-only budget below does not contain;
* every output also carries the reference's own summation-order error:
  the element-wise difference between the reference composition with its
  left-to-right f32 folds and the same composition with f64-folded sums
  (reference_budget); the kernels' fixed-order trees sit between the two;
* outputs that pass through a transcendental (tanh, exp, log): the reference
  calls the host libm (glibc: tanhf is off by 1-2 ulp from correct rounding on
  ~5% of inputs) and the kernels call CUDA's (tanhf <= 2 ulp; the row sums of
  exp in softmax / cross-entropy use the ex2.approx instruction), so each element
  may also differ by the propagated effect of a LIBM_ULPS-ulp change of that
  function, measured by re-running the oracle with the function's results
  shifted (libm_budget).
"""

import contextlib
import os

import numpy as np

LIBM_ULPS = 4

# One record per assert_close call: how many elements exceed the BARE
# tolerance (rtol as passed; atol 1e-6, or the Sigma|terms| * 1e-6 of a sum
# output, `strict_atol`), i.e. pass only because of the reference-defined
# budgets above.  tests/conftest.py writes them to $OXC_STRICT_REPORT.
STRICT_LOG = []


@contextlib.contextmanager
def perturbed(oracle, name, k):
    old = dict(oracle.PERTURB_ULPS)
    oracle.PERTURB_ULPS[name] = k
    try:
        yield
    finally:
        oracle.PERTURB_ULPS.clear()
        oracle.PERTURB_ULPS.update(old)


@contextlib.contextmanager
def precise_sums(oracle):
    oracle.PRECISE_SUMS[0] = True
    try:
        yield
    finally:
        oracle.PRECISE_SUMS[0] = False


def _absdiff(a, b):
    """|a - b| in f64; equal values (infinities included) give 0."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    with np.errstate(invalid="ignore"):
        return np.where(a == b, 0.0, np.abs(a - b))


def reference_budget_parts(oracle, run, libm=("tanh",), ulps=LIBM_ULPS):
    """(outputs, summation-order budgets, libm budgets) of the oracle run
    `run`; see reference_budget."""
    base = run()
    with precise_sums(oracle):
        exact = run()
    sums = [_absdiff(e, b) for b, e in zip(base, exact)]
    if libm:
        _, lb = libm_budget(oracle, run, libm, ulps)
    else:
        lb = [np.zeros(np.shape(b), np.float64) for b in base]
    return base, sums, lb


def reference_budget(oracle, run, libm=("tanh",), ulps=LIBM_ULPS):
    """(outputs, budgets) of the oracle run `run` (a callable returning a tuple
    of arrays).  The budget of each element is what the reference's result is
    only defined up to:
      |run() - run() with f64-folded sums|   (its own left-to-right f32 sums)
    + max over +-ulps of |run() - run() with `libm` results shifted| (libm ulps).
    """
    base, sums, lb = reference_budget_parts(oracle, run, libm, ulps)
    return base, [a + b for a, b in zip(sums, lb)]


def max_vjp_budget(oracle, run):
    """Per-element |run() - run() without the max node's VJP| (nonzero only on
    argmax columns): what the kernels' omission of that exact-zero term can
    change."""
    base = run()
    oracle.SKIP_MAX_VJP[0] = True
    try:
        alt = run()
    finally:
        oracle.SKIP_MAX_VJP[0] = False
    return [_absdiff(a, b) for a, b in zip(alt, base)]


def libm_budget(oracle, run, names=("tanh",), ulps=LIBM_ULPS):
    """Per-output elementwise |run() - run() with `names` shifted by +-ulps|,
    maximised over both directions.  `run` returns a tuple of arrays."""
    base = run()
    budget = [np.zeros(np.shape(b), np.float64) for b in base]
    for name in names:
        for k in (ulps, -ulps):
            with perturbed(oracle, name, k):
                alt = run()
            for i, (b, a) in enumerate(zip(base, alt)):
                budget[i] = np.maximum(budget[i], _absdiff(a, b))
    return base, budget

RTOL = 1e-5
ATOL = 1e-6
RTOL_BIG = 1e-4


def _current_test():
    return os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0]


def strict_breakdown(got, want, rtol, strict_atol, parts, what=""):
    """Attributes the elements that exceed the bare tolerance
    (strict_atol + rtol |want|) to the budgets that admit them, in order:
    `parts` is [(name, per-element budget), ...].  Appends the counts to
    STRICT_LOG and returns them."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    with np.errstate(invalid="ignore"):
        err = np.where(got == want, 0.0, np.abs(got - want))
        lim = np.broadcast_to(np.asarray(strict_atol, np.float64), want.shape) + rtol * np.abs(want)
        over = ~np.isnan(want) & ~(err <= lim)
        counts = {"bare": int(over.sum())}
        rest = over
        for name, b in parts:
            lim = lim + np.broadcast_to(np.asarray(b, np.float64), want.shape)
            admitted = rest & (err <= lim)
            counts[name] = int(admitted.sum())
            rest = rest & ~admitted
        counts["unadmitted"] = int(rest.sum())
    rec = {"test": _current_test(), "what": what, "n": int(want.size), "rtol": rtol,
           "breakdown": counts}
    STRICT_LOG.append(rec)
    return counts


def assert_close(got, want, rtol=RTOL, atol=ATOL, what="", strict_atol=None):
    """|got - want| <= atol + rtol |want| element-wise.  `strict_atol` is the
    bare absolute tolerance of this output (1e-6, or 1e-6 x Sigma|terms| for a
    sum); the number of elements beyond it is recorded in STRICT_LOG."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    atol = np.broadcast_to(np.asarray(atol, dtype=np.float64), want.shape)
    nan_ok = np.isnan(got) == np.isnan(want)
    assert nan_ok.all(), f"{what}: NaN pattern differs"
    fin = ~np.isnan(want)
    with np.errstate(invalid="ignore"):
        err = np.abs(got - want)
        lim = atol + rtol * np.abs(want)
        # exact equality always passes (infinities included)
        bad = fin & ~(err <= lim) & (got != want)
        slim = (np.broadcast_to(np.asarray(ATOL if strict_atol is None else strict_atol,
                                           np.float64), want.shape) + rtol * np.abs(want))
        over = fin & ~(err <= slim) & (got != want)
        worst = float(np.max(np.where(over, err / slim, 0.0), initial=0.0))
    STRICT_LOG.append({"test": _current_test(), "what": what, "n": int(want.size), "rtol": rtol,
                       "over_bare": int(over.sum()), "worst_err_over_bare": worst})
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, np.nan_to_num(err - lim, nan=np.inf), -np.inf)),
                             want.shape)
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{want.size} elements out of tolerance "
            f"(rtol={rtol}); worst at {i}: got {got[i]!r} want {want[i]!r} "
            f"err {err[i]:.3e} limit {lim[i]:.3e}")


def assert_bitexact(got, want, what=""):
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    if got.dtype.kind == "f":
        same = (got.view(np.uint32 if got.dtype == np.float32 else np.uint64)
                == want.astype(got.dtype).view(np.uint32 if got.dtype == np.float32 else np.uint64))
        same |= np.isnan(got) & np.isnan(want)
    else:
        same = got == want
    if not same.all():
        i = np.unravel_index(np.argmin(same), same.shape)
        raise AssertionError(f"{what}: {int((~same).sum())}/{same.size} elements differ; "
                             f"first at {i}: got {got[i]!r} want {want[i]!r}")
