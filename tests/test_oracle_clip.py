"""The oracle's gradient clipping against the reference's own clipping tests
(python/tests/test_phase4_training.py:188-235): the 2-norm, no-op under the
threshold, several parameters, the inf-norm, p = 1, clip_grad_value_ and its
error, and skipped gradients."""

import numpy as np
import pytest

from oracle import oxiref as O


def _a(x):
    return np.array(x, np.float32)


def test_clip_grad_norm_reference_cases():
    total, (g,) = O.clip_grad_norm_np([_a([[3.0, 4.0]])], 1.0)
    assert total == pytest.approx(5.0)
    np.testing.assert_allclose(g, [[0.6, 0.8]], rtol=1e-5)
    total, (g,) = O.clip_grad_norm_np([_a([[3.0, 4.0]])], 10.0)
    assert total == pytest.approx(5.0) and np.array_equal(g, [[3.0, 4.0]])
    total, (a, b) = O.clip_grad_norm_np([_a([[3.0, 0, 0]]), _a([[0, 4.0, 0, 0]])], 0.5)
    assert total == pytest.approx(5.0)
    np.testing.assert_allclose(a, [[0.3, 0, 0]], rtol=1e-5)
    np.testing.assert_allclose(b, [[0, 0.4, 0, 0]], rtol=1e-5)
    total, (g,) = O.clip_grad_norm_np([_a([[3.0, -4.0]])], 1.0, float("inf"))
    assert total == pytest.approx(4.0)
    np.testing.assert_allclose(g, [[0.75, -1.0]], rtol=1e-5)
    total, (g,) = O.clip_grad_norm_np([_a([[3.0, 4.0]])], 1.0, 1.0)
    assert total == pytest.approx(7.0)
    np.testing.assert_allclose(g, [[3 / 7, 4 / 7]], rtol=1e-5)
    total, _ = O.clip_grad_norm_np([_a([[3.0, 4.0]]), None], 1.0)
    assert total == pytest.approx(5.0)


def test_clip_grad_value_reference_case():
    (g,) = O.clip_grad_value_np([_a([[5.0, -5.0, 1.0]])], 2.0)
    assert np.array_equal(g, [[2.0, -2.0, 1.0]])
    with pytest.raises(ValueError, match="clip_value must be positive"):
        O.clip_grad_value_np([g], 0.0)
