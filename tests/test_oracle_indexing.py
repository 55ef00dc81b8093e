"""The oracle's scatter_dim0 and masked_select (forward and VJP) pinned on the
reference's own known answers:

* crates/oxi-tensor/src/tests.rs:378-406 (forward values and errors);
* crates/oxi-autograd/src/tests.rs:240-331 (last-write-wins grads, broadcast
  accumulation);
* python/tests/test_indexing_grad.py:20-70 (the Python surface's cases).
"""
import numpy as np
import pytest


def test_scatter_dim0_forward_kats(oracle):
    base = np.array([[1, 2], [3, 4]], np.float32)
    out = oracle.t_scatter_dim0(base, [1], np.array([[9, 8]], np.float32))
    np.testing.assert_array_equal(out, [[1, 2], [9, 8]])
    np.testing.assert_array_equal(oracle.t_index_select(out, 0, [1]), [[9, 8]])
    with pytest.raises(oracle.OutOfBounds, match="index 5 out of range for dim 0 of size 2"):
        oracle.t_scatter_dim0(base, [5], np.array([[9, 8]], np.float32))
    with pytest.raises(oracle.ShapeMismatch):
        oracle.t_scatter_dim0(base, [0], np.zeros((2, 2), np.float32))
    with pytest.raises(oracle.InvalidArgument):
        oracle.t_scatter_dim0(np.float32(1.0), [0], np.zeros((1,), np.float32))


def test_scatter_dim0_last_write_wins_kats(oracle):
    b = np.array([[10, 11], [20, 21], [30, 31]], np.float32)
    v = np.array([[1, 2], [3, 4], [5, 6]], np.float32)
    out = oracle.t_scatter_dim0(b, [2, 0, 2], v)
    np.testing.assert_array_equal(out, [[3, 4], [20, 21], [5, 6]])
    gb, gv = oracle.scatter_dim0_vjp(np.ones((3, 2), np.float32), 3, [2, 0, 2])
    np.testing.assert_array_equal(gb, [[0, 0], [1, 1], [0, 0]])
    np.testing.assert_array_equal(gv, [[0, 0], [1, 1], [1, 1]])
    # negative ids wrap like the forward (rows + i)
    gb, gv = oracle.scatter_dim0_vjp(np.ones((3, 2), np.float32), 3, [-1, 0, 2])
    np.testing.assert_array_equal(gb, [[0, 0], [1, 1], [0, 0]])
    np.testing.assert_array_equal(gv, [[0, 0], [1, 1], [1, 1]])


def test_scatter_dim0_matches_numpy_assignment(oracle):
    rng = np.random.default_rng(7)
    a = rng.standard_normal((5, 3)).astype(np.float32)
    vals = rng.standard_normal((3, 3)).astype(np.float32)
    want = a.copy()
    want[[4, 1, 4]] = vals
    np.testing.assert_array_equal(oracle.t_scatter_dim0(a, [4, 1, 4], vals), want)


def test_masked_select_forward_kats(oracle):
    base = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    mask = np.array([[1, 0, 1], [0, 1, 0]], np.float32)
    np.testing.assert_array_equal(oracle.t_masked_select(base, mask), [1, 3, 5])
    np.testing.assert_array_equal(oracle.t_masked_select(base, np.array([1, 0, 0], np.float32)),
                                  [1, 4])
    a = np.random.default_rng(3).standard_normal((4, 5)).astype(np.float32)
    np.testing.assert_array_equal(oracle.t_masked_select(a, (a > 0).astype(np.float32)), a[a > 0])


def test_masked_select_drops_picked_nan(oracle):
    """The NaN sentinel of lib.rs:952 also drops a picked NaN of x; a NaN mask
    entry is nonzero and picks."""
    x = np.array([1.0, np.nan, 3.0], np.float32)
    np.testing.assert_array_equal(oracle.t_masked_select(x, np.ones(3, np.float32)), [1, 3])
    np.testing.assert_array_equal(
        oracle.t_masked_select(np.array([1, 2], np.float32), np.array([np.nan, 0], np.float32)), [1])


def test_masked_select_vjp_kats(oracle):
    # broadcast row mask [1, 0, 1]: picks (0,0), (0,2), (1,0), (1,2)
    gx = oracle.masked_select_vjp(np.array([10, 20, 30, 40], np.float32), (2, 3),
                                  np.array([1, 0, 1], np.float32))
    np.testing.assert_array_equal(gx, [[10, 0, 20], [30, 0, 40]])
    # a column broadcast against a [2, 3] mask picks each element twice
    col = np.array([[7.0], [9.0]], np.float32)
    mc = np.array([[1, 1, 0], [0, 1, 1]], np.float32)
    np.testing.assert_array_equal(oracle.t_masked_select(col, mc), [7, 7, 9, 9])
    gx = oracle.masked_select_vjp(np.array([1, 2, 3, 4], np.float32), (2, 1), mc)
    np.testing.assert_array_equal(gx, [[3], [7]])


def test_masked_select_vjp_matches_dense_multiply(oracle):
    rng = np.random.default_rng(11)
    up = rng.standard_normal((2, 3)).astype(np.float32)
    mask = (rng.standard_normal((2, 3)) > 0).astype(np.float32)
    gx = oracle.masked_select_vjp(up[mask > 0], (2, 3), mask)
    np.testing.assert_array_equal(gx, mask * up)


def test_masked_select_vjp_rejects_short_grad(oracle):
    with pytest.raises(oracle.OutOfBounds):
        oracle.masked_select_vjp(np.array([1.0], np.float32), (2,), np.ones(2, np.float32))


# ---- the library's host-side scatter planning against the oracle ---------------------------------

def _apply(a, idx_map, b, inner_shape):
    """oxc_select_rows restated: out[i] = a[map[i]] if map[i] >= 0 else (b[i] or 0)."""
    out = np.zeros((len(idx_map),) + inner_shape, np.float32)
    for i, r in enumerate(idx_map):
        if r >= 0:
            out[i] = a[r]
        elif b is not None:
            out[i] = b[i]
    return out


@pytest.mark.parametrize("rows,indices", [
    (3, [2, 0, 2]), (3, [-1, 0, 2]), (5, [4, 1, 4]), (4, []), (6, [5, 5, 5, -6, 0, 3, -3]),
    (1, [0, 0]), (7, list(range(7))), (7, list(range(-1, -8, -1)))])
def test_library_scatter_maps_reproduce_oracle(oracle, rows, indices):
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(rows * 31 + len(indices))
    base = rng.standard_normal((rows, 2, 3)).astype(np.float32)
    values = rng.standard_normal((len(indices), 2, 3)).astype(np.float32)
    g = rng.standard_normal((rows, 2, 3)).astype(np.float32)
    fwd, keep, win = T.scatter_dim0_maps(rows, indices)
    np.testing.assert_array_equal(_apply(values, fwd, base, (2, 3)),
                                  oracle.t_scatter_dim0(base, indices, values))
    gb, gv = oracle.scatter_dim0_vjp(g, rows, indices)
    np.testing.assert_array_equal(_apply(g, keep, None, (2, 3)), gb)
    np.testing.assert_array_equal(_apply(g, win, None, (2, 3)), gv)


def test_library_scatter_maps_reject_out_of_range():
    from oxitorch_b200 import tensor_ops as T
    with pytest.raises(RuntimeError, match="index 5 out of range for dim 0 of size 2"):
        T.scatter_dim0_maps(2, [5])
    with pytest.raises(RuntimeError, match="index -3 out of range for dim 0 of size 2"):
        T.scatter_dim0_maps(2, [0, -3])


def test_narrow_dim0_vjp_pads_with_zero_rows(oracle):
    g = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    np.testing.assert_array_equal(oracle.narrow_dim0_vjp(g, (4, 3), 1, 2),
                                  [[0, 0, 0], [1, 2, 3], [4, 5, 6], [0, 0, 0]])
    np.testing.assert_array_equal(oracle.narrow_dim0_vjp(g[:1].reshape(1, 3, 1), (3, 3, 1), 2, 1),
                                  np.array([0, 0, 0, 0, 0, 0, 1, 2, 3], np.float32).reshape(3, 3, 1))


@pytest.mark.parametrize("rows,offset,length", [(4, 1, 2), (5, 0, 5), (5, 4, 1), (6, 2, 0),
                                                (3, 1, 5), (7, 0, 1)])
def test_library_narrow_map_reproduces_oracle(oracle, rows, offset, length):
    from oxitorch_b200 import tensor_ops as T
    m, lo, hi = T.narrow_dim0_map(rows, offset, length)
    kept = hi - lo
    assert kept == len(range(rows)[offset:offset + length])
    g = np.random.default_rng(rows + offset).standard_normal((kept, 2, 2)).astype(np.float32)
    np.testing.assert_array_equal(_apply(g, m, None, (2, 2)),
                                  oracle.narrow_dim0_vjp(g, (rows, 2, 2), offset, kept))
