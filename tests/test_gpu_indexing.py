"""Dim-0 scatter (Tensor.scatter / Tensor::scatter_dim0) and its VJP on the
device, bit-exact against the oracle: the forward and both gradients are row
copies, so every element must match exactly."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev(a, grad=False):
    import torch
    return torch.from_numpy(np.array(a, order="C", copy=True)).cuda().requires_grad_(grad)


def _host(t):
    return t.detach().cpu().numpy()


CASES = [
    ((3, 2), [2, 0, 2]),                     # the reference's last-write-wins case
    ((5, 3), [4, 1, 4]),
    ((4, 7), [-1, 0, -1, 2]),                # odd rows: scalar path, negative ids
    ((6,), [5, 5, -6, 0]),                   # 1-D base: one float per row
    ((1000, 4096), None),                    # float4 path, many repeats
    ((257, 3, 5), None),                     # 15-float rows
    ((4, 8), []),                            # nothing written
]


@pytest.mark.parametrize("shape,indices", CASES)
def test_scatter_dim0_forward_and_vjp_bitexact(oracle, shape, indices):
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(shape[0] * 7 + len(shape))
    if indices is None:
        indices = [int(i) for i in rng.integers(-shape[0], shape[0], 3 * shape[0] // 2)]
    base = rng.standard_normal(shape).astype(np.float32)
    values = rng.standard_normal((len(indices),) + shape[1:]).astype(np.float32)
    g = rng.standard_normal(shape).astype(np.float32)
    b, v = _dev(base, True), _dev(values, True)
    out = T.scatter_dim0(b, indices, v)
    assert tuple(out.shape) == shape
    np.testing.assert_array_equal(_host(out), oracle.t_scatter_dim0(base, indices, values))
    out.backward(_dev(g))
    gb, gv = oracle.scatter_dim0_vjp(g, shape[0], indices)
    np.testing.assert_array_equal(_host(b.grad), gb)
    np.testing.assert_array_equal(_host(v.grad), gv)


def test_scatter_dim0_errors_match_reference():
    import torch
    from oxitorch_b200 import tensor_ops as T
    base = torch.zeros(2, 2, device="cuda")
    with pytest.raises(RuntimeError, match="index 5 out of range for dim 0 of size 2"):
        T.scatter_dim0(base, [5], torch.zeros(1, 2, device="cuda"))
    with pytest.raises(ValueError, match="shape mismatch"):
        T.scatter_dim0(base, [0], torch.zeros(2, 2, device="cuda"))
    with pytest.raises(ValueError, match="CUDA device"):
        T.scatter_dim0(torch.zeros(2, 2), [0], torch.zeros(1, 2))


def test_select_rows_abi_records_a_map_past_the_source():
    """Through the C ABI: a map entry past the source rows is recorded in the
    error flag (read back as OutOfBounds) and its row is skipped; the other
    rows are still written."""
    import torch
    from oxitorch_b200 import _native as N
    L = N.load()
    a = torch.arange(12, dtype=torch.float32, device="cuda").reshape(3, 4)
    out = torch.full((3, 4), -1.0, device="cuda")
    m = torch.tensor([2, 3, -1], dtype=torch.int64, device="cuda")
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert L.oxc_select_rows(a.data_ptr(), 3, m.data_ptr(), 3, None, out.data_ptr(), 4,
                             flag.data_ptr(), s) == N.OK
    st = L.oxc_check_error_flag(flag.data_ptr(), s, 60000)
    assert st == N.ERR_OUT_OF_BOUNDS
    assert "index 3 out of range for dim 0 of size 3" in N.last_error()
    got = _host(out)
    np.testing.assert_array_equal(got[0], [8, 9, 10, 11])
    np.testing.assert_array_equal(got[1], [-1, -1, -1, -1])
    np.testing.assert_array_equal(got[2], [0, 0, 0, 0])
    assert L.oxc_select_rows(a.data_ptr(), 3, None, 3, None, out.data_ptr(), 4, None, s) \
        == N.ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("shape,offset,length", [((4, 3), 1, 2), ((512, 1024), 100, 300),
                                                 ((9, 5, 3), 8, 4), ((6, 4), 2, 0),
                                                 ((5, 3), 0, 2), ((7, 2, 2), 6, 1)])
def test_narrow_dim0_view_and_zero_padding_vjp(oracle, shape, offset, length):
    """Offset 0 (x[0:k]) and the last row (x[-1], which the binding's select
    normalises to offset rows - 1 before narrow_dim0 sees it) are included.
    At offset 0 the reference's VJP fails instead: its concat_rows takes the
    row width from the first block, the empty zeros_before, and from_vec then
    rejects [rows, 0] with the data of g (crates/oxi-autograd/src/ops.rs:
    427-455).  This path returns the zero-padded gradient there, the result
    the reference computes for every other offset."""
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(shape[0] + offset)
    x = rng.standard_normal(shape).astype(np.float32)
    xd = _dev(x, True)
    y = T.narrow_dim0(xd, offset, length)
    np.testing.assert_array_equal(_host(y), x[offset:offset + length])
    g = rng.standard_normal(tuple(y.shape)).astype(np.float32)
    y.backward(_dev(g))
    np.testing.assert_array_equal(_host(xd.grad),
                                  oracle.narrow_dim0_vjp(g, shape, offset, y.shape[0]))


MASKED = [
    ((2, 3), (2, 3)),          # the reference's basic case
    ((2, 3), (3,)),            # a row mask broadcast over x
    ((2, 1), (2, 3)),          # x broadcast: picks accumulate
    ((3, 1, 5), (1, 4, 1)),    # both broadcast, x folded over one dim
    ((1, 6, 1), (5, 1, 7)),    # x folded over two dims in grid order
    ((300, 200), (300, 200)),  # several count chunks
    ((4,), ()),                # a 0-d mask
    ((0, 3), (0, 3)),          # an empty grid
]


@pytest.mark.parametrize("xs,ms", MASKED)
def test_masked_select_forward_and_vjp_bitexact(oracle, xs, ms):
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(len(xs) * 10 + len(ms))
    x = rng.standard_normal(xs).astype(np.float32)
    mask = np.asarray(rng.random(ms) > 0.4, dtype=np.float32)
    mask = np.where(np.asarray(rng.random(ms) > 0.8), mask * np.float32(-2.5), mask).astype(np.float32)
    xd = _dev(x, True)
    out = T.masked_select(xd, _dev(mask))
    want = oracle.t_masked_select(x, mask)
    np.testing.assert_array_equal(_host(out), want)
    g = rng.standard_normal(want.shape).astype(np.float32)
    out.backward(_dev(g))
    np.testing.assert_array_equal(_host(xd.grad), oracle.masked_select_vjp(g, xs, mask))


def test_masked_select_reference_cases():
    import torch
    from oxitorch_b200 import tensor_ops as T
    base = torch.tensor([[1.0, 2, 3], [4, 5, 6]], device="cuda")
    m = torch.tensor([[1.0, 0, 1], [0, 1, 0]], device="cuda")
    np.testing.assert_array_equal(_host(T.masked_select(base, m)), [1, 3, 5])
    col = torch.tensor([[7.0], [9.0]], device="cuda", requires_grad=True)
    picked = T.masked_select(col, torch.tensor([[1.0, 1, 0], [0, 1, 1]], device="cuda"))
    np.testing.assert_array_equal(_host(picked), [7, 7, 9, 9])
    picked.backward(torch.tensor([1.0, 2, 3, 4], device="cuda"))
    np.testing.assert_array_equal(_host(col.grad), [[3], [7]])
    nan_x = torch.tensor([1.0, float("nan"), 3.0], device="cuda")
    np.testing.assert_array_equal(_host(T.masked_select(nan_x, torch.ones(3, device="cuda"))), [1, 3])
    with pytest.raises(ValueError, match="shape mismatch"):
        T.masked_select(base, torch.ones(4, device="cuda"))
