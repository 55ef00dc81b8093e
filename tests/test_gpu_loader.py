"""The data path on the device against the oracle: oxc_gather_rows (every
row width path: 16-byte, 4-byte and byte-wise lanes, rows packed several to a
warp), oxc_image_epoch through oxitorch_b200.data.DataLoader (epochs of the
reference's native loader with shuffling, drop_last, crop / flip / normalize
pipelines, several epochs of one loader), the reference's errors, and the
staged host<->device copies.  Copies, gathers and the per-operation f32
normalize are bit-exact."""

import numpy as np
import pytest

from oracle import oxiref as O

pytestmark = pytest.mark.gpu


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _gather(cols_dev, outs, idx_dev, nidx, nrows, err):
    from oxitorch_b200 import _native as N
    L = N.load()
    desc = (N.GatherColumn * len(cols_dev))(*[
        N.GatherColumn(c.data_ptr(), o.data_ptr(), c[0].numel() * c.element_size() if c.dim() > 1
                       else c.element_size()) for c, o in zip(cols_dev, outs)])
    return L.oxc_gather_rows(desc, len(cols_dev), idx_dev.data_ptr(), nidx, nrows,
                             None if err is None else err.data_ptr(), _stream())


@pytest.mark.parametrize("nrows,nidx", [(1000, 4096), (7, 3), (60000, 257)])
def test_gather_rows_every_width(nrows, nidx):
    import torch
    from oxitorch_b200 import _native as N
    rng = np.random.default_rng(nrows + nidx)
    cols = [rng.standard_normal((nrows, 1, 28, 28)).astype(np.float32),   # 3136 B: 16-byte lanes
            rng.standard_normal(nrows).astype(np.float32),                # 4 B: 32 rows a warp
            rng.standard_normal((nrows, 3)).astype(np.float32),           # 12 B: 4-byte lanes
            rng.integers(0, 255, (nrows, 5), dtype=np.uint8),             # 5 B: byte lanes
            rng.standard_normal((nrows, 40)).astype(np.float32)]          # 160 B: 16-byte, 10 lanes
    idx = rng.integers(0, nrows, nidx).astype(np.int64)
    cd = [_dev(c) for c in cols]
    outs = [torch.empty((nidx,) + c.shape[1:], dtype=t.dtype, device="cuda") for c, t in zip(cols, cd)]
    N.check(_gather(cd, outs, _dev(idx), nidx, nrows, None))
    for c, o in zip(cols, outs):
        assert np.array_equal(o.cpu().numpy(), c[idx])


def test_gather_rows_misaligned_and_bad_ids():
    import torch
    from oxitorch_b200 import _native as N
    L = N.load()
    rng = np.random.default_rng(3)
    base = rng.standard_normal((50, 9)).astype(np.float32)
    buf = _dev(np.concatenate([np.zeros(1, np.float32), base.reshape(-1)]))
    src = buf[1:].view(50, 9)                     # 4 bytes off 16-byte alignment
    out = torch.empty((6, 9), device="cuda")
    idx = np.array([3, 0, 49, 7, 7, 12], np.int64)
    N.check(_gather([src], [out], _dev(idx), 6, 50, None))
    assert np.array_equal(out.cpu().numpy(), base[idx])
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    bad = np.array([1, 50, 2], np.int64)
    N.check(_gather([src], [out], _dev(bad), 3, 50, err))
    assert L.oxc_check_error_flag(err.data_ptr(), _stream(), 10000) == 4
    assert "index 50 out of range for dim 0 of size 50" in N.last_error()
    assert np.array_equal(out[[0, 2]].cpu().numpy(), base[[1, 2]])


def _epoch_equal(got, want):
    assert len(got) == len(want)
    for gb, wb in zip(got, want):
        assert len(gb) == len(wb)
        for g, w in zip(gb, wb):
            g = g.cpu().numpy()
            assert g.shape == w.shape
            assert np.array_equal(g.view(np.uint32), np.ascontiguousarray(w).view(np.uint32))


CASES = [
    # (shape, batch, shuffle, drop_last, seed, transforms)
    ((1000, 1, 28, 28), 64, True, False, 3,
     [("crop", 24), ("flip",), ("normalize", [0.1307], [0.3081])]),
    ((1000, 1, 28, 28), 64, True, True, 3, None),
    ((300, 3, 32, 32), 50, True, True, 11,
     [("flip",), ("crop", 28), ("normalize", [0.4914, 0.4822, 0.4465], [0.247, 0.243, 0.261])]),
    ((97, 3, 8, 8), 10, False, False, None, [("crop", 5), ("crop", 3), ("flip",)]),
    ((45, 8, 8), 9, True, False, 2, [("crop", 5), ("flip",)]),
    ((5, 4, 4), 8, True, True, 1, [("flip",)]),   # one short batch, kept despite drop_last
    ((40, 2, 6, 6), 7, True, False, 5,             # three normalize steps: the 4-slot kernel
     [("normalize", [0.5, -0.5], [2.0, 0.5]), ("crop", 4), ("normalize", [0.1, 0.2], [0.3, 0.7]),
      ("flip",), ("normalize", [1.5, 0.0], [1.1, 0.9])]),
]


@pytest.mark.parametrize("shape,bs,shuffle,drop_last,seed,steps", CASES)
def test_loader_epochs_match_oracle(shape, bs, shuffle, drop_last, seed, steps):
    from oxitorch_b200 import data
    rng = np.random.default_rng(shape[0] + bs)
    images = rng.standard_normal(shape).astype(np.float32)
    labels = rng.integers(0, 10, shape[0]).astype(np.float32)
    wire = None
    if steps:
        wire = data.NativeTransform([
            ("crop", [s[1]]) if s[0] == "crop" else ("flip", []) if s[0] == "flip"
            else ("normalize", list(s[1]) + list(s[2])) for s in steps])
    loader = data.DataLoader([images, labels], batch_size=bs, shuffle=shuffle, drop_last=drop_last,
                             seed=seed, transforms=wire, transform_seed=21)
    for epoch in range(2):
        got = list(loader)
        want = O.loader_epoch([images, labels], bs, shuffle, drop_last, seed, steps, 21, epoch)
        _epoch_equal(got, want)


def test_loader_raises_at_the_failing_batch():
    """Rank-3 columns: a batch is one sample whose channels are its rows, so a
    4-channel normalize fails on the short last batch, after the others."""
    from oxitorch_b200 import data
    images = np.random.default_rng(0).standard_normal((10, 3, 3)).astype(np.float32)
    tf = data.NativeTransform([("normalize", [0.0] * 4 + [1.0] * 4)])
    it = iter(data.DataLoader([images], batch_size=4, transforms=tf))
    # the first two batches: the same rows and seeds as a loader over rows 0..7
    want = O.loader_epoch([images[:8]], 4, False, False, None, [("normalize", [0.0] * 4, [1.0] * 4)],
                          0)
    for k in range(2):
        _epoch_equal([next(it)], [want[k]])
    with pytest.raises(RuntimeError, match="DataLoader failed at batch 2: invalid argument: normalize "
                                           "expects 2 channels, got mean 4 / std 4"):
        next(it)
    with pytest.raises(RuntimeError, match="DataLoader worker failed: invalid argument: crop size 9"):
        list(data.DataLoader([images], batch_size=4, num_workers=2,
                             transforms=data.NativeTransform([("crop", [9])])))


def test_loader_constructor_errors():
    from oxitorch_b200 import data
    x = np.zeros((4, 2), np.float32)
    with pytest.raises(ValueError, match="DataLoader needs at least one tensor column"):
        data.DataLoader([])
    with pytest.raises(ValueError, match="DataLoader dataset is empty"):
        data.DataLoader([np.zeros((0, 2), np.float32)])
    with pytest.raises(ValueError, match="batch_size must be >= 1"):
        data.DataLoader([x], batch_size=0)
    with pytest.raises(ValueError, match="column 1 has 3 rows, expected 4"):
        data.DataLoader([x, np.zeros(3, np.float32)])
    with pytest.raises(ValueError, match="transforms pipeline is empty; pass None instead"):
        data.DataLoader([x], transforms=data.NativeTransform([]))
    with pytest.raises(TypeError, match="expected a numpy array or f32 buffer object"):
        data.DataLoader([np.zeros((4, 2), np.float64)])
    loader = data.DataLoader([x], batch_size=3)
    assert loader.n == 4 and loader.batch_size == 3


@pytest.mark.parametrize("nbytes,offset", [(4, 0), (4096, 4), (8 << 20, 0), ((8 << 20) + 12, 4),
                                           (50_000_012, 8)])
def test_upload_download_round_trip(nbytes, offset):
    import torch
    from oxitorch_b200 import _native as N
    from oxitorch_b200 import data
    L = N.load()
    n = nbytes // 4
    host = np.random.default_rng(nbytes).standard_normal(n + offset).astype(np.float32)[offset:]
    dev = data.from_numpy(host)
    assert np.array_equal(dev.cpu().numpy(), host)
    back = data.to_numpy(dev)
    assert np.array_equal(back, host)
    raw = torch.empty(n, dtype=torch.float32, device="cuda")
    N.check(L.oxc_upload(raw.data_ptr(), host.ctypes.data, nbytes, _stream()))
    out = np.empty(n + 3, np.float32)[3:]
    N.check(L.oxc_download(out.ctypes.data, raw.data_ptr(), nbytes, _stream()))
    assert np.array_equal(out, host)
    assert L.oxc_upload(raw.data_ptr(), host.ctypes.data, 0, _stream()) == 0
    assert L.oxc_upload(None, host.ctypes.data, 4, _stream()) == 1
