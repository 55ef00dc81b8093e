"""The data loader's index and augmentation arithmetic, on the CPU.

1. The oracle against the reference's own tests: rng.rs:127-162 (the NumPy
   random and permutation streams), batch.rs:430-470 (epoch plans, gathers)
   and transform.rs:253-402 (crop windows, flip outcomes, exact normalize,
   argument errors, pipeline order); and against NumPy's RandomState, whose
   stream the reference reproduces.
2. The library's host-side planning (oxc_permutation, oxc_epoch_seed,
   oxc_batch_seed, oxc_epoch_transform_plan: no device work) against the
   oracle.  The plane maps are applied here with the device kernel's index
   arithmetic restated in numpy, and must reproduce the oracle's augmented
   batches bit for bit."""

import ctypes

import numpy as np
import pytest

from oracle import oxiref as O


# ---- 1. oracle vs the reference's tests -------------------------------------------------------

def test_mt19937_matches_reference_streams():
    r = O.Mt19937(42)
    got = [float(r.random()) for _ in range(5)]
    want = [0.37454012, 0.9507143, 0.7319939, 0.5986585, 0.15601864]
    assert all(abs(g - w) < 1e-6 for g, w in zip(got, want))
    assert O.Mt19937(7).permutation(10) == [8, 5, 0, 2, 1, 9, 7, 3, 6, 4]


@pytest.mark.parametrize("seed,n", [(0, 1), (1, 2), (3, 17), (12345, 1000), (2**32 - 1, 4097)])
def test_permutation_matches_numpy_randomstate(seed, n):
    assert O.Mt19937(seed).permutation(n) == list(np.random.RandomState(seed).permutation(n))


def test_epoch_plan_matches_reference():
    order = list(range(7))
    assert O.epoch_plan(order, 3, False) == [[0, 1, 2], [3, 4, 5], [6]]
    assert O.epoch_plan(order, 3, True) == [[0, 1, 2], [3, 4, 5]]
    assert O.epoch_plan([9, 8], 4, True) == [[9, 8]]
    with pytest.raises(ValueError, match="batch_size must be >= 1"):
        O.epoch_plan([1], 0, False)


def test_gather_keeps_dims_and_rejects_out_of_range():
    imgs = np.arange(24, dtype=np.float32).reshape(6, 1, 2, 2)
    labels = np.arange(6, dtype=np.float32)
    a, b = O.gather_columns([imgs, labels], [5, 0])
    assert a.shape == (2, 1, 2, 2)
    assert a.reshape(-1).tolist() == [20, 21, 22, 23, 0, 1, 2, 3]
    assert b.tolist() == [5.0, 0.0]
    with pytest.raises(IndexError, match=r"index out of range \(n=1\)"):
        O.gather_columns([np.ones((1, 2), np.float32)], [1])


def test_crop_windows_and_reproducibility():
    batch = np.arange(32, dtype=np.float32).reshape(2, 1, 4, 4)
    out = O.random_crop(batch, 2, O.batch_rng(O.batch_seed(123, 0)))
    assert out.shape == (2, 1, 2, 2)
    for img in range(2):
        windows = [batch[img, 0, t:t + 2, l:l + 2] for t in range(3) for l in range(3)]
        assert any(np.array_equal(out[img, 0], w) for w in windows)
    batch = np.arange(150, dtype=np.float32).reshape(3, 2, 5, 5)
    ra = O.random_crop(batch, 3, O.batch_rng(O.batch_seed(9, 4)))
    rb = O.random_crop(batch, 3, O.batch_rng(O.batch_seed(9, 4)))
    rc = O.random_crop(batch, 3, O.batch_rng(O.batch_seed(9, 5)))
    assert np.array_equal(ra, rb) and not np.array_equal(ra, rc)
    with pytest.raises(ValueError, match="crop size 5 exceeds image 4x4"):
        O.random_crop(np.zeros((1, 1, 4, 4), np.float32), 5, O.batch_rng(1))
    with pytest.raises(ValueError, match="crop size 0 exceeds"):
        O.random_crop(np.zeros((1, 1, 4, 4), np.float32), 0, O.batch_rng(1))


def test_flip_outcomes_across_seeds():
    batch = np.array([1, 2, 3, 4], np.float32).reshape(1, 1, 1, 4)
    seen = set()
    for seed in range(64):
        out = O.random_horizontal_flip(batch, O.batch_rng(seed)).reshape(-1).tolist()
        assert out in ([4, 3, 2, 1], [1, 2, 3, 4])
        seen.add(tuple(out))
    assert len(seen) == 2


def test_flip_channels_after_the_first_always_reverse():
    """The coin decides only the sample's first plane (transform.rs:148-153)."""
    batch = np.array([0, 1, 2, 3, 10, 11, 12, 13], np.float32).reshape(1, 2, 2, 2)
    for seed in range(16):
        rng = O.batch_rng(seed)
        coin = O.batch_rng(seed).random()
        out = O.random_horizontal_flip(batch, rng)
        assert np.array_equal(out[0, 1], batch[0, 1, :, ::-1])
        want0 = batch[0, 0] if coin >= np.float32(0.5) else batch[0, 0, :, ::-1]
        assert np.array_equal(out[0, 0], want0)


def test_normalize_exact_and_validated():
    batch = np.arange(12, dtype=np.float32).reshape(2, 3, 1, 2)
    out = O.normalize(batch, [1.0, 2.0, 3.0], [2.0, 4.0, 8.0])
    mean, std = [1.0, 2.0, 3.0], [2.0, 4.0, 8.0]
    want = [(np.float32(i) - np.float32(mean[(i % 6) // 2])) / np.float32(std[(i % 6) // 2])
            for i in range(12)]
    assert out.reshape(-1).tolist() == [float(w) for w in want]
    z = np.zeros((2, 3, 2, 2), np.float32)
    with pytest.raises(ValueError, match="normalize expects 3 channels, got mean 1 / std 1"):
        O.normalize(z, [0.0], [1.0])
    with pytest.raises(ValueError, match="normalize std must be > 0"):
        O.normalize(z, [0.0] * 3, [0.0] * 3)


def test_pipeline_applies_steps_in_order():
    batch = np.array([2.0, 4.0], np.float32).reshape(1, 1, 1, 2)
    out = O.apply_transforms(batch, [("normalize", [1.0], [2.0]), ("flip",)], O.batch_rng(0))
    assert out.reshape(-1).tolist() in ([0.5, 1.5], [1.5, 0.5])


def test_loader_epochs_follow_the_epoch_counter():
    cols = [np.arange(40, dtype=np.float32).reshape(10, 4), np.arange(10, dtype=np.float32)]
    e0 = O.loader_epoch(cols, 3, True, False, 5, epoch=0)
    e1 = O.loader_epoch(cols, 3, True, False, 5, epoch=1)
    order0 = [int(v) for b in e0 for v in b[1]]
    assert sorted(order0) == list(range(10))
    assert order0 == O.Mt19937(O.epoch_seed(5, 0) & 0xFFFFFFFF).permutation(10)
    assert order0 != [int(v) for b in e1 for v in b[1]]
    # shuffle without a seed keeps the natural order (data.rs:217-226)
    assert [int(v) for b in O.loader_epoch(cols, 4, True, False, None) for v in b[1]] == list(range(10))


# ---- 2. the library's host-side planning ------------------------------------------------------

def _lib():
    from oxitorch_b200 import _native as N
    return N, N.load(require_device=False)


@pytest.mark.parametrize("seed,n", [(0, 1), (7, 10), (99, 5000), (2**31 + 5, 60000)])
def test_library_permutation_matches_oracle(seed, n):
    N, L = _lib()
    out = np.empty(n, np.int64)
    N.check(L.oxc_permutation(seed, n, out.ctypes.data))
    want = np.random.RandomState(seed).permutation(n)
    assert np.array_equal(out, want)
    if n <= 5000:
        assert out.tolist() == O.Mt19937(seed).permutation(n)


def test_library_seeds_match_oracle():
    N, L = _lib()
    for base, e in [(0, 0), (1, 3), (2**64 - 1, 7), (123456789, 2)]:
        assert L.oxc_epoch_seed(base, e) == O.epoch_seed(base, e)
    idx = np.array([5, 0, 3, 2**40], np.int64)
    for es in (0, 17, 2**63 + 11):
        assert L.oxc_batch_seed(es, idx.ctypes.data, len(idx)) == O.batch_seed(es, O.indices_seed(idx))


def _plan(L, N, order, batch_size, tseed, steps, shape):
    from oxitorch_b200.data import NativeTransform
    wire = []
    for s in steps:
        if s[0] == "crop":
            wire.append(("crop", [s[1]]))
        elif s[0] == "flip":
            wire.append(("flip", []))
        else:
            wire.append(("normalize", list(s[1]) + list(s[2])))
    tf = NativeTransform(wire)
    kinds, args, norm = tf._abi_arrays()
    rank = len(shape)
    row_shape = np.array(shape[1:], np.int64)
    used = len(order)
    cap = used * (shape[1] if rank == 4 else 1)
    planes = (N.PlaneMap * cap)()
    result = np.zeros(4, np.int64)
    order = np.ascontiguousarray(order, np.int64)
    st = L.oxc_epoch_transform_plan(order.ctypes.data, used, batch_size, tseed, kinds.ctypes.data,
                                    args.ctypes.data, norm.ctypes.data, len(kinds), rank,
                                    row_shape.ctypes.data, planes, cap, result.ctypes.data)
    return st, planes, result, tf


def _apply_planes(col, order, planes, nplanes, out_hw, norm_table, channels):
    """The image kernel's indexing, restated: plane q row r column x reads
    virtual element src_offset + (r + row_offset) * W + col_base + col_step * x."""
    n, W = col.shape[0], col.shape[-1]
    row_elems = col[0].size
    flat = col.reshape(n, row_elems)
    oh, ow = out_hw
    out = np.empty((nplanes, oh, ow), np.float32)
    xs = np.arange(ow)
    for q in range(nplanes):
        pm = planes[q]
        for r in range(oh):
            lin = pm.src_offset + (r + pm.row_offset) * W
            ds, off = divmod(lin, row_elems)
            v = flat[order[ds], off + pm.col_base + pm.col_step * xs].astype(np.float32)
            if norm_table is not None:
                for k in range(norm_table.shape[0] // 2):
                    v = ((v - norm_table[2 * k, pm.channel]).astype(np.float32)
                         * norm_table[2 * k + 1, pm.channel]).astype(np.float32)
            out[q, r] = v
    return out


@pytest.mark.parametrize("shape,bs,steps", [
    ((37, 3, 9, 8), 8, [("crop", 6), ("flip",), ("normalize", [0.5, 0.25, -1.0], [0.2, 3.0, 1.5])]),
    ((20, 1, 7, 7), 6, [("flip",), ("crop", 4), ("flip",)]),
    ((13, 2, 5, 6), 4, [("normalize", [1.0, 2.0], [2.0, 4.0]), ("crop", 5),
                        ("normalize", [0.1, -0.2], [0.7, 1.1])]),
    ((11, 6, 6), 11, [("crop", 3), ("flip",)]),
])
def test_library_transform_plan_reproduces_oracle(shape, bs, steps):
    N, L = _lib()
    rng = np.random.default_rng(len(shape) * 100 + bs)
    col = rng.standard_normal(shape).astype(np.float32)
    order = np.random.RandomState(bs).permutation(shape[0]).astype(np.int64)
    tseed = O.epoch_seed(77, 0)
    st, planes, result, tf = _plan(L, N, order, bs, tseed, steps, shape)
    assert st == 0, N.last_error()
    nplanes, oh, ow = int(result[0]), int(result[1]), int(result[2])
    channels = shape[1] if len(shape) == 4 else bs
    got = _apply_planes(col, order, planes, nplanes, (oh, ow), tf._norm_table(channels), channels)
    want = []
    for k in range(0, shape[0], bs):
        idx = order[k:k + bs].tolist()
        b = O.gather_columns([col], idx)[0]
        r = O.batch_rng(O.batch_seed(tseed, O.indices_seed(idx)))
        want.append(O.apply_transforms(b, steps, r).reshape(-1, oh, ow))
    want = np.concatenate(want)
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_library_transform_plan_reports_the_failing_batch():
    N, L = _lib()
    # rank 3: the batch is one sample whose channels are its rows; normalize
    # with 4 channels fits the full batches of 4 and fails on the last (3)
    order = np.arange(11, dtype=np.int64)
    st, planes, result, _ = _plan(L, N, order, 4, 1, [("normalize", [0.0] * 4, [1.0] * 4)], (11, 3, 3))
    assert st == 1 and int(result[3]) == 2 and int(result[0]) == 8
    assert "normalize expects 3 channels, got mean 4 / std 4" in N.last_error()
    st, _, result, _ = _plan(L, N, order, 4, 1, [("crop", 4)], (11, 3, 3))
    assert st == 1 and int(result[3]) == 0 and "crop size 4 exceeds image 3x3" in N.last_error()


def test_native_transform_wire_errors():
    from oxitorch_b200.data import NativeTransform
    with pytest.raises(ValueError, match="crop expects a single non-negative size argument"):
        NativeTransform([("crop", [])])
    with pytest.raises(ValueError, match="flip expects no arguments"):
        NativeTransform([("flip", [1.0])])
    with pytest.raises(ValueError, match="normalize expects mean... followed by std"):
        NativeTransform([("normalize", [1.0, 2.0, 3.0])])
    with pytest.raises(ValueError, match="unknown native transform 'blur'"):
        NativeTransform([("blur", [])])


def test_library_transform_plan_rejects_bad_arguments():
    N, L = _lib()
    order = np.arange(4, dtype=np.int64)
    kinds = np.array([2], np.int32)
    args = np.array([1], np.int64)
    result = np.zeros(4, np.int64)
    planes = (N.PlaneMap * 4)()
    shape = np.array([1, 2, 2], np.int64)
    # a normalize step without its parameters
    assert L.oxc_epoch_transform_plan(order.ctypes.data, 4, 2, 0, kinds.ctypes.data, args.ctypes.data,
                                      None, 1, 4, shape.ctypes.data, planes, 4, result.ctypes.data) == 1
    # no row shape, a zero dim, an unknown kind, a negative crop
    assert L.oxc_epoch_transform_plan(order.ctypes.data, 4, 2, 0, None, None, None, 0, 4, None, planes,
                                      4, result.ctypes.data) == 1
    zero = np.array([1, 0, 2], np.int64)
    assert L.oxc_epoch_transform_plan(order.ctypes.data, 4, 2, 0, None, None, None, 0, 4,
                                      zero.ctypes.data, planes, 4, result.ctypes.data) == 1
    bad = np.array([7], np.int32)
    assert L.oxc_epoch_transform_plan(order.ctypes.data, 4, 2, 0, bad.ctypes.data, args.ctypes.data,
                                      None, 1, 4, shape.ctypes.data, planes, 4, result.ctypes.data) == 1
    crop = np.array([0], np.int32)
    neg = np.array([-3], np.int64)
    assert L.oxc_epoch_transform_plan(order.ctypes.data, 4, 2, 0, crop.ctypes.data, neg.ctypes.data,
                                      None, 1, 4, shape.ctypes.data, planes, 4, result.ctypes.data) == 1
    # too small a plane buffer
    flip = np.array([1], np.int32)
    zarg = np.array([0], np.int64)
    assert L.oxc_epoch_transform_plan(order.ctypes.data, 4, 2, 0, flip.ctypes.data, zarg.ctypes.data,
                                      None, 1, 4, shape.ctypes.data, planes, 1, result.ctypes.data) == 1
    assert "plane buffer holds 1 planes" in N.last_error()


@pytest.mark.parametrize("case", range(12))
def test_library_transform_plan_random_pipelines(case):
    """Seeded random pipelines of one to five steps over rank-3 and rank-4
    columns with ragged last batches: the composed plane maps, applied with
    the kernel's indexing, reproduce the oracle batch by batch."""
    N, L = _lib()
    rng = np.random.default_rng(1000 + case)
    rank = 4 if case % 3 else 3
    c = int(rng.integers(1, 4))
    h, w = int(rng.integers(3, 9)), int(rng.integers(3, 9))
    n = int(rng.integers(5, 30))
    bs = int(rng.integers(1, 9))
    shape = (n, c, h, w) if rank == 4 else (n, h, w)
    steps, ch, hh, ww = [], None, h, w
    for _ in range(int(rng.integers(1, 6))):
        kind = rng.choice(["crop", "flip", "normalize"])
        if kind == "crop":
            size = int(rng.integers(1, min(hh, ww) + 1))
            steps.append(("crop", size))
            hh = ww = size
        elif kind == "flip":
            steps.append(("flip",))
        elif rank == 4 and sum(s[0] == "normalize" for s in steps) < 4:
            mean = rng.standard_normal(c).astype(np.float32).tolist()
            std = rng.uniform(0.2, 2.0, c).astype(np.float32).tolist()
            steps.append(("normalize", mean, std))
    if not steps:
        steps = [("flip",)]
    col = rng.standard_normal(shape).astype(np.float32)
    order = np.random.RandomState(case).permutation(n).astype(np.int64)
    tseed = O.epoch_seed(case, 3)
    st, planes, result, tf = _plan(L, N, order, bs, tseed, steps, shape)
    assert st == 0, N.last_error()
    nplanes, oh, ow = int(result[0]), int(result[1]), int(result[2])
    channels = c if rank == 4 else bs
    got = _apply_planes(col, order, planes, nplanes, (oh, ow), tf._norm_table(channels), channels)
    want = []
    for k in range(0, n, bs):
        idx = order[k:k + bs].tolist()
        b = O.gather_columns([col], idx)[0]
        r = O.batch_rng(O.batch_seed(tseed, O.indices_seed(idx)))
        want.append(O.apply_transforms(b, steps, r).reshape(-1, oh, ow))
    want = np.concatenate(want)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
