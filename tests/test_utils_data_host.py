"""oxitorch_b200.utils.data on the CPU: the routing, epoch seeding, samplers,
lengths and collation of the reference's utils/data.py (python/oxitorch/utils/
data.py:43-340), with the device calls replaced by recording fakes so that no
GPU is needed.  The device loader itself is checked against the oracle in
tests/test_gpu_loader.py."""

import numpy as np
import pytest

from oxitorch_b200 import data as device
from oxitorch_b200.utils import data as D


class _FakeLoader:
    made = []

    def __init__(self, columns, **kw):
        self.columns, self.kw = columns, kw
        _FakeLoader.made.append(self)

    def __iter__(self):
        return iter([["batch", self.kw["seed"]]])


@pytest.fixture
def fakes(monkeypatch):
    _FakeLoader.made = []
    uploads = []

    def fake_from_numpy(a, device=None):
        uploads.append(np.array(a))
        return np.array(a)

    def fake_gather_rows(columns, indices):
        import torch
        return [torch.from_numpy(np.asarray(c)[np.asarray(indices, np.int64)]) for c in columns]

    monkeypatch.setattr(device, "DataLoader", _FakeLoader)
    monkeypatch.setattr(device, "from_numpy", fake_from_numpy)
    monkeypatch.setattr(device, "gather_rows", fake_gather_rows)
    return uploads


def test_tensor_dataset_goes_to_the_device_loader_with_epoch_seeds(fakes):
    x = np.arange(12, dtype=np.float32).reshape(6, 2)
    y = np.arange(6, dtype=np.float32)
    loader = D.DataLoader(D.TensorDataset(x, y), batch_size=4, shuffle=True, seed=7, num_workers=3)
    assert list(loader) == [["batch", 7]]
    assert list(loader) == [["batch", 8]]
    a, b = _FakeLoader.made
    assert a.kw == dict(batch_size=4, shuffle=True, drop_last=False, seed=7, num_workers=3,
                        transforms=None, transform_seed=7)
    assert b.kw["seed"] == 8 and b.kw["transform_seed"] == 8
    assert len(fakes) == 2  # both columns uploaded once, then resident
    assert len(loader) == 2


def test_native_parts_carry_the_transform(fakes):
    class Images(D.Dataset):
        native_parts = ((np.zeros((3, 1, 4, 4), np.float32), np.zeros(3, np.float32)),
                        [("crop", [2.0]), ("flip", [])])

        def __len__(self):
            return 3

    list(D.DataLoader(Images(), batch_size=2, seed=1))
    kw = _FakeLoader.made[0].kw
    assert [s[0] for s in kw["transforms"].steps] == ["crop", "flip"]


def test_samplers_and_custom_collate_take_the_generic_path(fakes):
    x = np.arange(10, dtype=np.float32)
    ds = D.TensorDataset(x)
    got = list(D.DataLoader(ds, batch_size=4, sampler=[9, 1, 3, 5, 7], collate_fn=lambda it: it))
    assert got == [[(9.0,), (1.0,), (3.0,), (5.0,)], [(7.0,)]]
    assert not _FakeLoader.made
    # a sampler with the default collation: the sampled rows, gathered per batch
    batches = list(D.DataLoader(ds, batch_size=3, sampler=D.SequentialSampler(ds), drop_last=True))
    assert len(batches) == 3 and np.array_equal(batches[1][0], [3.0, 4.0, 5.0])
    got = list(D.DataLoader(ds, batch_sampler=[[4, 2], [9]]))
    assert np.array_equal(got[0][0], [4.0, 2.0]) and np.array_equal(got[1][0], [9.0])


def test_random_sampler_streams():
    ds = D.TensorDataset(np.zeros(20, np.float32))
    s = D.RandomSampler(ds, seed=4)
    assert list(s) == list(np.random.RandomState(4).permutation(20))
    assert list(s) == list(np.random.RandomState(5).permutation(20))


def test_lengths_and_errors(fakes):
    ds = D.TensorDataset(np.zeros(10, np.float32))
    assert len(D.DataLoader(ds, batch_size=4)) == 3
    assert len(D.DataLoader(ds, batch_size=4, drop_last=True)) == 2
    with pytest.raises(ValueError, match="batch_size must be >= 1"):
        D.DataLoader(ds, batch_size=0)
    with pytest.raises(ValueError, match="tensor 1 has 3 rows, expected 10"):
        D.TensorDataset(np.zeros(10), np.zeros(3))

    class Stream(D.IterableDataset):
        def __iter__(self):
            return iter(range(5))

    with pytest.raises(TypeError, match="IterableDataset has no length"):
        len(D.DataLoader(Stream()))
    assert [list(b) for b in D.DataLoader(Stream(), batch_size=2, drop_last=True)] == [[0, 1], [2, 3]]
    with pytest.raises(ValueError, match="cannot collate an empty item list"):
        D.default_collate([])
    with pytest.raises(TypeError, match="default_collate cannot handle items of type"):
        D.default_collate(["a"])
    pair = D.default_collate([(np.ones(2, np.float32), 1), (np.zeros(2, np.float32), 0)])
    assert np.array_equal(pair[0], [[1, 1], [0, 0]]) and np.array_equal(pair[1], [1.0, 0.0])
