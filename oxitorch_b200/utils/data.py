"""``torch.utils.data``-style pipeline: the reference's
``oxitorch.utils.data`` (python/oxitorch/utils/data.py:43-340), with the same
classes, arguments, epoch seeding and errors.

Two paths behind one ``DataLoader``, chosen as the reference chooses them
(data.py:217-264):

* datasets exposing ``tensors`` (``TensorDataset``, or a dataset without
  per-item transforms), or ``native_parts`` (raw columns plus a native
  transform repr), with no sampler and the default collation, go to
  ``oxitorch_b200.data.DataLoader``: columns resident on the device, each
  epoch built by two launches.  Each pass constructs it with the epoch seed
  ``seed + epoch`` (a random base when ``seed`` is None), like the
  reference's fresh ``_native.DataLoader`` per pass.  Host columns are
  uploaded on the first pass and stay resident for the later ones (the
  reference copies them again on every pass); CUDA columns are used in place;
* a tensor-backed dataset driven by a sampler or batch sampler keeps the
  default collation's result (the sampled rows stacked per column, float32)
  but builds it with one device gather per batch;
* anything else runs the reference's generic path: per-item ``__getitem__``
  (in a thread pool when ``num_workers > 1``) and ``default_collate``, whose
  stacked host arrays are uploaded with ``from_numpy``.
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch

from .. import data as _device

__all__ = [
    "DataLoader",
    "Dataset",
    "IterableDataset",
    "RandomSampler",
    "SequentialSampler",
    "Subset",
    "TensorDataset",
    "default_collate",
]


class Dataset:
    """Map-style datasets implement ``__getitem__`` and ``__len__``."""

    def __getitem__(self, index):
        raise NotImplementedError

    def __len__(self):
        raise NotImplementedError


class IterableDataset(Dataset):
    """Stream-style datasets implement ``__iter__``."""

    def __iter__(self):
        raise NotImplementedError


class TensorDataset(Dataset):
    """Zips columns along dim 0: ``TensorDataset(features, labels)``."""

    def __init__(self, *tensors):
        n = tensors[0].shape[0]
        for i, t in enumerate(tensors):
            if t.shape[0] != n:
                raise ValueError(f"tensor {i} has {t.shape[0]} rows, expected {n}")
        self.tensors = tensors

    def __getitem__(self, index):
        return tuple(t[index] for t in self.tensors)

    def __len__(self):
        return self.tensors[0].shape[0]


class Subset(Dataset):
    """A fixed-index view of another dataset (generic path)."""

    def __init__(self, dataset, indices):
        self.dataset = dataset
        self.indices = list(indices)

    def __getitem__(self, index):
        return self.dataset[self.indices[index]]

    def __len__(self):
        return len(self.indices)


class Sampler:
    def __iter__(self):
        raise NotImplementedError

    def __len__(self):
        raise NotImplementedError


class SequentialSampler(Sampler):
    def __init__(self, data_source):
        self.data_source = data_source

    def __iter__(self):
        return iter(range(len(self.data_source)))

    def __len__(self):
        return len(self.data_source)


class RandomSampler(Sampler):
    """Permuted indices; a seeded sampler draws NumPy's
    ``RandomState(seed + epoch).permutation`` per pass (data.py:114-131)."""

    def __init__(self, data_source, seed=None):
        self.data_source = data_source
        self.seed = seed
        self._epoch = 0

    def __iter__(self):
        n = len(self.data_source)
        if self.seed is None:
            order = np.random.permutation(n)
        else:
            order = np.random.RandomState(self.seed + self._epoch).permutation(n)
            self._epoch += 1
        return iter(int(i) for i in order)

    def __len__(self):
        return len(self.data_source)


def _host_array(x):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().numpy()
    return np.asarray(x)


def default_collate(items):
    """data.py:135-164: tuples per field; arrays and tensors stacked to f32;
    numbers to an f32 label tensor; every batch a float32 CUDA tensor."""
    if not items:
        raise ValueError("cannot collate an empty item list")
    first = items[0]
    if isinstance(first, (tuple, list)):
        return tuple(default_collate([item[i] for item in items]) for i in range(len(first)))
    if isinstance(first, (np.ndarray, torch.Tensor)):
        stacked = np.stack([np.asarray(_host_array(x), dtype=np.float32) for x in items])
        out = _device.from_numpy(np.ascontiguousarray(stacked))
        if isinstance(first, torch.Tensor) and all(bool(x.requires_grad) for x in items):
            out.requires_grad_(True)
        return out
    if isinstance(first, (int, float, np.integer, np.floating)):
        return _device.from_numpy(np.ascontiguousarray(np.asarray(items, dtype=np.float32)))
    raise TypeError(f"default_collate cannot handle items of type {type(first)!r}")


class DataLoader:
    """Batches a dataset; torch's constructor surface (data.py:167-340)."""

    def __init__(self, dataset, batch_size=1, shuffle=False, sampler=None, batch_sampler=None,
                 num_workers=0, collate_fn=default_collate, drop_last=False, seed=None):
        if batch_size < 1:
            raise ValueError("batch_size must be >= 1")
        self.dataset = dataset
        self.batch_size = batch_size
        self.shuffle = shuffle
        self.sampler = sampler
        self.batch_sampler = batch_sampler
        self.num_workers = num_workers
        self.collate_fn = collate_fn
        self.drop_last = drop_last
        self.seed = seed
        self._auto_seed = int.from_bytes(os.urandom(4), "little")
        self._epoch = 0
        self._resident = None  # the dataset's columns on the device, uploaded once

    def __len__(self):
        n = self._length_source()
        if self.batch_sampler is not None:
            return len(self.batch_sampler)
        if self.drop_last:
            return n // self.batch_size
        return (n + self.batch_size - 1) // self.batch_size

    def _length_source(self):
        if isinstance(self.dataset, IterableDataset):
            raise TypeError("IterableDataset has no length; len(DataLoader) is undefined")
        return len(self.dataset)

    def _device_loader_for(self, epoch):
        """The device loader for tensor-backed datasets, or None."""
        if self.sampler is not None or self.batch_sampler is not None:
            return None
        if self.collate_fn is not default_collate:
            return None
        base = self.seed if self.seed is not None else self._auto_seed
        epoch_seed = base + epoch
        parts = getattr(self.dataset, "native_parts", None)
        transforms = None
        if parts is not None:
            raw, native_repr = parts
            transforms = _device.NativeTransform(native_repr)
        else:
            raw = getattr(self.dataset, "tensors", None)
            if raw is None:
                return None
        if self._resident is None or self._resident[0] is not raw:
            self._resident = (raw, [c if isinstance(c, torch.Tensor) and c.is_cuda
                                    else _device.from_numpy(np.ascontiguousarray(_host_array(c)))
                                    for c in raw])
        return _device.DataLoader(self._resident[1], batch_size=self.batch_size, shuffle=self.shuffle,
                                  drop_last=self.drop_last, seed=epoch_seed,
                                  num_workers=self.num_workers, transforms=transforms,
                                  transform_seed=epoch_seed)

    def __iter__(self):
        epoch = self._epoch
        self._epoch += 1
        loader = self._device_loader_for(epoch)
        if loader is not None:
            yield from iter(loader)
            return
        if self.batch_sampler is not None:
            for idx in self.batch_sampler:
                yield self._collate_index_batch(list(idx))
            return
        if isinstance(self.dataset, IterableDataset):
            yield from self._iter_stream()
            return
        if self.sampler is not None:
            indices = iter(self.sampler)
        elif self.shuffle:
            indices = iter(RandomSampler(self.dataset, seed=self._seed_for_epoch(epoch)))
        else:
            indices = iter(SequentialSampler(self.dataset))
        yield from self._iter_index_batches(indices)

    def _seed_for_epoch(self, epoch):
        return None if self.seed is None else self.seed + epoch

    def _iter_index_batches(self, indices):
        batch = []
        for i in indices:
            batch.append(i)
            if len(batch) == self.batch_size:
                yield self._collate_index_batch(batch)
                batch = []
        if batch and (not self.drop_last or len(batch) == self.batch_size):
            yield self._collate_index_batch(batch)

    def _gatherable_columns(self):
        """The resident device columns when a batch of items can be gathered
        on the device (tensor columns, default collation, no per-item
        transform), else None."""
        if self.collate_fn is not default_collate:
            return None
        raw = getattr(self.dataset, "tensors", None)
        if raw is None or getattr(self.dataset, "native_parts", None) is not None:
            return None
        if any(isinstance(c, torch.Tensor) and c.requires_grad for c in raw):
            return None  # default_collate keeps requires_grad: take the per-item path
        if self._resident is None or self._resident[0] is not raw:
            self._resident = (raw, [c if isinstance(c, torch.Tensor) and c.is_cuda
                                    else _device.from_numpy(np.ascontiguousarray(_host_array(c)))
                                    for c in raw])
        return self._resident[1]

    def _iter_stream(self):
        items = []
        for item in self.dataset:
            items.append(item)
            if len(items) == self.batch_size:
                yield self.collate_fn(items)
                items = []
        if items and not self.drop_last:
            yield self.collate_fn(items)

    def _collate_index_batch(self, batch):
        cols = self._gatherable_columns()
        if cols is not None:
            # default_collate of TensorDataset items is the rows stacked per
            # column, as float32: one device gather instead of per-item fetches
            out = _device.gather_rows(cols, batch)
            return tuple(o if o.dtype == torch.float32 else o.float() for o in out)
        if self.num_workers > 1 and len(batch) > 1:
            with ThreadPoolExecutor(max_workers=self.num_workers) as pool:
                items = list(pool.map(self.dataset.__getitem__, batch))
        else:
            items = [self.dataset[i] for i in batch]
        return self.collate_fn(items)
