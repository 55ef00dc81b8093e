"""The data path on the device: the reference's native ``DataLoader`` and
``NativeTransform`` (crates/oxi-bindings/src/data.rs:60-330) and its
``from_numpy`` / ``Tensor.numpy`` copies (crates/oxi-bindings/src/lib.rs:769-780,
382-391), with the same constructor arguments, defaults, batch order,
augmentation draws and errors.

The reference gathers every batch on CPU worker threads.  Here the dataset
columns are uploaded once and stay in device memory, and each ``__iter__``
builds the whole epoch with two launches:

* the host computes the epoch order (``oxc_permutation``: MT19937, the
  reference's shuffle stream) and, when there are transforms, every batch's
  crop and flip draws (``oxc_epoch_transform_plan``), in the library's C++;
* ``oxc_gather_rows`` gathers the plain columns for the whole epoch, and
  ``oxc_image_epoch`` gathers, crops, flips and normalises the image column
  in one pass;
* batches are views of those epoch buffers, in plan order.

``num_workers`` is accepted for signature parity; there are no worker
threads to size.  A transform the reference rejects at batch ``k`` yields
batches ``0..k`` and then raises at ``k``, with the reference's message.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N

_KINDS = {"crop": 0, "flip": 1, "normalize": 2}


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def from_numpy(array, device=None) -> torch.Tensor:
    """A float32 device tensor holding ``array`` (``oxitorch.from_numpy``),
    copied through the library's pinned staging ring (``oxc_upload``)."""
    a = np.asarray(array)
    if a.dtype != np.float32:
        raise TypeError("expected a numpy array or f32 buffer object")
    a = np.ascontiguousarray(a)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    L = N.load()
    out = torch.empty(a.shape, dtype=torch.float32, device=dev)
    N.check(L.oxc_upload(out.data_ptr(), a.ctypes.data, a.nbytes, _stream(dev)), "from_numpy")
    return out


def to_numpy(tensor: torch.Tensor) -> np.ndarray:
    """A host copy of a device tensor (``Tensor.numpy``), through
    ``oxc_download``; non-contiguous tensors are made contiguous first."""
    if not isinstance(tensor, torch.Tensor) or not tensor.is_cuda:
        raise ValueError("invalid argument: to_numpy takes a CUDA tensor (oxitorch_b200 has no CPU path)")
    t = tensor.detach().contiguous()
    out = np.empty(tuple(t.shape), dtype=np.dtype(str(t.dtype).replace("torch.", "")))
    L = N.load()
    N.check(L.oxc_download(out.ctypes.data, t.data_ptr(), out.nbytes, _stream(t.device)), "to_numpy")
    return out


def gather_rows(columns, indices):
    """``[c[indices] for c in columns]`` for device columns: one
    ``oxc_gather_rows`` launch per 8 columns, the indices uploaded once.
    Indices are validated on the host like NumPy indexing (negative ones
    count from the end; out of range raises IndexError)."""
    cols = list(columns)
    n = cols[0].shape[0]
    idx = np.asarray(indices, dtype=np.int64).reshape(-1)
    if idx.size and (idx.min() < -n or idx.max() >= n):
        bad = int(idx[(idx < -n) | (idx >= n)][0])
        raise IndexError(f"index {bad} is out of bounds for axis 0 with size {n}")
    idx = np.where(idx < 0, idx + n, idx)
    dev = cols[0].device
    stream = _stream(dev)
    L = N.load()
    outs = [torch.empty((idx.size,) + tuple(c.shape[1:]), dtype=c.dtype, device=dev) for c in cols]
    if idx.size == 0:
        return outs
    idx_dev = torch.empty(idx.size, dtype=torch.int64, device=dev)
    N.check(L.oxc_upload(idx_dev.data_ptr(), idx.ctypes.data, idx.nbytes, stream), "gather indices")
    for g in range(0, len(cols), 8):
        group = list(zip(cols[g:g + 8], outs[g:g + 8]))
        desc = (N.GatherColumn * len(group))(*[
            N.GatherColumn(c.data_ptr(), o.data_ptr(), c[0].numel() * c.element_size() if c.dim() > 1
                           else c.element_size()) for c, o in group])
        N.check(L.oxc_gather_rows(desc, len(group), idx_dev.data_ptr(), idx.size, n, None, stream),
                "gather_rows")
    return outs


class NativeTransform:
    """The augmentation pipeline applied to the first column inside the
    loader (data.rs:60-105).  Wire format: ``("crop", [size])``,
    ``("flip", [])`` and ``("normalize", [mean..., std...])``."""

    def __init__(self, steps):
        parsed = []
        for name, args in steps:
            args = [float(a) for a in args]
            if name == "crop":
                if len(args) != 1 or not args[0] >= 0.0:
                    raise ValueError("crop expects a single non-negative size argument")
                parsed.append(("crop", int(args[0])))
            elif name == "flip":
                if args:
                    raise ValueError("flip expects no arguments")
                parsed.append(("flip",))
            elif name == "normalize":
                if len(args) < 2 or len(args) % 2:
                    raise ValueError("normalize expects mean... followed by std... of equal length")
                mid = len(args) // 2
                parsed.append(("normalize", np.float32(args[:mid]), np.float32(args[mid:])))
            else:
                raise ValueError(f"unknown native transform {name!r}")
        self.steps = parsed

    def _abi_arrays(self):
        kinds = np.array([_KINDS[s[0]] for s in self.steps], dtype=np.int32)
        args = np.array([s[1] if s[0] == "crop" else (len(s[1]) if s[0] == "normalize" else 0)
                         for s in self.steps], dtype=np.int64)
        packed = [np.concatenate([s[1], s[2]]) for s in self.steps if s[0] == "normalize"]
        norm = np.concatenate(packed).astype(np.float32) if packed else np.zeros(1, np.float32)
        return kinds, args, norm

    def _norm_table(self, channels):
        """[nnorm][2][channels]: each normalize step's mean, then 1/std in f32
        (transform.rs:185-188)."""
        rows = []
        for s in self.steps:
            if s[0] == "normalize":
                rows.append(s[1][:channels])
                rows.append((np.float32(1.0) / s[2][:channels]).astype(np.float32))
        return np.stack(rows).astype(np.float32) if rows else None


class _EpochSeeds:
    """The reference's per-loader epoch counter (data.rs:38-55)."""

    def __init__(self, base):
        self.base, self.counter = base, 0

    def next(self, L):
        seed = L.oxc_epoch_seed(self.base & (2**64 - 1), self.counter)
        self.counter += 1
        return seed


class DataLoader:
    """``DataLoader(columns, batch_size=1, shuffle=False, drop_last=False,
    seed=None, num_workers=0, transforms=None, transform_seed=0)``: batches of
    column tensors in the reference's order (data.rs:140-262).  Columns are
    CUDA tensors, or numpy arrays / CPU tensors that are uploaded once."""

    def __init__(self, columns, batch_size=1, shuffle=False, drop_last=False, seed=None,
                 num_workers=0, transforms=None, transform_seed=0, device=None):
        columns = list(columns)
        if not columns:
            raise ValueError("DataLoader needs at least one tensor column")
        cols = [self._to_device(c, device) for c in columns]
        n = cols[0].shape[0] if cols[0].dim() else 0
        if n == 0:
            raise ValueError("DataLoader dataset is empty")
        if batch_size == 0:
            raise ValueError("batch_size must be >= 1")
        for i, c in enumerate(cols):
            if c.dim() == 0 or c.shape[0] != n:
                raise ValueError(f"column {i} has {c.shape[0] if c.dim() else 0} rows, expected {n}")
        if transforms is not None and not transforms.steps:
            raise ValueError("transforms pipeline is empty; pass None instead")
        self.columns = cols
        self._n = n
        self._batch_size = int(batch_size)
        self.shuffle = bool(shuffle)
        self.drop_last = bool(drop_last)
        self.num_workers = int(num_workers)
        self.transforms = transforms
        self._seeds = _EpochSeeds(seed) if seed is not None else None
        self._tseeds = _EpochSeeds(transform_seed)

    @staticmethod
    def _to_device(c, device):
        if isinstance(c, torch.Tensor) and c.is_cuda:
            return c.contiguous()
        a = c.numpy() if isinstance(c, torch.Tensor) else np.asarray(c)
        return from_numpy(a, device)

    @property
    def n(self):
        return self._n

    @property
    def batch_size(self):
        return self._batch_size

    def _order(self, L):
        if self.shuffle and self._seeds is not None:
            seed = self._seeds.next(L)
            order = np.empty(self._n, np.int64)
            N.check(L.oxc_permutation(seed & 0xFFFFFFFF, self._n, order.ctypes.data), "permutation")
            return order
        return np.arange(self._n, dtype=np.int64)

    def _used(self):
        """Rows the epoch plan covers (batch.rs:271-291): a short last batch
        is dropped with drop_last only when an earlier batch exists."""
        bs, n = self._batch_size, self._n
        if self.drop_last and n % bs and n >= bs:
            return n - n % bs
        return n

    def __iter__(self):
        L = N.load()
        ep = self._plan_epoch(L)
        self._launch_epoch(L, ep)
        N.check(L.oxc_check_error_flag(ep.err.data_ptr(), ep.stream, 60000), "loader")
        return self._batches(ep.outs, ep.used, ep.failed, ep.fail_msg)

    def _plan_epoch(self, L):
        """The host half of an epoch: this pass's order and transform draws
        (advancing the epoch counters), their upload, and the epoch buffers."""
        ep = _Epoch()
        dev = self.columns[0].device
        ep.stream = _stream(dev)
        order = self._order(L)
        tseed = self._tseeds.next(L)
        ep.used = used = self._used()
        ep.order_dev = torch.empty(used, dtype=torch.int64, device=dev)
        N.check(L.oxc_upload(ep.order_dev.data_ptr(), order.ctypes.data, used * 8, ep.stream),
                "loader order")
        ep.err = torch.zeros(4, dtype=torch.int32, device=dev)
        plain = self.columns[1:] if self.transforms else self.columns
        plain_out = [torch.empty((used,) + tuple(c.shape[1:]), dtype=c.dtype, device=dev)
                     for c in plain]
        ep.groups = []
        for g in range(0, len(plain), 8):
            group = list(zip(plain[g:g + 8], plain_out[g:g + 8]))
            ep.groups.append((N.GatherColumn * len(group))(*[
                N.GatherColumn(c.data_ptr(), o.data_ptr(), c[0].numel() * c.element_size())
                for c, o in group]))
        ep.image = None
        if self.transforms:
            self._plan_image(L, ep, order, tseed)
            ep.outs = [ep.image["out"]] + plain_out
        else:
            ep.outs = plain_out
        return ep

    def _plan_image(self, L, ep, order, tseed):
        col = self.columns[0]
        if col.dtype != torch.float32:
            raise ValueError("invalid argument: transforms take a float32 image column")
        rank = col.dim()
        row_shape = np.array(col.shape[1:], dtype=np.int64)
        kinds, args, norm = self.transforms._abi_arrays()
        used = ep.used
        cap = used * (int(row_shape[0]) if rank == 4 else 1)
        planes = (N.PlaneMap * max(cap, 1))()
        result = np.zeros(4, np.int64)
        st = L.oxc_epoch_transform_plan(order.ctypes.data, used, self._batch_size, tseed,
                                        kinds.ctypes.data, args.ctypes.data, norm.ctypes.data,
                                        len(kinds), rank, row_shape.ctypes.data, planes, cap,
                                        result.ctypes.data)
        if st != 0:
            if result[3] < 0:
                N.check(st, "transforms")
            ep.failed, ep.fail_msg = int(result[3]), N.last_error()
        nplanes, out_h, out_w = int(result[0]), int(result[1]), int(result[2])
        rows = used if ep.failed is None else ep.failed * self._batch_size
        dev = col.device
        im = {"nplanes": nplanes, "out_h": out_h, "out_w": out_w, "table": None, "planes": None,
              "out": torch.empty((rows,) + tuple(col.shape[1:-2]) + (out_h, out_w),
                                 dtype=torch.float32, device=dev),
              "channels": int(row_shape[0]) if rank == 4 else min(self._batch_size, used)}
        if nplanes:
            pl = torch.empty(nplanes * ctypes.sizeof(N.PlaneMap), dtype=torch.uint8, device=dev)
            N.check(L.oxc_upload(pl.data_ptr(), ctypes.addressof(planes), pl.numel(), ep.stream),
                    "planes")
            im["planes"] = pl
            table = self.transforms._norm_table(im["channels"])
            if table is not None:
                nt = torch.empty(table.size, dtype=torch.float32, device=dev)
                N.check(L.oxc_upload(nt.data_ptr(), table.ctypes.data, table.nbytes, ep.stream),
                        "normalize table")
                im["table"], im["nnorm"] = nt, table.shape[0] // 2
        ep.image = im

    def _launch_epoch(self, L, ep):
        """The device half: one gather launch per 8 plain columns and one
        image launch, all on the current stream."""
        for desc in ep.groups:
            N.check(L.oxc_gather_rows(desc, len(desc), ep.order_dev.data_ptr(), ep.used, self._n,
                                      ep.err.data_ptr(), ep.stream), "loader gather")
        im = ep.image
        if im is not None and im["nplanes"]:
            col = self.columns[0]
            table = im["table"]
            N.check(L.oxc_image_epoch(col.data_ptr(), col[0].numel(), ep.order_dev.data_ptr(), ep.used,
                                      self._n, im["planes"].data_ptr(), im["nplanes"],
                                      int(col.shape[-2]), int(col.shape[-1]), im["out_h"], im["out_w"],
                                      None if table is None else table.data_ptr(),
                                      0 if table is None else im["nnorm"], im["channels"],
                                      im["out"].data_ptr(), ep.err.data_ptr(), ep.stream),
                    "image epoch")

    def _batches(self, outs, used, failed, msg):
        bs = self._batch_size
        nb = (used + bs - 1) // bs
        for k in range(nb):
            if failed is not None and k == failed:
                if self.num_workers == 0:
                    raise RuntimeError(f"DataLoader failed at batch {k}: {msg}")
                raise RuntimeError(f"DataLoader worker failed: {msg}")
            yield [o[k * bs:min(used, (k + 1) * bs)] for o in outs]


class _Epoch:
    """One planned epoch: device order, gather descriptors, image plan, outputs."""

    failed = None
    fail_msg = None
