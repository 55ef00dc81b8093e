"""oxc_layer_norm_bwd_noalloc: the LayerNorm(+GELU) backward for callers that
cannot allocate device memory (a host that owns all device memory through
its own pool, or a latency-critical step that cannot take cudaMalloc's
implicit synchronisation).  Its scratch is a fixed 16 MiB array inside the
library instead of a caller workspace.

This file is collected last on purpose, so that a run stopping at the first
failure has already run every other test.  It passes both on its own in a
fresh process and after the rest of the suite (the array's contents from
earlier calls must not matter).
"""

import numpy as np
import pytest

from parity import assert_bitexact

pytestmark = pytest.mark.gpu


def _inputs(rows, cols, seed):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randn(rows, cols, device="cuda", generator=g)
    dy = torch.randn(rows, cols, device="cuda", generator=g)
    w = torch.rand(cols, device="cuda", generator=g) + 0.5
    b = torch.randn(cols, device="cuda", generator=g) * 0.1
    return x, dy, w, b


def _bwd_with_workspace(L, N, x, dy, w, b, mean, rstd, act, stream):
    import torch
    rows, cols = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(cols, device="cuda")
    db = torch.empty(cols, device="cuda")
    nbytes = L.oxc_layer_norm_bwd_workspace_size(rows, cols)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    N.check(L.oxc_layer_norm_bwd(x.data_ptr(), w.data_ptr(), b.data_ptr(), mean.data_ptr(),
                                 rstd.data_ptr(), dy.data_ptr(), dx.data_ptr(), dw.data_ptr(),
                                 db.data_ptr(), rows, cols, act, N.GRAD_REF, ws.data_ptr(), nbytes,
                                 stream))
    return dx, dw, db


def _bwd_noalloc(L, N, x, dy, w, b, mean, rstd, act, stream):
    import torch
    rows, cols = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(cols, device="cuda")
    db = torch.empty(cols, device="cuda")
    N.check(L.oxc_layer_norm_bwd_noalloc(x.data_ptr(), w.data_ptr(), b.data_ptr(),
                                         mean.data_ptr(), rstd.data_ptr(), dy.data_ptr(),
                                         dx.data_ptr(), dw.data_ptr(), db.data_ptr(), rows, cols,
                                         act, N.GRAD_REF, stream))
    return dx, dw, db


@pytest.mark.parametrize("rows,cols,act", [(4096, 4096, 1), (1000, 777, 0)])
def test_noalloc_matches_workspace_entry_point_twice(rows, cols, act):
    import torch
    from oxitorch_b200 import _native as N
    L = N.load()
    stream = torch.cuda.current_stream().cuda_stream
    x, dy, w, b = _inputs(rows, cols, 1234 + rows)
    y = torch.empty_like(x)
    mean = torch.empty(rows, device="cuda")
    rstd = torch.empty(rows, device="cuda")
    N.check(L.oxc_layer_norm_fwd(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(),
                                 mean.data_ptr(), rstd.data_ptr(), rows, cols, 1e-5, act, stream))
    want = [t.cpu().numpy() for t in _bwd_with_workspace(L, N, x, dy, w, b, mean, rstd, act, stream)]
    # Two calls in a row share (and reuse) the fixed scratch.  The same kernels
    # run with the same CTA and partial geometry as the workspace entry point,
    # so the results must be identical bit for bit, not merely close.
    for call in range(2):
        got = [t.cpu().numpy() for t in _bwd_noalloc(L, N, x, dy, w, b, mean, rstd, act, stream)]
        for name, g, r in zip(("dx", "dweight", "dbias"), got, want):
            assert_bitexact(g, r, what=f"call {call}: {name}")


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch():
    import torch
    from oxitorch_b200 import _native as N
    L = N.load()
    rows, cols = 1 << 20, 32768
    assert L.oxc_layer_norm_bwd_workspace_size(rows, cols) > N.NOALLOC_SCRATCH_BYTES
    t = torch.zeros(4, device="cuda")
    p = t.data_ptr()
    st = L.oxc_layer_norm_bwd_noalloc(p, p, p, p, p, p, p, p, p, rows, cols, 1, N.GRAD_REF,
                                      torch.cuda.current_stream().cuda_stream)
    with pytest.raises(ValueError, match="fixed 16777216-byte scratch"):
        N.check(st)
