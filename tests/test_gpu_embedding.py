"""Embedding gather (bit-exact) and its duplicate-id VJP vs the oracle.

Rows of dtable whose id occurs at most 128 times are the reference's
left-to-right position-order sum and must match bit for bit; hotter rows are
summed in 128-occurrence pieces (rtol 1e-4 plus the reference's own
summation-order error, tests/parity.py)."""

import json
import os

import numpy as np
import pytest

from parity import ATOL, RTOL_BIG, assert_bitexact, assert_close

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    return t.detach().cpu().numpy()


def _oracle_dtable(oracle, dout, ids, rows, precise=False):
    cols = dout.shape[1]
    r = np.where(ids < 0, ids + rows, ids)
    if not precise:
        return oracle.scatter_index_select(dout, 0, r, (rows, cols))
    out = np.zeros((rows, cols), np.float64)
    np.add.at(out, r, dout.astype(np.float64))
    return out.astype(np.float32)


def _check_dtable(oracle, got, dout, ids, rows):
    want = _oracle_dtable(oracle, dout, ids, rows)
    counts = np.bincount(np.where(ids < 0, ids + rows, ids), minlength=rows)
    cold = counts <= 128
    assert_bitexact(got[cold], want[cold], "dtable rows with <= 128 occurrences")
    if (~cold).any():
        exact = _oracle_dtable(oracle, dout, ids, rows, precise=True)
        budget = np.abs(want.astype(np.float64) - exact)
        scale = np.zeros((rows, dout.shape[1]))
        np.add.at(scale, np.where(ids < 0, ids + rows, ids), np.abs(dout.astype(np.float64)))
        assert_close(got[~cold], want[~cold], rtol=RTOL_BIG,
                     atol=ATOL * np.maximum(scale[~cold], 1.0) + budget[~cold],
                     what="dtable hot rows", strict_atol=ATOL * np.maximum(scale[~cold], 1.0))


def _run(table, ids, dout):
    from oxitorch_b200 import functional as F
    dids = _dev(np.asarray(ids, np.int64))
    out, f1 = F.embedding_fwd(dids, _dev(table))
    dtable, f2 = F.embedding_bwd(dids, _dev(dout), table.shape[0])
    assert int(f1.cpu()[0]) == 0 and int(f2.cpu()[0]) == 0
    return _host(out), _host(dtable)


@pytest.mark.parametrize("name", ["emb_300x32_n1500", "emb_40x6_n50"])
def test_embedding_golden(oracle, golden, name):
    g = {k.split(".", 1)[1]: v for k, v in golden.items() if k.startswith(name + ".")}
    out, dtable = _run(g["table"], g["ids"], g["dout"])
    assert_bitexact(out, g["out"], "out")
    _check_dtable(oracle, dtable, g["dout"], g["ids"], g["table"].shape[0])


def test_embedding_reference_known_answers():
    kats = json.load(open(os.path.join(HERE, "golden", "reference_kats.json")))["embedding_grad"]
    for case in kats:
        table = np.asarray(case["table"], np.float32).reshape(case["table_shape"])
        n, d = len(case["ids"]), table.shape[1]
        seed = (np.ones((n, d), np.float32) if case["seed"] == "ones"
                else np.asarray(case["seed"], np.float32).reshape(n, d))
        out, dtable = _run(table, case["ids"], seed)
        if "want_out" in case:
            np.testing.assert_array_equal(out.reshape(-1), case["want_out"], err_msg=case["src"])
        np.testing.assert_array_equal(dtable.reshape(-1), case["want_grad"], err_msg=case["src"])


@pytest.mark.parametrize("v,d,n", [(1000, 4096, 20000), (97, 33, 5000), (5, 4, 3), (300, 128, 1)])
def test_embedding_vs_oracle(oracle, v, d, n):
    rng = np.random.default_rng(v + d + n)
    table = rng.standard_normal((v, d), dtype=np.float32)
    ids = np.minimum(rng.zipf(1.1, n) - 1, v - 1).astype(np.int64)
    ids[rng.random(n) < 0.05] -= v  # some negative ids (count from the end)
    dout = rng.standard_normal((n, d), dtype=np.float32)
    out, dtable = _run(table, ids, dout)
    assert_bitexact(out, oracle.t_index_select(table, 0, ids), "out")
    _check_dtable(oracle, dtable, dout, ids, v)


def test_embedding_config4_full_size(oracle):
    """table [32000, 4096] ~ N(0,1); ids [64, 2048] =
    min(zipf(1.1) - 1, 31999) (id 31999 occurs ~43k times); dout N(0,1)."""
    import bench
    v, d = 32000, 4096
    inp = bench.config_inputs(4)  # the arrays the benchmark times
    table, ids, dout = inp["table"], inp["ids"], inp["dout"]
    rng = np.random.default_rng(4)
    counts = np.bincount(ids, minlength=v)
    assert counts.max() > 40000  # the clip mass on the last id
    out, dtable = _run(table, ids, dout)
    sample = rng.choice(ids.size, 2048, replace=False)
    assert_bitexact(out[sample], table[ids[sample]], "out rows")
    _check_dtable(oracle, dtable, dout, ids, v)


def test_embedding_errors_and_autograd():
    import torch
    from oxitorch_b200 import functional as F
    w = torch.zeros(3, 2, device="cuda", requires_grad=True)
    with pytest.raises(RuntimeError, match="index 3 out of range for dim 0 of size 3"):
        F.embedding([0, 3], w)
    out = F.embedding([2, 0, 2], torch.tensor([[1.0, 1], [2, 2], [3, 3]], device="cuda",
                                              requires_grad=True))
    np.testing.assert_array_equal(_host(out), [[3, 3], [1, 1], [3, 3]])
    ww = torch.tensor([[1.0, 1], [2, 2], [3, 3]], device="cuda", requires_grad=True)
    F.embedding([2, 0, 2], ww).sum().backward()
    np.testing.assert_array_equal(_host(ww.grad), [[1, 1], [0, 0], [2, 2]])


def test_embedding_sharded_matches_full(oracle):
    """Vocab-parallel shards: each shard's forward is the full forward masked
    to its rows; shard outputs sum to the full output; shard gradients are the
    reference gradient's rows (hot rows are cut into pieces at positions that
    depend on the shard, so they follow the hot-row tolerance)."""
    from oxitorch_b200 import functional as F
    rng = np.random.default_rng(8)
    v, d, n = 1000, 256, 4000
    table = rng.standard_normal((v, d), dtype=np.float32)
    ids = np.minimum(rng.zipf(1.2, n) - 1, v - 1).astype(np.int64)
    dout = rng.standard_normal((n, d), dtype=np.float32)
    full_out, full_dt = _run(table, ids, dout)
    dids = _dev(ids)
    acc = np.zeros_like(full_out)
    for lo, hi in [(0, 250), (250, 600), (600, 1000)]:
        out, _ = F.embedding_fwd(dids, _dev(table[lo:hi]), vocab_offset=lo, vocab_total=v)
        acc += _host(out)
        dt, _ = F.embedding_bwd(dids, _dev(dout), hi - lo, vocab_offset=lo, vocab_total=v)
        mine = (ids >= lo) & (ids < hi)
        _check_dtable(oracle, _host(dt), dout[mine], ids[mine] - lo, hi - lo)
    assert_bitexact(acc, full_out, "sum of shard outputs")
