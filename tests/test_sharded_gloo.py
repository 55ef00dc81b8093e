"""Multi-rank host logic of ``oxitorch_b200.sharded`` on CPU: world_size 2
(and 3, for ragged shards) over gloo.

What crosses ranks on the layer path is small partials (weight gradients,
the cross-entropy loss and row count, f64 sums of squares) and, for a
vocab-sharded table, the gathered rows summed with zeros.  Each rank here
computes its shard's partials with the CPU oracle (the reference's composed
graph) and combines them with the module's own collectives; the result must
match the oracle run on the whole batch.  The CUDA kernels that make the
partials on a GPU box are covered by the ``-m gpu`` tests.
"""

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, fn):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    try:
        for _ in procs:
            out.append(q.get(timeout=180))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    fails = [o for o in out if o[0] != "ok"]
    assert not fails, "\n".join(f"rank {o[1]}:\n{o[2]}" for o in fails)
    return sorted(out, key=lambda o: o[1])


def _worker(rank, world, port, fn, q):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=60))
        try:
            res = globals()[fn](rank, world)
            q.put(("ok", rank, res))
        finally:
            dist.destroy_process_group()
    except BaseException:
        q.put(("fail", rank, traceback.format_exc()))


# ---- rank bodies (module-level so spawn can find them) -------------------------------------

def _geometry(rank, world):
    from oxitorch_b200 import sharded as S
    import torch.distributed as dist
    for n in (0, 1, 2, 5, 7, 4096, 32000):
        lo, hi = S.shard_range(n, rank, world)
        got = [None] * world
        dist.all_gather_object(got, (lo, hi))
        # contiguous, covering, balanced
        assert got[0][0] == 0 and got[-1][1] == n
        assert all(got[i][1] == got[i + 1][0] for i in range(world - 1))
        sizes = [b - a for a, b in got]
        assert max(sizes) - min(sizes) <= 1
    off, rows = S.vocab_shard(32000, rank, world)
    assert (off, off + rows) == S.shard_range(32000, rank, world)
    x = torch.arange(10 * 3, dtype=torch.float32).reshape(10, 3)
    loc = S.local_rows(x)
    lo, hi = S.shard_range(10, rank, world)
    assert torch.equal(loc, x[lo:hi])
    assert S.global_count(hi - lo, "cpu") == 10
    return None


def _collectives(rank, world):
    from oxitorch_b200 import sharded as S
    a = torch.full((4,), float(rank + 1))
    b = torch.arange(3, dtype=torch.float64) * (rank + 1)
    S.allreduce_sum_(a, b)
    tot = world * (world + 1) / 2
    assert torch.equal(a, torch.full((4,), tot))
    assert torch.equal(b, torch.arange(3, dtype=torch.float64) * tot)
    # sync_grads_: parameters without a gradient are skipped on every rank
    p1 = torch.zeros(5, requires_grad=True)
    p2 = torch.zeros(2, requires_grad=True)
    p1.grad = torch.full((5,), float(rank))
    S.sync_grads_([p1, p2])
    assert p2.grad is None
    assert torch.equal(p1.grad, torch.full((5,), float(sum(range(world)))))
    return None


def _reduce_scatter_rows(rank, world):
    """Each rank keeps its row shard of the sum over ranks (on gloo: the
    all-reduce-and-slice path; 7 rows do not split evenly over 2 or 3)."""
    from oxitorch_b200 import sharded as S
    full = [torch.arange(7 * 3, dtype=torch.float32).reshape(7, 3) * (r + 1) for r in range(world)]
    got = S.reduce_scatter_rows(full[rank].clone())
    lo, hi = S.shard_range(7, rank, world)
    want = sum(full)[lo:hi]
    assert torch.equal(got, want)
    return None


def _layer_norm_grads(rank, world):
    """LayerNorm+GELU weight gradients: per-shard VJP partials summed over the
    ranks equal the whole-batch VJP."""
    from oracle import oxiref as O
    from oxitorch_b200 import sharded as S
    rng = np.random.default_rng(11)
    M, C = 13, 24
    x = rng.standard_normal((M, C)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, C).astype(np.float32)
    b = (0.1 * rng.standard_normal(C)).astype(np.float32)
    dy = rng.standard_normal((M, C)).astype(np.float32)

    def grads(rows):
        xt = O.from_numpy(x[rows], True)
        wt, bt = O.from_numpy(w, True), O.from_numpy(b, True)
        y = O.gelu(O.layer_norm(xt, wt, bt, 1e-5))
        y.backward(dy[rows])
        return wt.grad.numpy(), bt.grad.numpy()

    lo, hi = S.shard_range(M, rank, world)
    dw, db = (torch.from_numpy(g.copy()) for g in grads(slice(lo, hi)))
    S.allreduce_sum_(dw, db)
    fw, fb = grads(slice(0, M))
    # the row sums are regrouped (per shard, then across shards)
    for got, want in ((dw.numpy(), fw), (db.numpy(), fb)):
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
    return None


def _cross_entropy_mean(rank, world):
    """Global-mean cross-entropy: the global row count is agreed first; each
    rank's partial is its rows' nll sum divided by that count; the partials
    sum to the whole-batch mean."""
    from oracle import oxiref as O
    from oxitorch_b200 import sharded as S
    rng = np.random.default_rng(12)
    M, C = 11, 17
    logits = (2 * rng.standard_normal((M, C))).astype(np.float32)
    targets = rng.integers(-C, C, M)  # negative targets wrap (numpy one-hot)
    lo, hi = S.shard_range(M, rank, world)
    m = S.global_count(hi - lo, "cpu")
    assert m == M
    if hi > lo:
        local_mean = float(O.cross_entropy(O.from_numpy(logits[lo:hi]),
                                           [int(t) for t in targets[lo:hi]]).numpy())
        part = local_mean * (hi - lo) / m
    else:
        part = 0.0
    loss = torch.tensor([part], dtype=torch.float64)
    S.allreduce_sum_(loss)
    full = float(O.cross_entropy(O.from_numpy(logits), [int(t) for t in targets]).numpy())
    np.testing.assert_allclose(loss.item(), full, rtol=1e-5)
    return None


def _embedding_vocab_sharded(rank, world):
    """Vocab-sharded lookup: each rank fills the rows its shard owns and zeros
    elsewhere; the summed outputs equal the whole-table lookup bit for bit."""
    from oracle import oxiref as O
    from oxitorch_b200 import sharded as S
    rng = np.random.default_rng(13)
    V, D = 10, 6
    table = rng.standard_normal((V, D)).astype(np.float32)
    ids = [0, 3, -1, 9, 3, 3, -10, 5, 4]  # negatives count from the end
    off, rows = S.vocab_shard(V, rank, world)
    out = np.zeros((len(ids), D), dtype=np.float32)
    for k, i in enumerate(ids):
        r = i + V if i < 0 else i
        if off <= r < off + rows:
            out[k] = table[r]
    t = torch.from_numpy(out)
    S.allreduce_sum_(t)
    want = O.embedding(ids, O.from_numpy(table)).numpy()
    assert np.array_equal(t.numpy(), want)
    return None


def _embedding_sparse_exchange(rank, world):
    """The sparse exchange of a replicated table's gradient (token-sharded
    ids): each rank keeps the touched rows of its tokens' VJP (the oracle's
    position-order sums), sends each to its vocab shard's owner with
    S.exchange_rows, and the owner sums what arrives in rank order (what
    oxc_embedding_exchange_reduce does on a GPU).  Rows touched by one rank
    equal the whole batch's VJP bit for bit; the rest within rtol 1e-4."""
    from oracle import oxiref as O
    from oxitorch_b200 import sharded as S
    rng = np.random.default_rng(15)
    V, D, n = 23, 5, 60
    ids = np.minimum(rng.zipf(1.3, n) - 1, V - 1).astype(np.int64)
    dout = rng.standard_normal((n, D)).astype(np.float32)
    lo, hi = S.shard_range(n, rank, world)
    local = O.scatter_index_select(dout[lo:hi], 0, [int(i) for i in ids[lo:hi]], (V, D))
    touched = np.unique(ids[lo:hi]).astype(np.int32)  # ascending: the compact order
    bounds = [V * s // world for s in range(world + 1)]
    counts = torch.tensor([int(((touched >= bounds[s]) & (touched < bounds[s + 1])).sum())
                           for s in range(world)])
    rid, rrows, rc = S.exchange_rows(torch.from_numpy(touched), torch.from_numpy(local[touched]),
                                     counts)
    assert sum(rc) == rid.numel() == rrows.shape[0]
    own_lo, own_rows = S.vocab_shard(V, rank, world)
    got = np.zeros((own_rows, D), np.float32)
    src = np.repeat(np.arange(world), rc)
    for s in range(world):  # rank order
        for i in np.nonzero(src == s)[0]:
            v = int(rid[i]) - own_lo
            assert 0 <= v < own_rows
            got[v] = got[v] + rrows[i].numpy()
    full = O.scatter_index_select(dout, 0, [int(i) for i in ids], (V, D))[own_lo:own_lo + own_rows]
    owners = [set(ids[S.shard_range(n, r, world)[0]:S.shard_range(n, r, world)[1]]) for r in range(world)]
    single = np.array([sum((own_lo + v) in o for o in owners) <= 1 for v in range(own_rows)])
    assert np.array_equal(got[single], full[single])
    np.testing.assert_allclose(got, full, rtol=1e-4, atol=1e-6)
    return None


def _sum_squares(rank, world):
    """Whole-tensor sum of squares over row shards: f64 partials, summed."""
    from oxitorch_b200 import sharded as S
    rng = np.random.default_rng(14)
    g = rng.standard_normal((37, 19)).astype(np.float32)
    lo, hi = S.shard_range(37, rank, world)
    part = torch.tensor(float(np.sum(g[lo:hi].astype(np.float64) ** 2)), dtype=torch.float64)
    S.allreduce_sum_(part)
    np.testing.assert_allclose(part.item(), np.sum(g.astype(np.float64) ** 2), rtol=1e-13)
    return None


def _rank_error_surfaces(rank, world):
    """Bad shard arguments raise ValueError on the host of the rank that
    passed them, before any collective."""
    from oxitorch_b200 import sharded as S
    with pytest.raises(ValueError):
        S.shard_range(4, world, world)
    with pytest.raises(ValueError):
        S.shard_range(-1, 0, world)
    return None


@pytest.mark.parametrize("world", [2, 3])
def test_shard_geometry(world):
    _run(world, "_geometry")


def test_collectives():
    _run(2, "_collectives")


@pytest.mark.parametrize("world", [2, 3])
def test_reduce_scatter_rows(world):
    _run(world, "_reduce_scatter_rows")


@pytest.mark.parametrize("world", [2, 3])
def test_layer_norm_weight_grads_sum_over_ranks(world):
    _run(world, "_layer_norm_grads")


@pytest.mark.parametrize("world", [2, 3])
def test_cross_entropy_global_mean(world):
    _run(world, "_cross_entropy_mean")


@pytest.mark.parametrize("world", [2, 3])
def test_embedding_vocab_shards_sum_exact(world):
    _run(world, "_embedding_vocab_sharded")


@pytest.mark.parametrize("world", [2, 3])
def test_embedding_sparse_gradient_exchange(world):
    _run(world, "_embedding_sparse_exchange")


def test_sum_squares_over_shards():
    _run(2, "_sum_squares")


def test_argument_errors():
    _run(2, "_rank_error_surfaces")


def test_single_process_is_a_no_op():
    """Without an initialised process group every collective is a no-op and
    the shard is the whole tensor."""
    from oxitorch_b200 import sharded as S
    t = torch.ones(3)
    S.allreduce_sum_(t)
    assert torch.equal(t, torch.ones(3))
    assert S.global_count(7, "cpu") == 7
    x = torch.zeros(5, 2)
    assert S.local_rows(x).shape == (5, 2)
