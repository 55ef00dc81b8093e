"""Row/token sharding on the GPU: the kernels' shard parameters, emulated on
one device, and (with two or more GPUs visible) the ``sharded`` layers on real
NCCL ranks against the single-GPU result.

Sharded results follow the single-GPU rules: every row-local output (and the
cross-entropy VJP, whose scale is g / M_global on every rank) is bit-exact;
sums over rows that the shards regroup (weight gradients, the loss) are
compared at rtol 1e-5.
"""

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest

from parity import assert_bitexact, assert_close

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _dev(a, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _host(t):
    return t.detach().cpu().numpy()


def test_cross_entropy_row_shards_match_full():
    """Shards run with the global row count: the per-shard losses sum to the
    full loss and the per-shard VJPs are the full VJP's rows, bit for bit."""
    from oxitorch_b200 import functional as F
    from oxitorch_b200 import sharded as S
    rng = np.random.default_rng(21)
    m, c = 1037, 5003
    logits = (3 * rng.standard_normal((m, c))).astype(np.float32)
    targets = rng.integers(-c, c, m)
    g = _dev(np.array([0.75], np.float32))
    loss, rmax, rsum, _, t, _ = F.cross_entropy_fwd(_dev(logits), _dev(targets))
    full_d = _host(F.cross_entropy_bwd(_dev(logits), t, rmax, rsum, g))
    parts = []
    for r in range(3):
        lo, hi = S.shard_range(m, r, 3)
        sl, smax, ssum, _, st, _ = F.cross_entropy_fwd(_dev(logits[lo:hi]), _dev(targets[lo:hi]),
                                                       total_rows=m)
        parts.append(float(_host(sl)[0]))
        d = _host(F.cross_entropy_bwd(_dev(logits[lo:hi]), st, smax, ssum, g, total_rows=m))
        assert_bitexact(d, full_d[lo:hi], f"cross-entropy VJP rows of shard {r}")
    assert_close(np.array([sum(parts)]), _host(loss), rtol=1e-5, atol=0, what="sum of shard losses")


def test_sharded_layers_single_process():
    """Without a process group the sharded layers are the single-GPU layers."""
    import torch
    from oxitorch_b200 import functional as F
    from oxitorch_b200 import sharded as S
    from oxitorch_b200 import tensor_ops as T
    rng = np.random.default_rng(22)
    logits = _dev(rng.standard_normal((64, 300)).astype(np.float32))
    targets = [int(v) for v in rng.integers(0, 300, 64)]
    a = logits.clone().requires_grad_()
    b = logits.clone().requires_grad_()
    la, lb = S.cross_entropy(a, targets), F.cross_entropy(b, targets)
    la.backward()
    lb.backward()
    assert_bitexact(_host(la), _host(lb), "loss")
    assert_bitexact(_host(a.grad), _host(b.grad), "dlogits")
    table = _dev(rng.standard_normal((50, 16)).astype(np.float32))
    ids = [3, -1, 49, 3, 0]
    ta, tb = table.clone().requires_grad_(), table.clone().requires_grad_()
    oa, ob = S.embedding(ids, ta, 50), F.embedding(ids, tb)
    assert_bitexact(_host(oa), _host(ob), "lookup")
    dout = _dev(rng.standard_normal((5, 16)).astype(np.float32))
    oa.backward(dout)
    ob.backward(dout)
    assert_bitexact(_host(ta.grad), _host(tb.grad), "dtable")
    g1 = _dev(rng.standard_normal((33, 7)).astype(np.float32))
    g2 = g1.clone()
    n1 = S.clip_grad_norm_([g1], 0.5)
    n2 = T.clip_grad_norm_([g2], 0.5)
    assert n1 == n2
    assert_bitexact(_host(g1), _host(g2), "clipped gradient")
    with pytest.raises(ValueError):
        S.embedding(ids, table[:10], 50)


def _compact(ids_np, dout_np, vocab, shards):
    """oxc_embedding_bwd_compact on one device: (ids, rows, count, shard counts)."""
    import torch
    from oxitorch_b200 import _native as N
    from oxitorch_b200 import functional as F
    L = N.load()
    n, d = dout_np.shape
    ids, dout = _dev(ids_np), _dev(dout_np)
    cap = max(1, min(n, vocab))
    out_ids = torch.empty(cap, dtype=torch.int32, device="cuda")
    out_rows = torch.empty(cap, d, device="cuda")
    count = torch.empty(1, dtype=torch.int64, device="cuda")
    sc = torch.empty(shards, dtype=torch.int64, device="cuda")
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    ws = F._workspace(L.oxc_embedding_bwd_compact_workspace_size(n, vocab, d), dout.device)
    N.check(L.oxc_embedding_bwd_compact(dout.data_ptr(), ids.data_ptr(), n, vocab, 0, vocab, d,
                                        out_ids.data_ptr(), out_rows.data_ptr(), count.data_ptr(),
                                        shards, sc.data_ptr(), flag.data_ptr(), ws.data_ptr(),
                                        ws.numel(), F._stream()))
    k = int(count.item())
    return _host(out_ids)[:k], _host(out_rows)[:k], k, _host(sc)


def test_embedding_sparse_exchange_emulated(oracle):
    """The sparse gradient exchange of a replicated table, its G ranks emulated
    on one GPU: each token shard's compact VJP is the dense VJP's touched rows
    (bit-exact) with the right per-shard counts; the owner's
    oxc_embedding_exchange_reduce of the rows routed to it gives the whole
    batch's gradient rows -- bit-exact where one rank touched the row, within
    rtol 1e-4 (duplicate-id accumulation) elsewhere."""
    import torch
    from oxitorch_b200 import _native as N
    from oxitorch_b200 import functional as F
    from oxitorch_b200 import sharded as S
    rng = np.random.default_rng(24)
    V, D, n, G = 3000, 512, 20000, 4
    ids = np.minimum(rng.zipf(1.1, n) - 1, V - 1).astype(np.int64)
    ids[::97] -= V  # negative ids count from the end
    dout = rng.standard_normal((n, D)).astype(np.float32)
    res = np.where(ids < 0, ids + V, ids)
    bounds = [V * s // G for s in range(G + 1)]
    sends = []
    for g in range(G):
        lo, hi = S.shard_range(n, g, G)
        oid, orow, k, sc = _compact(ids[lo:hi], dout[lo:hi], V, G)
        u = np.unique(res[lo:hi])
        assert k == u.size and np.array_equal(oid, u)
        dense, _ = F.embedding_bwd(_dev(ids[lo:hi]), _dev(dout[lo:hi]), V)
        assert_bitexact(orow, _host(dense)[u], f"compact rows of rank {g}")
        assert list(sc) == [int(((u >= bounds[s]) & (u < bounds[s + 1])).sum()) for s in range(G)]
        sends.append((oid, orow, sc))
    full = oracle.scatter_index_select(dout, 0, [int(i) for i in res], (V, D))
    L = N.load()
    for s in range(G):
        rid, rrow, off = [], [], [0]
        for oid, orow, sc in sends:  # source order
            a = int(sc[:s].sum())
            rid.append(oid[a:a + sc[s]])
            rrow.append(orow[a:a + sc[s]])
            off.append(off[-1] + int(sc[s]))
        rid, rrow = np.concatenate(rid).astype(np.int32), np.concatenate(rrow)
        lo, rows = S.vocab_shard(V, s, G)
        dshard = torch.empty(rows, D, device="cuda")
        flag = torch.zeros(4, dtype=torch.int32, device="cuda")
        ws = F._workspace(L.oxc_embedding_exchange_reduce_workspace_size(G, rows), dshard.device)
        # device copies held in names: a temporary freed before the launch
        # could hand its memory to the next copy
        d_rid, d_rrow, d_off = _dev(rid), _dev(rrow), _dev(np.array(off, np.int64))
        N.check(L.oxc_embedding_exchange_reduce(
            d_rid.data_ptr(), d_rrow.data_ptr(), d_off.data_ptr(), G, lo, rows, D,
            dshard.data_ptr(), flag.data_ptr(), ws.data_ptr(), ws.numel(), F._stream()))
        got, want = _host(dshard), full[lo:lo + rows]
        touched_by = np.zeros(rows, np.int64)
        for g in range(G):
            glo, ghi = S.shard_range(n, g, G)
            u = np.unique(res[glo:ghi])
            u = u[(u >= lo) & (u < lo + rows)] - lo
            touched_by[u] += 1
        counts = np.bincount(res, minlength=V)[lo:lo + rows]
        exact = (touched_by <= 1) & (counts <= 128)
        assert_bitexact(got[exact], want[exact], f"shard {s} rows touched by one rank")
        scale = np.zeros((V, D))
        np.add.at(scale, res, np.abs(dout.astype(np.float64)))
        assert_close(got, want, rtol=1e-4, atol=1e-6 * np.maximum(scale[lo:lo + rows], 1.0),
                     what=f"shard {s}", strict_atol=1e-6 * np.maximum(scale[lo:lo + rows], 1.0))
        assert int(flag[0]) == 0


@pytest.mark.parametrize("mode", ["push", "pull"])
@pytest.mark.parametrize("cyclic", [False, True])
@pytest.mark.parametrize("d,G", [(512, 3), (37, 3), (512, 8)])
def test_embedding_push_exchange_emulated(d, G, cyclic, mode):
    """The fused exchange with three (or eight) ranks emulated on one GPU, every buffer in
    this GPU's memory, for contiguous and cyclic ownership and both forms:
    push (oxc_embedding_bwd_push into the owners' buffers, then each owner's
    oxc_embedding_exchange_reduce_regions) and pull (the push kernel into the
    sources' own buffers, then each owner's oxc_embedding_exchange_pull).  The
    regions hold each source's touched ids of that owner (ascending) and their
    counts, and every owner's dense shard is, bit for bit, the sum in source
    order from 0.0 of the sources' rows -- each source's rows being its
    single-GPU dense VJP's.  With contiguous ownership the shard is also the
    NCCL route's (compact VJP, rows routed in source order,
    oxc_embedding_exchange_reduce).  A vocabulary that does not split evenly
    and odd rows (d = 37, the scalar path) included; two rounds over the same
    regions, the second with other gradients."""
    import torch
    from oxitorch_b200 import _native as N
    from oxitorch_b200 import functional as F
    from oxitorch_b200 import sharded as S
    L = N.load()
    rng = np.random.default_rng(25)
    V, n = 3001, 20000
    ids = np.minimum(rng.zipf(1.1, n) - 1, V - 1).astype(np.int64)
    ids[::89] -= V  # negative ids count from the end
    res = np.where(ids < 0, ids + V, ids)
    bounds = [V * p // G for p in range(G + 1)]
    cap = -(-V // G)

    def owned(p):  # table rows of owner p, ascending
        return np.arange(p, V, G) if cyclic else np.arange(bounds[p], bounds[p + 1])

    # buffer h holds G regions; region (owner, source) is at index source of
    # the owner's buffer (push) or index owner of the source's buffer (pull)
    brows = [torch.empty(G * cap * d, device="cuda") for _ in range(G)]
    bids = [torch.full((G * cap,), -7, dtype=torch.int32, device="cuda") for _ in range(G)]
    bcount = [torch.full((G,), -1, dtype=torch.int64, device="cuda") for _ in range(G)]

    def region(owner, source):
        h, i = (owner, source) if mode == "push" else (source, owner)
        return (brows[h].data_ptr() + i * cap * d * 4, bids[h].data_ptr() + i * cap * 4,
                bcount[h].data_ptr() + i * 8, h, i)

    def to_dev(tab):
        return torch.tensor(list(bytes(tab)), dtype=torch.uint8).to("cuda")

    tabs, pulls = [], []
    for g in range(G):
        tab = N.EmbPush()
        tab.world, tab.source, tab.cyclic, tab.local, tab.cap = G, g, int(cyclic), \
            int(mode == "pull"), cap
        for p in range(G + 1):
            tab.lo[p] = bounds[p]
        for p in range(G):
            tab.rows[p], tab.ids[p], tab.count[p] = region(p, g)[:3]
        tabs.append(to_dev(tab))
    for p in range(G):
        pt = N.EmbPull()
        for g in range(G):
            pt.rows[g], pt.ids[g], pt.count[g] = region(p, g)[:3]
        pulls.append(to_dev(pt))
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    ws_bytes = L.oxc_embedding_bwd_compact_workspace_size(n, V, d)
    ws = F._workspace(ws_bytes, torch.device("cuda"))
    shards = [S.shard_range(n, g, G) for g in range(G)]
    for rnd in range(2):
        dout = (rng.standard_normal((n, d)) * (rnd + 1)).astype(np.float32)
        d_in = [(_dev(ids[lo:hi]), _dev(dout[lo:hi])) for lo, hi in shards]
        for g, (lo, hi) in enumerate(shards):
            N.check(L.oxc_embedding_bwd_push(
                d_in[g][1].data_ptr(), d_in[g][0].data_ptr(), hi - lo, V, d, tabs[g].data_ptr(),
                flag.data_ptr(), ws.data_ptr(), ws_bytes, F._stream()), "push")
        # the expected sums: every source's dense VJP rows, added in source order from 0.0
        expect = np.zeros((V, d), np.float32)
        touched = []
        for g, (lo, hi) in enumerate(shards):
            dense, _ = F.embedding_bwd(d_in[g][0], d_in[g][1], V)
            u = np.unique(res[lo:hi])
            touched.append(u)
            expect[u] = expect[u] + _host(dense)[u]
        for p in range(G):
            rows_p = owned(p)
            for g in range(G):
                h, i = region(p, g)[3:]
                u = np.intersect1d(touched[g], rows_p)
                assert int(_host(bcount[h])[i]) == u.size, (p, g)
                assert np.array_equal(_host(bids[h]).reshape(G, cap)[i, :u.size], u), (p, g)
            lo_p, stride = (p, G) if cyclic else (bounds[p], 1)
            ws2 = F._workspace(L.oxc_embedding_exchange_reduce_workspace_size(G, rows_p.size),
                               torch.device("cuda"))
            got = torch.empty(rows_p.size, d, device="cuda")
            if mode == "push":
                N.check(L.oxc_embedding_exchange_reduce_regions(
                    bids[p].data_ptr(), brows[p].data_ptr(), bcount[p].data_ptr(), G, cap, lo_p,
                    stride, rows_p.size, d, got.data_ptr(), flag.data_ptr(), ws2.data_ptr(),
                    ws2.numel(), F._stream()), "reduce regions")
            else:
                N.check(L.oxc_embedding_exchange_pull(
                    pulls[p].data_ptr(), G, cap, lo_p, stride, rows_p.size, d, got.data_ptr(),
                    flag.data_ptr(), ws2.data_ptr(), ws2.numel(), F._stream()), "pull")
            assert_bitexact(_host(got), expect[rows_p], f"owner {p} shard, round {rnd}")
            if not cyclic:
                # the NCCL route's owner reduce over the same rows in source order
                sends = [_compact(ids[lo:hi], dout[lo:hi], V, G) for lo, hi in shards]
                rid, rrow, off = [], [], [0]
                for oid, orow, k, sc in sends:
                    a = int(sc[:p].sum())
                    rid.append(oid[a:a + sc[p]])
                    rrow.append(orow[a:a + sc[p]])
                    off.append(off[-1] + int(sc[p]))
                d_rid = _dev(np.concatenate(rid).astype(np.int32))
                d_rrow = _dev(np.concatenate(rrow))
                d_off = _dev(np.array(off, np.int64))
                want = torch.empty(rows_p.size, d, device="cuda")
                N.check(L.oxc_embedding_exchange_reduce(
                    d_rid.data_ptr(), d_rrow.data_ptr(), d_off.data_ptr(), G, bounds[p],
                    rows_p.size, d, want.data_ptr(), flag.data_ptr(), ws2.data_ptr(),
                    ws2.numel(), F._stream()))
                assert_bitexact(_host(got), _host(want), f"owner {p} vs the NCCL route")
        assert int(flag.abs().sum().item()) == 0


# ---- real NCCL ranks ---------------------------------------------------------------------

def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    try:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        try:
            _nccl_body(rank, world, dev)
            torch.cuda.synchronize()
            dist.barrier()
            q.put(("ok", rank, ""))
        finally:
            dist.destroy_process_group()
    except BaseException:
        q.put(("fail", rank, traceback.format_exc()))


def _nccl_body(rank, world, dev):
    import torch
    import torch.distributed as dist
    from oxitorch_b200 import functional as F
    from oxitorch_b200 import sharded as S
    rng = np.random.default_rng(23)  # the same data on every rank
    # LayerNorm+GELU: row shards + weight-gradient sync
    m, c = 4099, 1024
    x = rng.standard_normal((m, c)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, c).astype(np.float32)
    b = (0.1 * rng.standard_normal(c)).astype(np.float32)
    dy = rng.standard_normal((m, c)).astype(np.float32)
    lo, hi = S.shard_range(m, rank, world)
    wf, bf = _dev(w, dev).requires_grad_(), _dev(b, dev).requires_grad_()
    F.layer_norm_gelu(_dev(x, dev), wf, bf).backward(_dev(dy, dev))
    ws, bs = _dev(w, dev).requires_grad_(), _dev(b, dev).requires_grad_()
    xs = _dev(x[lo:hi], dev).requires_grad_()
    ys = F.layer_norm_gelu(xs, ws, bs)
    ys.backward(_dev(dy[lo:hi], dev))
    S.sync_grads_([ws, bs])
    yf = F.layer_norm_gelu(_dev(x, dev), wf.detach(), bf.detach())
    assert_bitexact(_host(ys), _host(yf)[lo:hi], "layer_norm_gelu rows")
    assert_close(_host(ws.grad), _host(wf.grad), rtol=1e-5, atol=1e-4, what="synced dweight")
    assert_close(_host(bs.grad), _host(bf.grad), rtol=1e-5, atol=1e-4, what="synced dbias")
    # cross-entropy: the global mean on every rank, VJP rows bit-exact
    m, c = 2053, 3001
    logits = (2 * rng.standard_normal((m, c))).astype(np.float32)
    targets = rng.integers(0, c, m)
    lo, hi = S.shard_range(m, rank, world)
    full = _dev(logits, dev).requires_grad_()
    lf = F.cross_entropy(full, [int(t) for t in targets])
    lf.backward()
    part = _dev(logits[lo:hi], dev).requires_grad_()
    ls = S.cross_entropy(part, [int(t) for t in targets[lo:hi]])
    ls.backward()
    assert_close(_host(ls).reshape(1), _host(lf).reshape(1), rtol=1e-5, atol=0, what="global loss")
    assert_bitexact(_host(part.grad), _host(full.grad)[lo:hi], "cross-entropy VJP rows")
    # vocab-sharded embedding: the lookup is exact on every rank; each rank's
    # dtable is its rows of the full dtable (ids here occur <= 128 times)
    v, d = 1000, 256
    table = rng.standard_normal((v, d)).astype(np.float32)
    ids = [int(i) for i in rng.integers(-v, v, 3000)]
    dout = rng.standard_normal((len(ids), d)).astype(np.float32)
    off, rows = S.vocab_shard(v, rank, world)
    shard = _dev(table[off:off + rows], dev).requires_grad_()
    out = S.embedding(ids, shard, v)
    tf = _dev(table, dev).requires_grad_()
    of = F.embedding(ids, tf)
    assert_bitexact(_host(out), _host(of), "vocab-sharded lookup")
    out.backward(_dev(dout, dev))
    of.backward(_dev(dout, dev))
    assert_bitexact(_host(shard.grad), _host(tf.grad)[off:off + rows], "dtable shard")
    # reduce-scatter of a replicated table's gradient: this rank's rows of the sum
    parts_t = [(_dev(np.arange(1000 * 16, dtype=np.float32).reshape(1000, 16), dev) * (r + 1))
               for r in range(world)]
    mine = S.reduce_scatter_rows(parts_t[rank].clone())
    lo_t, hi_t = S.shard_range(1000, rank, world)
    assert_bitexact(_host(mine), _host(sum(parts_t))[lo_t:hi_t], "reduce-scattered rows")
    # sparse exchange of a replicated table's gradient (token-sharded ids):
    # this rank's vocab rows of the whole batch's gradient
    v2, d2, n2 = 2000, 256, 12000
    ids2 = np.minimum(rng.zipf(1.1, n2) - 1, v2 - 1).astype(np.int64)
    dout2 = rng.standard_normal((n2, d2)).astype(np.float32)
    lo2, hi2 = S.shard_range(n2, rank, world)
    dsh = S.embedding_grad(_dev(ids2[lo2:hi2], dev), _dev(dout2[lo2:hi2], dev), v2)
    full2, _ = F.embedding_bwd(_dev(ids2, dev), _dev(dout2, dev), v2)
    voff, vrows = S.vocab_shard(v2, rank, world)
    assert_close(_host(dsh), _host(full2)[voff:voff + vrows], rtol=1e-4, atol=1e-4,
                 what="sparse-exchanged dtable shard")
    # the fused exchange over peer memory: the same sums in the same order as
    # the NCCL all-to-all exchange, so bit for bit the same rows, over three
    # steps that alternate the two slots; contiguous ownership gives the NCCL
    # route's shard, cyclic ownership its rows rank, rank + world, ...
    ids_r = _dev(ids2[lo2:hi2], dev)
    for mode, cyclic in (("push", False), ("push", True), ("pull", False), ("pull", True)):
        ex = S.PeerGradExchange(hi2 - lo2, v2, d2, dev, slots=2, cyclic=cyclic, mode=mode)
        for step in range(3):
            dout_k = _dev(dout2[lo2:hi2] * np.float32(step + 1), dev)
            ex.vjp(ids_r, dout_k, step % 2)
            got, done = ex.exchange(step % 2)
            torch.cuda.current_stream().wait_event(done)
            want_k = S.embedding_grad(ids_r, dout_k, v2)
            if cyclic:
                parts = [torch.empty(S.vocab_shard(v2, p, world)[1], d2, device=dev)
                         for p in range(world)]
                dist.all_gather(parts, want_k)
                want_k = torch.cat(parts)[rank::world]
            assert_bitexact(_host(got), _host(want_k),
                            f"peer-exchanged dtable shard ({mode}, cyclic={cyclic}), step {step}")
        assert int(ex.flag.abs().sum().item()) == 0
        ex.close()
    # the C-ABI communicator (oxc_comm_*), the route of a native host
    import ctypes
    from oxitorch_b200 import _native as N
    L = N.load()
    idbuf = (ctypes.c_uint8 * 128)()
    if rank == 0:
        N.check(L.oxc_comm_unique_id(idbuf))
    obj = [bytes(idbuf)]
    dist.broadcast_object_list(obj, src=0)
    idbuf = (ctypes.c_uint8 * 128).from_buffer_copy(obj[0])
    comm = ctypes.c_void_p()
    N.check(L.oxc_comm_init(ctypes.byref(comm), idbuf, world, rank))
    s_ = torch.cuda.current_stream().cuda_stream
    a = _dev(np.arange(4099, dtype=np.float32) * (rank + 1), dev)
    b = a.clone()
    N.check(L.oxc_comm_allreduce_sum_f32(comm, a.data_ptr(), a.numel(), s_))
    dist.all_reduce(b)
    assert_bitexact(_host(a), _host(b), "oxc_comm_allreduce_sum_f32")
    d64 = torch.full((7,), float(rank + 1), dtype=torch.float64, device=dev)
    N.check(L.oxc_comm_allreduce_sum_f64(comm, d64.data_ptr(), 7, s_))
    assert float(d64[0]) == world * (world + 1) / 2
    rs_in = _dev(np.arange(world * 33, dtype=np.float32), dev)
    rs_out = torch.empty(33, device=dev)
    N.check(L.oxc_comm_reduce_scatter_f32(comm, rs_in.data_ptr(), rs_out.data_ptr(), 33, s_))
    assert_bitexact(_host(rs_out), world * np.arange(rank * 33, rank * 33 + 33, dtype=np.float32),
                    "oxc_comm_reduce_scatter_f32")
    # all-to-all: rank r sends r + p + 1 int32 values (all = 100 r + p) to rank p
    sc = [rank + p + 1 for p in range(world)]
    rc = [p + rank + 1 for p in range(world)]
    send = _dev(np.concatenate([np.full(c, 100 * rank + p, np.int32) for p, c in enumerate(sc)]), dev)
    recv = torch.empty(sum(rc), dtype=torch.int32, device=dev)
    N.check(L.oxc_comm_alltoallv(comm, send.data_ptr(), (ctypes.c_int64 * world)(*sc),
                                 recv.data_ptr(), (ctypes.c_int64 * world)(*rc), 4, s_))
    want = np.concatenate([np.full(c, 100 * p + rank, np.int32) for p, c in enumerate(rc)])
    assert np.array_equal(_host(recv), want)
    torch.cuda.synchronize()
    N.check(L.oxc_comm_destroy(comm))
    # global sum of squares over row shards
    gsh = _dev(x[lo % 100:lo % 100 + 50], dev)
    tot = S.sum_squares([gsh])
    parts = [None] * world
    dist.all_gather_object(parts, float(np.sum(x[lo % 100:lo % 100 + 50].astype(np.float64) ** 2)))
    assert_close(np.array([tot.item()]), np.array([sum(parts)]), rtol=1e-9, atol=0,
                 what="global sum of squares")


def test_nccl_two_ranks():
    import torch
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    try:
        for _ in procs:
            out.append(q.get(timeout=300))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    fails = [o for o in out if o[0] != "ok"]
    assert not fails, "\n".join(f"rank {o[1]}:\n{o[2]}" for o in fails)
