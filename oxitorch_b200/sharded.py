"""Row/token-sharded data parallelism for the layer path: one process per GPU.

Every layer on the path is row-local (a row is a token: one norm row, one
softmax row, one logits row, one embedding lookup), so G ranks split the rows
and run the single-GPU kernels on their slice with no exchange on the data
path.  What crosses ranks is small:

* weight gradients of the norms (dweight / dbias, [cols]) and of a replicated
  embedding table: each rank's VJP leaves the sum over its own rows, and one
  all-reduce (sum) makes it the sum over every row -- ``allreduce_sum_``; a
  large table's gradient can instead be reduce-scattered so each rank keeps
  the summed rows of its own shard -- ``reduce_scatter_rows``;
* the cross-entropy mean: the global row count M is agreed before the forward
  (one int64 all-reduce), each rank's loss kernel divides its partial sum by
  that M, and the partials are summed -- ``cross_entropy``; the VJP scale
  g / M needs no exchange;
* whole-tensor sums and sums of squares (``clip_grad_norm_`` over sharded
  activation gradients): f64 partials, summed -- ``sum_squares``;
* a vocab-sharded embedding table: every rank gathers the rows its shard owns
  (zeros for the other ids) and the outputs are summed -- ``embedding``; each
  rank's VJP writes its own dtable rows with no exchange;
* a replicated embedding table with token-sharded ids: each rank's VJP keeps
  only the rows its tokens touch (``oxc_embedding_bwd_compact``), an
  all-to-all sends every row to the rank owning its vocab shard, and the owner
  sums what arrives in rank order -- ``embedding_grad``.  Only the touched rows
  cross the links (Zipf(1.1) ids over 131072 tokens touch about 11.5k of 32000
  rows), against the whole table for a dense reduce-scatter.

The reference has no distributed runtime (its plan lists a gloo-like backend
as a stretch goal, plan.md:325); this module is this package's own design for
the multi-GPU rows.  ``torch.distributed`` is the transport: NCCL over
NVLink/NVSwitch between GPUs, and the same calls run on gloo, which is how the
host logic is tested without GPUs.  Every rank issues the same collectives in
the same order.  A process group that is not initialised, or has one rank,
turns every collective into a no-op, so the functions below are also the
single-GPU path.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import functional as F
from . import tensor_ops as T


def _world(group=None) -> int:
    if not (dist.is_available() and dist.is_initialized()):
        return 1
    return dist.get_world_size(group)


def _rank(group=None) -> int:
    if not (dist.is_available() and dist.is_initialized()):
        return 0
    return dist.get_rank(group)


# ---- shard geometry ---------------------------------------------------------------------

def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous balanced split of n rows: rank r owns [n*r//G, n*(r+1)//G).
    Shard sizes differ by at most one row and concatenate to [0, n)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"invalid argument: rank {rank} of world {world}")
    if n < 0:
        raise ValueError(f"invalid argument: {n} rows")
    return n * rank // world, n * (rank + 1) // world


def vocab_shard(vocab: int, rank: int, world: int) -> tuple[int, int]:
    """(vocab_offset, rows) of rank r's slice of a vocab-sharded table."""
    lo, hi = shard_range(vocab, rank, world)
    return lo, hi - lo


def local_rows(x: torch.Tensor, group=None) -> torch.Tensor:
    """This rank's row slice of a tensor every rank holds in full (a view)."""
    lo, hi = shard_range(x.shape[0], _rank(group), _world(group))
    return x[lo:hi]


# ---- collectives on small partials ------------------------------------------------------

def allreduce_sum_(*tensors: torch.Tensor, group=None):
    """Sums each tensor over the ranks, in place, in argument order (every rank
    passes the same list).  Returns the tensors."""
    if _world(group) > 1:
        for t in tensors:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return tensors


def global_count(n_local: int, device, group=None) -> int:
    """Sum of n_local over the ranks (exact: int64)."""
    if _world(group) == 1:
        return int(n_local)
    t = torch.tensor([int(n_local)], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return int(t.item())


def sync_grads_(params, group=None):
    """Data-parallel weight-gradient sync: every parameter's .grad becomes the
    sum over ranks of the per-rank VJP partials (each a sum over that rank's
    rows).  Parameters without a gradient are skipped on every rank alike
    (the graph is the same on every rank)."""
    grads = [p.grad for p in params if p.grad is not None]
    allreduce_sum_(*grads, group=group)
    return grads


def reduce_scatter_rows(t: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of t over the ranks, of which this rank keeps only its row shard
    (rows shard_range(t.shape[0], rank, G)): the gradient of a replicated
    table for a caller that updates the table shard by shard.  Half the bytes
    of an all-reduce cross the links.  One reduce-scatter when the backend has
    it and the rows split evenly; otherwise an all-reduce and a slice (same
    result)."""
    world, rank = _world(group), _rank(group)
    lo, hi = shard_range(t.shape[0], rank, world)
    if world == 1:
        return t
    if dist.get_backend(group) == "nccl" and t.shape[0] % world == 0 and t.is_contiguous():
        out = torch.empty((hi - lo,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.reduce_scatter_tensor(out, t, op=dist.ReduceOp.SUM, group=group)
        return out
    allreduce_sum_(t, group=group)
    return t[lo:hi]


# ---- sharded layers -------------------------------------------------------------------

class _CrossEntropySharded(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, group):
        m = global_count(logits.shape[0], logits.device, group)
        loss, row_max, row_sum, _, t, _ = F.cross_entropy_fwd(logits, targets, total_rows=m)
        allreduce_sum_(loss, group=group)
        ctx.save_for_backward(logits, t, row_max, row_sum)
        ctx.m = m
        return loss.reshape(())

    @staticmethod
    def backward(ctx, g):
        logits, t, row_max, row_sum = ctx.saved_tensors
        g = g.reshape(1).to(torch.float32).contiguous()
        return F.cross_entropy_bwd(logits, t, row_max, row_sum, g, total_rows=ctx.m), None, None


def cross_entropy(logits, targets, group=None):
    """F.cross_entropy over row-sharded logits: the mean over ALL ranks' rows
    of -log_softmax(logits)[i, targets[i]], the same value on every rank.
    Each rank's VJP is its slice of the global VJP (scale g / M_global)."""
    return _CrossEntropySharded.apply(logits, targets, group)


class _EmbeddingVocabSharded(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight_shard, vocab_offset, vocab_total, group):
        out, _ = F.embedding_fwd(ids, weight_shard, vocab_offset, vocab_total)
        allreduce_sum_(out, group=group)
        ctx.save_for_backward(ids)
        ctx.meta = (weight_shard.shape[0], vocab_offset, vocab_total)
        return out

    @staticmethod
    def backward(ctx, dout):
        (ids,) = ctx.saved_tensors
        rows, off, total = ctx.meta
        dshard, _ = F.embedding_bwd(ids, F.dense(dout), rows, off, total)
        return None, dshard, None, None, None


def embedding(indices, weight_shard, vocab_total, group=None):
    """F.embedding over a vocab-sharded table.  Rank r holds rows
    ``vocab_shard(vocab_total, r, G)`` of the table and every rank passes the
    same ids; the result (every rank) is the full lookup.  Ids are validated
    against the whole vocabulary (negative ids count from its end), like the
    reference's index_select (crates/oxi-core/src/lib.rs:665-675).  The
    exchange is one sum of the [n, dim] output; a row owned by one shard is
    summed with zeros only, so the lookup is exact (a -0.0 entry comes back
    as +0.0)."""
    F._require_cuda_f32("weight", weight_shard)
    off, rows = vocab_shard(vocab_total, _rank(group), _world(group))
    if weight_shard.shape[0] != rows:
        raise ValueError(f"shape mismatch: rank {_rank(group)} holds {weight_shard.shape[0]} "
                         f"table rows, its shard of {vocab_total} has {rows}")
    ids = F._ids_tensor(indices, vocab_total, weight_shard.device)
    return _EmbeddingVocabSharded.apply(ids, weight_shard, off, vocab_total, group)


def exchange_rows(send_ids, send_rows, send_counts, group=None):
    """Variable-size all-to-all of rows: this rank sends rows
    [sum(send_counts[:s]), sum(send_counts[:s+1])) of (send_ids, send_rows) to
    rank s.  Returns (recv_ids, recv_rows, recv_counts) with the rows from
    rank s at [sum(recv_counts[:s]), ...).  The counts cross first (one small
    all-to-all, read on the host: the receive sizes depend on them)."""
    counts = send_counts.to(torch.int64).reshape(-1)
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    sc, rc = counts.tolist(), recv_counts.tolist()
    nsend, nrecv = sum(sc), sum(rc)
    recv_ids = torch.empty(nrecv, dtype=send_ids.dtype, device=send_ids.device)
    dist.all_to_all_single(recv_ids, send_ids[:nsend], rc, sc, group=group)
    recv_rows = torch.empty((nrecv,) + tuple(send_rows.shape[1:]), dtype=send_rows.dtype,
                            device=send_rows.device)
    dist.all_to_all_single(recv_rows, send_rows[:nsend], rc, sc, group=group)
    return recv_ids, recv_rows, rc


class SparseGradExchange:
    """The sparse exchange of a replicated [vocab_total, cols] table's gradient
    over token-sharded ids, with its buffers held for repeated steps.

    ``vjp(ids, dout, slot)`` runs the compact VJP in two calls: the plan (sort,
    distinct ids, per-shard counts) on the current stream, then -- while the
    sums run -- the counts' all-to-all on a side stream and their copy to the
    host, which is the only thing the host waits for.  ``exchange(slot)``
    sends the rows to their owners and sums them (``oxc_embedding_exchange_
    reduce``) on a communication stream that waits for the sums; it returns
    the rank's dense shard of the gradient and an event recorded after the
    reduce, so the caller's next forward can overlap the exchange.  Two slots
    let step i's exchange run while step i + 1 computes its VJP into the other
    slot."""

    def __init__(self, n, vocab_total, cols, device, group=None, slots=2):
        from . import _native as N
        self.N, self.L = N, N.load()
        self.group = group
        self.world, self.rank = _world(group), _rank(group)
        self.n, self.v, self.d, self.dev = int(n), int(vocab_total), int(cols), device
        cap = max(1, min(self.n, self.v))
        t = torch
        self.ids = [t.empty(cap, dtype=t.int32, device=device) for _ in range(slots)]
        self.rows = [t.empty(cap, self.d, dtype=t.float32, device=device) for _ in range(slots)]
        self.count = [t.empty(1, dtype=t.int64, device=device) for _ in range(slots)]
        self.sc = [t.empty(self.world, dtype=t.int64, device=device) for _ in range(slots)]
        self.rc = [t.empty(self.world, dtype=t.int64, device=device) for _ in range(slots)]
        self.lo, self.shard_rows = vocab_shard(self.v, self.rank, self.world)
        self.dshard = [t.empty(self.shard_rows, self.d, dtype=t.float32, device=device)
                       for _ in range(slots)]
        self.host_counts = [t.empty(2 * self.world, dtype=t.int64, pin_memory=True)
                            for _ in range(slots)]
        self.flag = t.zeros(4, dtype=t.int32, device=device)
        self.ws_bytes = self.L.oxc_embedding_bwd_compact_workspace_size(self.n, self.v, self.d)
        self.ws = [F._workspace(self.ws_bytes, device) for _ in range(slots)]
        self.ws2_bytes = self.L.oxc_embedding_exchange_reduce_workspace_size(self.world,
                                                                              self.shard_rows)
        self.ws2 = [F._workspace(self.ws2_bytes, device) for _ in range(slots)]
        self.side = torch.cuda.Stream(device=device)
        self.comm = torch.cuda.Stream(device=device)
        self.counts = [None] * slots
        self.planned = [torch.cuda.Event() for _ in range(slots)]
        self.summed = [torch.cuda.Event() for _ in range(slots)]

    def vjp(self, ids, dout, slot=0):
        N, L = self.N, self.L
        cur = torch.cuda.current_stream()
        N.check(L.oxc_embedding_bwd_compact_plan(
            ids.data_ptr(), self.n, self.v, 0, self.v, self.d, self.ids[slot].data_ptr(),
            self.count[slot].data_ptr(), self.world, self.sc[slot].data_ptr(),
            self.flag.data_ptr(), self.ws[slot].data_ptr(), self.ws_bytes, cur.cuda_stream),
            "embedding backward (compact)")
        self.planned[slot].record(cur)
        with torch.cuda.stream(self.side):
            self.side.wait_event(self.planned[slot])
            dist.all_to_all_single(self.rc[slot], self.sc[slot], group=self.group)
            h = self.host_counts[slot]
            h[:self.world].copy_(self.sc[slot], non_blocking=True)
            h[self.world:].copy_(self.rc[slot], non_blocking=True)
        N.check(L.oxc_embedding_bwd_compact_sum(
            dout.data_ptr(), self.n, self.v, self.d, self.rows[slot].data_ptr(),
            self.ws[slot].data_ptr(), self.ws_bytes, cur.cuda_stream),
            "embedding backward (compact sums)")
        self.summed[slot].record(cur)
        self.side.synchronize()  # the counts only: the sums keep running
        h = self.host_counts[slot]
        self.counts[slot] = (h[:self.world].tolist(), h[self.world:].tolist())

    def exchange(self, slot=0):
        N, L = self.N, self.L
        sc, rc = self.counts[slot]
        nsend, nrecv = sum(sc), sum(rc)
        with torch.cuda.stream(self.comm):
            self.comm.wait_event(self.summed[slot])
            rid = torch.empty(nrecv, dtype=torch.int32, device=self.dev)
            dist.all_to_all_single(rid, self.ids[slot][:nsend], rc, sc, group=self.group)
            rrows = torch.empty(nrecv, self.d, dtype=torch.float32, device=self.dev)
            dist.all_to_all_single(rrows, self.rows[slot][:nsend], rc, sc, group=self.group)
            off = [0]
            for c in rc:
                off.append(off[-1] + c)
            src_off = torch.tensor(off, dtype=torch.int64).to(self.dev)
            N.check(L.oxc_embedding_exchange_reduce(
                rid.data_ptr(), rrows.data_ptr(), src_off.data_ptr(), self.world, self.lo,
                self.shard_rows, self.d, self.dshard[slot].data_ptr(), self.flag.data_ptr(),
                self.ws2[slot].data_ptr(), self.ws2_bytes, self.comm.cuda_stream),
                "embedding gradient exchange")
            done = torch.cuda.Event()
            done.record(self.comm)
        return self.dshard[slot], done


class PeerGradExchange:
    """The same exchange over peer memory (NVLink), without NCCL moving the
    rows and without the host waiting on counts.  Every (owner p, source s)
    pair has a region: rows [cap, cols], ids [cap], a count.  The VJP kernel
    (``oxc_embedding_bwd_push``) writes each occurring row's sum into the
    region of the row's owner.  Per slot, each rank holds one buffer of regions
    (rows [ranks, cap, cols], ids [ranks, cap], counts [ranks]), exported once
    with CUDA IPC and mapped by every other rank.

    ``mode="push"`` (the default): the buffer of rank p holds every source's
    region for owner p, so the VJP kernel stores the rows into the owners'
    memory itself (fenced at system scope) and the owner sums its own buffer
    (``oxc_embedding_exchange_reduce_regions``).  ``mode="pull"``: the buffer of
    rank s holds s's regions for every owner, so the VJP writes only this GPU's
    memory; after the barrier each owner's ``oxc_embedding_exchange_pull``
    reads its region from every source's memory and sums them in rank order
    into its dense shard, on the communication stream.  Both give the same
    bits.  On two B200s (config 4) push took 1.17 ms per step and pull 1.41:
    pull's VJP is shorter (0.61 against 0.70 ms), but its owner-side reads over
    NVLink outlast the next forward they overlap.  ``exchange(slot)`` is a stream-ordered barrier (a
    one-element all-reduce: it completes on a rank only after every rank's VJP
    kernel has completed) followed by the owner's sum on a communication
    stream; it returns the dense gradient shard and an event.

    Ownership: ``cyclic`` (the default) gives rank p the table rows p, p + N,
    p + 2N, ... (N ranks), so its dense shard's row v is table row p + v * N;
    a Zipf id stream touches its low ids most, and cyclic ownership spreads
    them, and the NVLink traffic they bring, over every owner.  ``cyclic=False``
    gives rank p the contiguous ``vocab_shard`` rows.

    Ordering across steps: a source writes a slot's regions again two steps
    later, after the barrier of the step in between (``vjp`` waits for it),
    which every owner enters only after its reduce of that slot (both run in
    order on the owner's communication stream)."""

    def __init__(self, n, vocab_total, cols, device, group=None, slots=2, cyclic=True,
                 mode="push"):
        import ctypes
        import math
        from . import _native as N
        self.N, self.L, self.ctypes = N, N.load(), ctypes
        self.group = group
        self.world, self.rank = _world(group), _rank(group)
        if slots < 2:
            raise ValueError("invalid argument: the fused exchange needs two slots (a source "
                             "writes a slot again only after the owner's reduce of it)")
        if self.world > N.PUSH_MAX_RANKS:
            raise NotImplementedError(f"not implemented: the fused exchange over {self.world} "
                                      f"ranks (at most {N.PUSH_MAX_RANKS})")
        if mode not in ("pull", "push"):
            raise ValueError(f"invalid argument: exchange mode {mode!r} (pull or push)")
        self.mode = mode
        self.n, self.v, self.d, self.dev, self.slots = int(n), int(vocab_total), int(cols), \
            device, slots
        self.cap = math.ceil(self.v / self.world)  # rows of the largest vocab shard
        self.cyclic = bool(cyclic)
        if self.cyclic:  # rows rank, rank + N, ...
            self.lo, self.stride = self.rank, self.world
            self.shard_rows = (self.v - self.rank + self.world - 1) // self.world
        else:
            self.lo, self.shard_rows = vocab_shard(self.v, self.rank, self.world)
            self.stride = 1
        G, cap, d = self.world, self.cap, self.d
        t = torch
        self.rrows = [t.empty(G * cap * d, dtype=t.float32, device=device) for _ in range(slots)]
        self.rids = [t.empty(G * cap, dtype=t.int32, device=device) for _ in range(slots)]
        self.rcount = [t.zeros(G, dtype=t.int64, device=device) for _ in range(slots)]
        self.dshard = [t.empty(self.shard_rows, d, dtype=t.float32, device=device)
                       for _ in range(slots)]
        self.flag = t.zeros(4, dtype=t.int32, device=device)
        self.ws_bytes = self.L.oxc_embedding_bwd_compact_workspace_size(self.n, self.v, d)
        self.ws = [F._workspace(self.ws_bytes, device) for _ in range(slots)]
        self.ws2_bytes = self.L.oxc_embedding_exchange_reduce_workspace_size(G, self.shard_rows)
        self.ws2 = [F._workspace(self.ws2_bytes, device) for _ in range(slots)]
        self.comm = torch.cuda.Stream(device=device)
        self.token = t.zeros(1, dtype=t.float32, device=device)
        self.passed = None  # the last exchange's barrier, on the communication stream
        # export this rank's regions (one handle per allocation), map every other rank's
        mine, handles = [], {}
        try:
            for k in range(slots):
                entry = []
                for buf in (self.rrows[k], self.rids[k], self.rcount[k]):
                    h = (ctypes.c_uint8 * 64)()
                    off = ctypes.c_int64(0)
                    N.check(self.L.oxc_ipc_export(buf.data_ptr(), h, ctypes.byref(off)),
                            "ipc export")
                    key = buf.data_ptr() - off.value
                    handles.setdefault(key, bytes(h))
                    entry.append((handles[key], off.value))
                mine.append(entry)
        except RuntimeError as e:  # every rank learns of it through the gather
            mine = str(e)
        every = [None] * G
        dist.all_gather_object(every, mine, group=group)
        bad = [f"rank {p}: {e}" for p, e in enumerate(every) if isinstance(e, str)]
        if bad:
            raise RuntimeError("peer memory could not be exported on every rank: " + "; ".join(bad))
        # Map every other rank's allocations, each distinct handle once (buffers
        # of one allocation share it; a process maps a handle only once).
        self.mapped = []  # base pointers to unmap
        opened, base, err = {}, {}, ""
        try:
            for p in range(G):
                for k in range(slots):
                    for j, buf in enumerate((self.rrows[k], self.rids[k], self.rcount[k])):
                        if p == self.rank:
                            base[(p, k, j)] = buf.data_ptr()
                            continue
                        h, off = every[p][k][j]
                        if (p, h) not in opened:
                            ptr = ctypes.c_void_p()
                            N.check(self.L.oxc_ipc_import(
                                (ctypes.c_uint8 * 64).from_buffer_copy(h), 0, ctypes.byref(ptr)),
                                "ipc import")
                            opened[(p, h)] = ptr.value
                            self.mapped.append(ptr.value)
                        base[(p, k, j)] = opened[(p, h)] + off
        except RuntimeError as e:  # reported on every rank alike below
            err = str(e)
        ok = torch.tensor([0.0 if err else 1.0], device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if ok.item() < 1.0:
            for ptr in self.mapped:
                self.L.oxc_ipc_close(ptr, 0)
            self.mapped = []
            raise RuntimeError("peer memory could not be mapped on every rank"
                               + (f": {err}" if err else ""))
        # region (owner p, source s): in owner p's buffer at index s (push), or
        # in source s's buffer at index p (pull)
        def region(owner, source, k):
            holder, index = (owner, source) if mode == "push" else (source, owner)
            return (base[(holder, k, 0)] + index * cap * d * 4, base[(holder, k, 1)] + index * cap * 4,
                    base[(holder, k, 2)] + index * 8)

        def to_device(tab):
            return t.tensor(list(bytes(tab)), dtype=t.uint8).to(device)

        self.push, self.pull = [], []
        for k in range(slots):
            tab = N.EmbPush()
            tab.world, tab.source, tab.cyclic, tab.cap = G, self.rank, int(self.cyclic), cap
            tab.local = int(mode == "pull")
            for p in range(G + 1):
                tab.lo[p] = self.v * p // G
            for p in range(G):
                tab.rows[p], tab.ids[p], tab.count[p] = region(p, self.rank, k)
            self.push.append(to_device(tab))
            if mode == "pull":
                pt = N.EmbPull()
                for src in range(G):
                    pt.rows[src], pt.ids[src], pt.count[src] = region(self.rank, src, k)
                self.pull.append(to_device(pt))
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def vjp(self, ids, dout, slot=0):
        cur = torch.cuda.current_stream()
        if self.passed is not None:
            # Slot k was last written two exchanges ago; every owner's reduce of
            # it precedes that owner's part in the last barrier.
            cur.wait_event(self.passed)
        self.N.check(self.L.oxc_embedding_bwd_push(
            dout.data_ptr(), ids.data_ptr(), self.n, self.v, self.d, self.push[slot].data_ptr(),
            self.flag.data_ptr(), self.ws[slot].data_ptr(), self.ws_bytes, cur.cuda_stream),
            "embedding backward (push)")

    def exchange(self, slot=0):
        """Runs on the communication stream after the current stream's VJP, so
        the next forward overlaps the barrier and the reduce."""
        cur = torch.cuda.current_stream()
        pushed = torch.cuda.Event()
        pushed.record(cur)
        with torch.cuda.stream(self.comm):
            self.comm.wait_event(pushed)
            # stream-ordered barrier: behind this stream's previous reduce here,
            # behind every rank's VJP of this slot everywhere
            dist.all_reduce(self.token, group=self.group)
            self.passed = torch.cuda.Event()
            self.passed.record(self.comm)
            if self.mode == "pull":
                self.N.check(self.L.oxc_embedding_exchange_pull(
                    self.pull[slot].data_ptr(), self.world, self.cap, self.lo, self.stride,
                    self.shard_rows, self.d, self.dshard[slot].data_ptr(), self.flag.data_ptr(),
                    self.ws2[slot].data_ptr(), self.ws2_bytes, self.comm.cuda_stream),
                    "embedding gradient exchange (pull)")
            else:
                self.N.check(self.L.oxc_embedding_exchange_reduce_regions(
                    self.rids[slot].data_ptr(), self.rrows[slot].data_ptr(),
                    self.rcount[slot].data_ptr(), self.world, self.cap, self.lo, self.stride,
                    self.shard_rows, self.d, self.dshard[slot].data_ptr(), self.flag.data_ptr(),
                    self.ws2[slot].data_ptr(), self.ws2_bytes, self.comm.cuda_stream),
                    "embedding gradient exchange")
            done = torch.cuda.Event()
            done.record(self.comm)
        return self.dshard[slot], done

    def close(self):
        """Unmaps the other ranks' regions after every rank's last use, and
        returns once every rank has unmapped this rank's (so its buffers may be
        freed).  Collective: every rank calls it."""
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        for ptr in self.mapped:
            self.N.check(self.L.oxc_ipc_close(ptr, 0), "ipc close")
        self.mapped = []
        dist.barrier(group=self.group)


def embedding_grad(ids, dout, vocab_total, group=None):
    """Gradient of a replicated [vocab_total, cols] table from this rank's
    tokens (ids [n], dout [n, cols]), summed over every rank's tokens; each
    rank returns the rows of its vocab shard (``vocab_shard``).  The sparse
    exchange (``SparseGradExchange``): the compact VJP (touched rows only), an
    all-to-all of those rows to their shard's owner, and
    ``oxc_embedding_exchange_reduce`` (a sum in rank order per row).  A row
    touched by one rank's tokens only is that rank's position-order sum, bit
    for bit; a row touched by several ranks is the sum of their partials in
    rank order.  One rank: the plain VJP.  The result is ordered on the
    current stream."""
    world = _world(group)
    F._require_cuda_f32("dout", dout)
    dout = F.dense(dout)
    if world == 1:
        return F.embedding_bwd(ids, dout, vocab_total)[0]
    ex = SparseGradExchange(ids.numel(), vocab_total, dout.shape[-1], dout.device, group, slots=1)
    ex.vjp(ids, dout, 0)
    dshard, done = ex.exchange(0)
    torch.cuda.current_stream().wait_event(done)
    return dshard


def sum_squares(tensors, group=None) -> torch.Tensor:
    """Sum over ranks and tensors of sum(v*v) (0-d f64 tensor, every rank)."""
    tot = T.sum_squares(tensors)
    allreduce_sum_(tot, group=group)
    return tot


def sum_all(x, group=None) -> torch.Tensor:
    """Whole-tensor sum over every rank's shard, f64 partials (0-d f64)."""
    tot = T.reduce_all("sum", x, f64=True)
    allreduce_sum_(tot, group=group)
    return tot


def clip_grad_norm_(grads, max_norm, norm_type=2.0, group=None):
    """clip_grad_norm_ (python/oxitorch/optim.py:242-263) over gradients that
    are sharded across ranks (activation gradients of row-sharded tensors):
    the total norm is taken over every rank's shard, and each rank scales its
    own shard.  Returns the pre-clip total norm (every rank)."""
    if norm_type != 2.0:
        raise NotImplementedError("not implemented: clip_grad_norm_ with norm_type != 2 on device")
    grads = [g for g in grads if g is not None]
    dev = grads[0].device if grads else torch.device("cuda")
    tot = torch.zeros((), dtype=torch.float64, device=dev)
    for i in range(0, len(grads), 16):
        tot += T.sum_squares(grads[i:i + 16])
    allreduce_sum_(tot, group=group)
    total = float(tot.item()) ** 0.5
    scale = max_norm / (total + 1e-6)
    if scale < 1.0:
        for g in grads:
            T.scale_(g, scale)
    return total
