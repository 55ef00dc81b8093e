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


def embedding_grad(ids, dout, vocab_total, group=None):
    """Gradient of a replicated [vocab_total, cols] table from this rank's
    tokens (ids [n], dout [n, cols]), summed over every rank's tokens; each
    rank returns the rows of its vocab shard (``vocab_shard``).  The sparse
    exchange: the compact VJP (touched rows only), ``exchange_rows`` to the
    shard owners, and ``oxc_embedding_exchange_reduce`` (a sum in rank order
    per row).  A row touched by one rank's tokens only is that rank's
    position-order sum, bit for bit; a row touched by several ranks is the sum
    of their partials in rank order.  One rank: the plain VJP."""
    from . import _native as N
    world, rank = _world(group), _rank(group)
    F._require_cuda_f32("dout", dout)
    dout = F.dense(dout)
    n, cols = ids.numel(), dout.shape[-1]
    if world == 1:
        return F.embedding_bwd(ids, dout, vocab_total)[0]
    L = N.load()
    dev = dout.device
    cap = max(1, min(n, vocab_total))
    out_ids = torch.empty(cap, dtype=torch.int32, device=dev)
    out_rows = torch.empty(cap, cols, dtype=torch.float32, device=dev)
    count = torch.empty(1, dtype=torch.int64, device=dev)
    shard_counts = torch.empty(world, dtype=torch.int64, device=dev)
    flag = torch.zeros(4, dtype=torch.int32, device=dev)
    ws = F._workspace(L.oxc_embedding_bwd_compact_workspace_size(n, vocab_total, cols), dev)
    N.check(L.oxc_embedding_bwd_compact(dout.data_ptr(), ids.data_ptr(), n, vocab_total, 0,
                                        vocab_total, cols, out_ids.data_ptr(), out_rows.data_ptr(),
                                        count.data_ptr(), world, shard_counts.data_ptr(),
                                        flag.data_ptr(), ws.data_ptr(), ws.numel(), F._stream()),
            "embedding backward (compact)")
    recv_ids, recv_rows, rc = exchange_rows(out_ids, out_rows, shard_counts, group)
    off = [0]
    for c in rc:
        off.append(off[-1] + c)
    src_off = torch.tensor(off, dtype=torch.int64, device=dev)
    lo, rows = vocab_shard(vocab_total, rank, world)
    dshard = torch.empty(rows, cols, dtype=torch.float32, device=dev)
    ws2 = F._workspace(L.oxc_embedding_exchange_reduce_workspace_size(world, rows), dev)
    N.check(L.oxc_embedding_exchange_reduce(recv_ids.data_ptr(), recv_rows.data_ptr(),
                                            src_off.data_ptr(), world, lo, rows, cols,
                                            dshard.data_ptr(), flag.data_ptr(), ws2.data_ptr(),
                                            ws2.numel(), F._stream()),
            "embedding gradient exchange")
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
