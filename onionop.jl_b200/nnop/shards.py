"""Sharding the hot path over ranks, one process per GPU.

Every op of the path is independent across its outer dimension, so a job is
split into per-rank shards with no data exchange on the attention path:

* attention shards by (batch, kv head) units (``shard_batch_heads``): the
  query heads of one kv head stay together, so dK and dV need no cross-rank
  sum, and a workload with few batches (the GQA workload has B = 4) still
  spreads over 8 GPUs by kv-head groups;
  with a key-padding mask the work of batch b grows with its key length
  len_b (the kernels skip key tiles past len_b), so ``balance_by_length``
  splits the batch by the total of len_b instead of by count;
* the norms, softmax and RoPE shard by rows; the norms' weight (and bias)
  gradients are sums over all rows, so their backward takes ONE all-reduce
  of the emb-long fp32 partials (``allreduce_norm_grads``) -- 16 KB at
  emb = 4096, a latency-bound step outside the kernels.

The collectives go through ``torch.distributed`` (NCCL between GPUs, gloo for
the CPU tests).  Without an initialised process group, or with one rank,
every function here is the single-GPU path.
"""
from __future__ import annotations

import heapq

import torch

from . import grad_layer_norm, grad_rms_norm

__all__ = ["row_shard", "balance_by_length", "shard_batch_heads", "piece_views", "allreduce_norm_grads",
           "grad_rms_norm_sharded", "grad_layer_norm_sharded"]


def row_shard(n: int, rank: int, world: int) -> slice:
    """Contiguous rows ``[lo, hi)`` of rank ``rank`` among ``world``: the first
    ``n % world`` ranks take one row more, so shard sizes differ by at most 1."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if n < 0:
        raise ValueError(f"negative row count {n}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return slice(lo, lo + base + (1 if rank < extra else 0))


def balance_by_length(lens, world: int) -> list[list[int]]:
    """Batch indices of each rank, balancing the total key length Σ len_b.

    Longest-processing-time-first: batches in decreasing length (ties by
    index) each go to the rank with the least total so far (ties by rank), so
    the largest total exceeds the mean by less than the longest single length.
    The result is deterministic, so every rank computes the same split from
    the same lengths without a collective.  Each rank's list is ascending."""
    if world < 1:
        raise ValueError(f"world of size {world}")
    lens = [int(x) for x in lens]
    if any(x < 0 for x in lens):
        raise ValueError("negative length")
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for b in sorted(range(len(lens)), key=lambda i: (-lens[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(b)
        heapq.heappush(heap, (load + lens[b], r))
    return [sorted(s) for s in out]


def shard_batch_heads(B: int, KH: int, rank: int, world: int) -> list[tuple[int, int, int, int]]:
    """This rank's share of an attention job, as pieces ``(b0, b1, h0, h1)``:
    batches ``[b0, b1)`` x kv heads ``[h0, h1)`` (query heads
    ``[h0·n_rep, h1·n_rep)``).

    The job's units are its (batch, kv head) pairs in batch-major order; each
    rank takes a contiguous run of them (``row_shard``: sizes differ by at most
    one unit, so with B·KH divisible by the world size every rank gets the same
    work).  A run is cut into at most three pieces, each a plain slice of the
    (B, H, L, E) tensors: a partial batch (one batch, a range of kv heads),
    whole batches (every kv head), a partial batch.  Every piece is an
    independent attention call; no piece needs data of another rank."""
    if B < 0 or KH <= 0:
        raise ValueError(f"invalid job: B={B}, KH={KH}")
    units = row_shard(B * KH, rank, world)
    lo, hi = units.start, units.stop
    out = []
    if lo == hi:
        return out
    if lo % KH:                                    # leading partial batch
        b, h0 = divmod(lo, KH)
        h1 = min(KH, h0 + (hi - lo))
        out.append((b, b + 1, h0, h1))
        lo = b * KH + h1
    if hi - lo >= KH:                              # whole batches
        nb = (hi - lo) // KH
        out.append((lo // KH, lo // KH + nb, 0, KH))
        lo += nb * KH
    if lo < hi:                                    # trailing partial batch
        b = lo // KH
        out.append((b, b + 1, 0, hi - lo))
    return out


def piece_views(piece, n_rep: int, q=None, k=None, v=None, pair=None):
    """The slices of (B, H, L, E) tensors q / k, v and of a (B, KL, QL, QH)
    pair bias that belong to one piece of ``shard_batch_heads``.  q, k, v views
    are contiguous; the pair view is contiguous only for whole-batch pieces
    (its head axis is innermost), so partial-batch pieces copy it."""
    b0, b1, h0, h1 = piece
    out = []
    if q is not None:
        out.append(q[b0:b1, h0 * n_rep:h1 * n_rep])
    if k is not None:
        out.append(k[b0:b1, h0:h1])
    if v is not None:
        out.append(v[b0:b1, h0:h1])
    if pair is not None:
        pv = pair[b0:b1, :, :, h0 * n_rep:h1 * n_rep]
        out.append(pv if pv.is_contiguous() else pv.contiguous())
    return out


def _world(group) -> int:
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return 1
    return dist.get_world_size(group)


def allreduce_norm_grads(*grads, group=None):
    """Sum per-rank weight / bias gradients over the ranks of ``group``.

    The gradients are packed into one fp32 buffer, reduced by ONE
    ``all_reduce(SUM)`` and unpacked into tensors of their own dtypes and
    shapes (a 16-bit dw is summed in fp32, then rounded once).  Every rank must
    call it with the same shapes, in the same order relative to its other
    collectives.  One rank or no process group: the inputs are returned."""
    if _world(group) == 1:
        return grads
    import torch.distributed as dist
    flat = torch.cat([g.reshape(-1).to(torch.float32) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    out, off = [], 0
    for g in grads:
        out.append(flat[off:off + g.numel()].reshape(g.shape).to(g.dtype))
        off += g.numel()
    return tuple(out)


def grad_rms_norm_sharded(dy, rstd, x, w, *, offset: float = 0.0, group=None):
    """``grad_rms_norm`` on this rank's rows, with dw summed over all ranks:
    returns ``(dx, dw)``; dx covers the local rows only, dw (fp32) is the
    gradient of the whole job's rows."""
    dx, dw = grad_rms_norm(dy, rstd, x, w, offset=offset)
    (dw,) = allreduce_norm_grads(dw, group=group)
    return dx, dw


def grad_layer_norm_sharded(dy, mean, rstd, x, w, b=None, *, group=None):
    """``grad_layer_norm`` on this rank's rows, with dw and db summed over all
    ranks by one all-reduce: returns ``(dx, dw, db)``."""
    dx, dw, db = grad_layer_norm(dy, mean, rstd, x, w, b)
    dw, db = allreduce_norm_grads(dw, db, group=group)
    return dx, dw, db
