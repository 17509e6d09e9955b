"""Host logic of the multi-GPU forms of the sampler (one process per GPU).

Row sharding needs no collective: rows are independent, so each rank samples
``row_bounds(rows, world, rank)`` of the batch.

Vocab sharding (a row split over ranks by columns, as a tensor-parallel LM head
leaves it): every rank holds a contiguous column shard
``shard_bounds(vocab, world, rank)`` and calls the library's
``verbo_cuda_sharded_sample`` through a ``verbo_b200.Comm``: the shard's top-k
(value, global id) candidates, one NCCL all-gather of the packed candidates
of every rank over NVLink, and the merge with the same per-row RNG state on
every rank, so all ranks draw the same ids, all on the caller's stream.  The
global top_k set lies in the union of the shards' top-k sets when
top_k <= k, so the result equals the unsharded pick.  ``make_comm`` builds the
communicator: rank 0's NCCL id reaches the other ranks through
torch.distributed (any backend), the only thing torch is used for here.

Tensor-parallel logits tail: with the LM head split by vocab rows (rank r
holds rows ``shard_bounds(vocab, world, r)``, e.g. ``verbo_b200.Tail`` built
from that slice of the head), every rank turns the same hidden rows into the
logits of its own shard only and feeds them to the same sharded pick
(``sample_tail_sharded``): no rank ever holds a full logits row, and each reads
1/world of the head.

``gather_candidates`` is the same exchange through torch.distributed (the
layout ``verbo_cuda_merge_sample`` expects), for hosts without the library's
communicator (CPU tests with gloo).  ``Comm.wait`` bounds the wait for a
collective: a rank that died turns into an error on the others, not a hang.
"""
from __future__ import annotations

from typing import Tuple


def row_bounds(rows: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous rows [lo, hi) of `rank` (the first rows % world ranks get one more)."""
    base, extra = divmod(rows, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_bounds(vocab: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous global columns [lo, hi) held by `rank`."""
    return row_bounds(vocab, world, rank)


def gather_candidates(cand_val, cand_id, group=None):
    """All-gathers per-rank [rows][k] candidates into [world][rows][k] on every rank."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rows, k = cand_val.shape
    out_v = torch.empty((world, rows, k), dtype=cand_val.dtype, device=cand_val.device)
    out_i = torch.empty((world, rows, k), dtype=cand_id.dtype, device=cand_id.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out_v, cand_val.contiguous(), group=group)
        dist.all_gather_into_tensor(out_i, cand_id.contiguous(), group=group)
    else:
        dist.all_gather(list(out_v.unbind(0)), cand_val.contiguous(), group=group)
        dist.all_gather(list(out_i.unbind(0)), cand_id.contiguous(), group=group)
    return out_v, out_i


def broadcast_unique_id(make_id, group=None) -> bytes:
    """The id rank 0 of `group` makes with `make_id()`, on every rank."""
    import torch.distributed as dist

    obj = [make_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def make_comm(device: int, group=None):
    """The library's communicator over the ranks of `group` (collective: every
    rank calls it); a single process (no process group) gets a one-rank one."""
    import torch.distributed as dist

    import verbo_b200 as vb

    if not dist.is_available() or not dist.is_initialized():
        return vb.Comm(vb.Comm.unique_id(), 1, 0, device)
    uid = broadcast_unique_id(vb.Comm.unique_id, group)
    return vb.Comm(uid, dist.get_world_size(group), dist.get_rank(group), device)


def sample_vocab_sharded(comm, shard, col_offset: int, vocab: int, opts, k: int, rng, hist=None, hist_off=None,
                         out=None, stats=None, stream=None):
    """One vocab-sharded pick over this rank's column shard (CUDA tensors):
    verbo_cuda_sharded_sample on `comm`.  Returns the ids, identical on every
    rank."""
    return comm.sample(shard, col_offset, vocab, opts, k, rng, hist, hist_off, out=out, stats=stats, stream=stream)


def sample_tail_sharded(comm, tail, x, col_offset: int, vocab: int, opts, k: int, rng, hist=None, hist_off=None,
                        out=None, logits=None, stream=None):
    """Tensor-parallel logits tail + pick: `tail` holds the head rows
    [col_offset, col_offset + tail.vocab) of a vocab sharding of the LM head,
    `x` the hidden rows (the same on every rank).  This rank's shard of the
    logits (into `logits` if given) feeds the vocab-sharded pick; returns the
    ids, identical on every rank."""
    shard = tail.logits(x, out=logits, stream=stream)
    return sample_vocab_sharded(comm, shard, col_offset, vocab, opts, k, rng, hist, hist_off, out=out, stream=stream)
