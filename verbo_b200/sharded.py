"""Host logic of the multi-GPU forms of the sampler (one process per GPU).

Row sharding needs no collective: rows are independent, so each rank samples
``row_bounds(rows, world, rank)`` of the batch.

Vocab sharding (a row split over ranks by columns, as a tensor-parallel LM head
leaves it): every rank runs ``verbo_cuda_shard_topk`` on its contiguous column
shard ``shard_bounds(vocab, world, rank)``, the per-rank candidate buffers
``[rows][k]`` are all-gathered into ``[world][rows][k]``, and every rank runs
``verbo_cuda_merge_sample`` with the same per-row RNG state, so all ranks draw
the same ids.  The global top_k set lies in the union of the shards' top-k
sets when top_k <= k, so the result equals the unsharded pick.

Tensor-parallel logits tail: with the LM head split by vocab rows (rank r
holds rows ``shard_bounds(vocab, world, r)``, e.g. ``verbo_b200.Tail`` built
from that slice of the head), every rank turns the same hidden rows into the
logits of its own shard only and feeds them to the same sharded pick
(``sample_tail_sharded``): no rank ever holds a full logits row, and each reads
1/world of the head.

The collective is the only cross-rank step; ``gather_candidates`` uses the
process group's timeout, so a rank that died turns into an error on the
others instead of a hang.
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


def sample_vocab_sharded(shard, col_offset: int, vocab: int, opts, k: int, rng, hist=None, hist_off=None,
                         out=None, group=None, stream=None):
    """One vocab-sharded pick over this rank's column shard (CUDA tensors).
    Returns the ids, identical on every rank."""
    import verbo_b200 as vb

    cv, ci = vb.shard_topk(shard, col_offset, vocab, opts, k, hist, hist_off, stream=stream)
    gv, gi = gather_candidates(cv, ci, group)
    return vb.merge_sample(gv, gi, vocab, opts, rng=rng, out=out, stream=stream)


def sample_tail_sharded(tail, x, col_offset: int, vocab: int, opts, k: int, rng, hist=None, hist_off=None,
                        out=None, logits=None, group=None, stream=None):
    """Tensor-parallel logits tail + pick: `tail` holds the head rows
    [col_offset, col_offset + tail.vocab) of a vocab sharding of the LM head,
    `x` the hidden rows (the same on every rank).  This rank's shard of the
    logits (into `logits` if given) feeds the vocab-sharded pick; returns the
    ids, identical on every rank."""
    shard = tail.logits(x, out=logits, stream=stream)
    return sample_vocab_sharded(shard, col_offset, vocab, opts, k, rng, hist, hist_off, out=out, group=group,
                                stream=stream)
