"""Multi-process host logic on CPU (gloo, world size 2).

The per-shard candidate extraction and the merge are computed by the oracle
here (no GPU); what is under test is the product's host logic around them:
shard bounds, the all-gather layout [world][rows][k] that merge expects, that
every rank draws the same ids, and that a rank that dies before the
collective becomes an error (a short process-group timeout), not a hang.
"""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from verbo_b200 import sharded

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=timeout_s))


def _vocab_sharded_worker(rank, port, q):
    from oracle import pyoracle as po
    from verbo_b200 import workloads as wl

    _init(rank, port)
    try:
        w = wl.WORKLOADS["c5"].with_rows(6)
        x = wl.make_rows_np(w)
        h, off = wl.make_hist_np(w)
        o = po.sampling(**w.sampling_kwargs())
        lo, hi = sharded.shard_bounds(w.vocab, WORLD, rank)
        v, i = po.shard_topk(x[:, lo:hi], lo, w.vocab, o, 64, h, off)
        gv, gi = sharded.gather_candidates(torch.from_numpy(v), torch.from_numpy(i))
        ids, _ = po.merge_sample(gv.numpy(), gi.numpy(), w.vocab, o, po.seed_states(w.sampler_seeds(0, 6)))
        q.put((rank, ids.tolist(), gv.shape))
    finally:
        dist.destroy_process_group()


def _dead_rank_worker(rank, port, q):
    _init(rank, port, timeout_s=5)
    if rank == 1:
        os._exit(0)   # leaves before the collective
    try:
        sharded.gather_candidates(torch.zeros(2, 4), torch.zeros(2, 4, dtype=torch.int32))
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, type(e).__name__))


def _run(fn):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    return out


def test_bounds_partition():
    for n, world in ((151936, 8), (10, 3), (5, 8), (1024, 2)):
        spans = [sharded.row_bounds(n, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def test_vocab_sharded_gloo_matches_unsharded():
    from oracle import pyoracle as po
    from verbo_b200 import workloads as wl

    res = sorted(_run(_vocab_sharded_worker))
    assert len(res) == WORLD
    assert res[0][1] == res[1][1]                 # every rank draws the same ids
    assert tuple(res[0][2]) == (WORLD, 6, 64)
    w = wl.WORKLOADS["c5"].with_rows(6)
    x = wl.make_rows_np(w)
    h, off = wl.make_hist_np(w)
    direct, _ = po.sample_rows(x, po.sampling(**w.sampling_kwargs()), po.seed_states(w.sampler_seeds(0, 6)), h, off)
    assert res[0][1] == direct.tolist()


def test_dead_rank_becomes_an_error():
    res = _run(_dead_rank_worker)
    assert res == [(0, "DistBackendError")] or (len(res) == 1 and res[0][0] == 0 and res[0][1] != "no error")
