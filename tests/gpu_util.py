"""Helpers for the GPU parity tests: run the CUDA path and the oracle on the
same seeded inputs and compare them with the parity criteria of the path.

Parity criteria (the reference's sampler, src/sampler.cpp:50-109):
  * greedy ids and top-k candidate sets: bit-exact;
  * probabilities (softmax normaliser, kept mass): within 1e-5 relative;
  * sampled ids: identical, except where the oracle reports the uniform or a
    top-p / min-p decision within 1e-6 of a boundary.  Such rows are counted
    and returned, never hidden.
"""
from __future__ import annotations

import numpy as np
import torch

import verbo_b200 as vb
from oracle import pyoracle as po

BOUNDARY = 1e-6
PROB_RTOL = 1e-5


def to_dev_rng(states: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(states).view(np.int64).copy()).cuda()


def from_dev_rng(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint64).copy()


def stats_np(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(po.STATS_DTYPE).copy()


def run_gpu(x: np.ndarray, opts: dict, seeds=None, hist=None, off=None, steps: int = 1, ld: int | None = None,
            states: np.ndarray | None = None):
    """CUDA path: `steps` consecutive picks per row.  Returns (ids[rows,steps],
    stats of the last step, final rng states)."""
    rows, V = x.shape
    if ld is not None and ld != V:
        pad = np.zeros((rows, ld), dtype=np.float32)
        pad[:, :V] = x
        dx = torch.from_numpy(pad).cuda()
    else:
        dx = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    if states is None:
        states = po.seed_states(seeds if seeds is not None else np.arange(1, rows + 1, dtype=np.uint64))
    rng = to_dev_rng(states)
    dh = None if hist is None else torch.from_numpy(np.ascontiguousarray(hist, dtype=np.int32)).cuda()
    do = None if off is None else torch.from_numpy(np.ascontiguousarray(off, dtype=np.int64)).cuda()
    st = torch.zeros(rows * vb.ROW_STATS_BYTES, dtype=torch.uint8, device="cuda")
    o = vb.Sampling(**opts)
    ids = []
    for _ in range(steps):
        out = vb.sample(dx, o, rng=rng, hist=dh, hist_off=do, stats=st, vocab=V)
        ids.append(out.cpu().numpy())
    vb.check()
    return np.stack(ids, axis=1), stats_np(st), from_dev_rng(rng)


def run_oracle(x: np.ndarray, opts: dict, seeds=None, hist=None, off=None, steps: int = 1, states=None):
    rows = x.shape[0]
    st = po.seed_states(seeds if seeds is not None else np.arange(1, rows + 1, dtype=np.uint64)) \
        if states is None else states.copy()
    o = po.sampling(**opts)
    ids, all_stats = [], []
    for _ in range(steps):
        i, s = po.sample_rows(x, o, st, hist, off)
        ids.append(i)
        all_stats.append(s)
    return np.stack(ids, axis=1), np.stack(all_stats, axis=1), st


def compare(gpu_ids: np.ndarray, ora_ids: np.ndarray, ora_stats: np.ndarray, what: str = ""):
    """Asserts parity; returns the number of boundary rows that differ."""
    diff = gpu_ids != ora_ids
    if not diff.any():
        return 0
    # a step that differs also desynchronises nothing (the rng advances once per
    # pick either way), so each differing (row, step) is judged on its own
    margin = np.minimum(ora_stats["draw_margin"], ora_stats["cut_margin"])
    bad = diff & ~(margin < BOUNDARY)
    assert not bad.any(), (f"{what}: {int(bad.sum())} non-boundary mismatches; first at "
                           f"{np.argwhere(bad)[0].tolist()} gpu={gpu_ids[bad][:5]} oracle={ora_ids[bad][:5]} "
                           f"margins={margin[bad][:5]}")
    return int(diff.sum())
