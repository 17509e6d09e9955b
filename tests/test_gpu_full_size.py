"""Parity at the benchmark configurations' full sizes.

Every configuration of the benchmark plan (verbo_b200/workloads.py: C1 one
row, C2 256 greedy rows, C3 1024 top-k rows, C4 4096 full-vocabulary nucleus
rows, C5 512 rows in 8 column shards merged on one GPU) runs at its stated
size and seed through the C ABI and is compared with the C oracle (the
reference's Sampler::pick restated, pinned against the reference by
tests/test_oracle.py).  These sizes reach what the small cases cannot: split
grids of several resident waves, the multi-wave slice merge, and the
streaming full-vocabulary kernel's item pipeline over thousands of rows.

Criteria (src/sampler.cpp:50-109): greedy ids and top-k sets bit-exact;
the softmax normaliser and kept mass within 1e-5 relative; sampled ids equal
except rows whose oracle margin (uniform or top-p / min-p decision to the
nearest boundary, in units of the kept mass) is below 1e-6.  Every differing
row is counted; a differing row with a margin above 1e-7 fails the test.
With VERBO_PARITY_RECORD=<file> the counts are written there as JSON.
"""
from __future__ import annotations

import json
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

from oracle import pyoracle as po
from tests.gpu_util import BOUNDARY, PROB_RTOL, from_dev_rng, stats_np, to_dev_rng

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TIGHT = 1e-7  # a differing row needs an oracle margin below this


@pytest.fixture(scope="module", autouse=True)
def _lib(cuda_lib):
    if not torch.cuda.is_available():
        pytest.fail("gpu tests need a CUDA device")
    yield


def oracle_parallel(x, opts, seeds, h, off):
    """The C oracle over row chunks on all host threads (ctypes releases the
    GIL).  Returns (ids, stats, advanced rng states)."""
    rows = x.shape[0]
    nt = max(1, min(po.host_threads(), rows))
    bounds = np.linspace(0, rows, nt + 1).astype(int)
    states = po.seed_states(seeds)
    ids = np.zeros(rows, dtype=np.int32)
    stats = np.zeros(rows, dtype=po.STATS_DTYPE)
    o = po.sampling(**opts)

    def run(i):
        a, b = bounds[i], bounds[i + 1]
        if a == b:
            return
        hh = oo = None
        if h is not None:
            hh = h[off[a]:off[b]]
            oo = off[a:b + 1] - off[a]
        st = np.ascontiguousarray(states[a:b])
        ii, ss = po.sample_rows(x[a:b], o, st, hh, oo)
        ids[a:b] = ii
        stats[a:b] = ss
        states[a:b] = st

    with ThreadPoolExecutor(max_workers=nt) as ex:
        list(ex.map(run, range(nt)))
    return ids, stats, states


def record(name, **kw):
    path = os.environ.get("VERBO_PARITY_RECORD")
    if not path:
        return
    d = json.loads(open(path).read()) if os.path.exists(path) else {}
    d[name] = kw
    with open(path, "w") as f:
        f.write(json.dumps(d, indent=1) + "\n")


def judge(name, w, gpu_ids, gst, ora_ids, ost, gpu_rng=None, ora_rng=None, fallbacks=None):
    greedy = w.temp <= 0
    diff = gpu_ids != ora_ids
    margin = np.minimum(ost["draw_margin"], ost["cut_margin"])
    boundary = margin < BOUNDARY
    sampled = not greedy
    rel_sum = rel_tot = 0.0
    if sampled and gst is not None:
        rel_sum = float(np.max(np.abs(gst["sum"] - ost["sum"]) / np.abs(ost["sum"])))
        rel_tot = float(np.max(np.abs(gst["tot"] - ost["tot"]) / np.abs(ost["tot"])))
    record(name, workload=f"{w.rows} x {w.vocab}, temp {w.temp}, top_k {w.top_k}, top_p {w.top_p}, "
                          f"min_p {w.min_p}, repeat {w.repeat} over {w.hist_len} ids",
           rows=int(w.rows), differing_rows=int(diff.sum()),
           differing_margins=[float(m) for m in margin[diff]],
           oracle_boundary_rows_1e6=int(boundary.sum()), oracle_boundary_rows_1e9=int((margin < 1e-9).sum()),
           max_rel_err_sum=rel_sum, max_rel_err_tot=rel_tot,
           rng_states_equal=None if gpu_rng is None else bool(np.array_equal(gpu_rng, ora_rng)),
           full_vocab_fallback_rows=fallbacks)
    if greedy:
        assert not diff.any(), f"{name}: greedy ids differ in {int(diff.sum())} rows"
        return
    bad = diff & ~(margin < TIGHT)
    assert not bad.any(), (f"{name}: {int(bad.sum())} differing rows away from a boundary; first "
                           f"{np.argwhere(bad)[:3].ravel().tolist()} margins {margin[bad][:3]}")
    if gst is not None:
        assert rel_sum <= PROB_RTOL and rel_tot <= PROB_RTOL, (name, rel_sum, rel_tot)
    if gpu_rng is not None:
        assert np.array_equal(gpu_rng, ora_rng), f"{name}: rng states differ"


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4"])
def test_row_configs_full_size(name):
    import verbo_b200 as vb
    from verbo_b200 import workloads as wl

    w = wl.WORKLOADS[name]
    x = wl.make_rows_np(w)
    h, off = wl.make_hist_np(w)
    seeds = w.sampler_seeds(0, w.rows)
    opts = w.sampling_kwargs()
    dx = torch.from_numpy(x).cuda()
    dh = None if h is None else torch.from_numpy(h).cuda()
    do = None if off is None else torch.from_numpy(off).cuda()
    rng = to_dev_rng(po.seed_states(seeds))
    st = torch.zeros(w.rows * vb.ROW_STATS_BYTES, dtype=torch.uint8, device="cuda")
    ids = vb.sample(dx, vb.Sampling(**opts), rng=rng, hist=dh, hist_off=do, stats=st).cpu().numpy()
    vb.check()
    fb = vb.full_vocab_fallbacks() if name == "c4" else None
    gst = stats_np(st)
    grng = from_dev_rng(rng)
    del dx
    ora, ost, orng = oracle_parallel(x, opts, seeds, h, off)
    judge(name, w, ids, gst, ora, ost, grng, orng, fb)
    if fb is not None:  # the streaming kernel settles (almost) every row of C4
        assert fb <= w.rows // 100, f"{fb} of {w.rows} rows went to the staged kernel"


def test_c5_sharded_full_size():
    """C5: 8 column shards of 18992, per-shard top-64 (shard_topk), the merge
    (merge_sample) on one GPU, against the unsharded oracle."""
    import verbo_b200 as vb
    from verbo_b200 import workloads as wl

    w = wl.WORKLOADS["c5"]
    x = wl.make_rows_np(w)
    h, off = wl.make_hist_np(w)
    seeds = w.sampler_seeds(0, w.rows)
    opts = w.sampling_kwargs()
    o = vb.Sampling(**opts)
    k, n = 64, w.shards
    cols = w.vocab // n
    dx = torch.from_numpy(x).cuda()
    dh, do = torch.from_numpy(h).cuda(), torch.from_numpy(off).cuda()
    cv = torch.empty(n, w.rows, k, dtype=torch.float32, device="cuda")
    ci = torch.empty(n, w.rows, k, dtype=torch.int32, device="cuda")
    for s in range(n):
        vb.shard_topk(dx[:, s * cols:(s + 1) * cols], s * cols, w.vocab, o, k, dh, do, cand_val=cv[s], cand_id=ci[s])
    rng = to_dev_rng(po.seed_states(seeds))
    st = torch.zeros(w.rows * vb.ROW_STATS_BYTES, dtype=torch.uint8, device="cuda")
    ids = vb.merge_sample(cv, ci, w.vocab, o, rng=rng, stats=st).cpu().numpy()
    vb.check()
    # step 1 against the oracle's shard top-k, bit for bit (one shard suffices)
    ov, oi = po.shard_topk(x[:, :cols], 0, w.vocab, po.sampling(**opts), k, h, off)
    assert np.array_equal(ci[0].cpu().numpy(), oi) and np.array_equal(cv[0].cpu().numpy(), ov)
    ora, ost, orng = oracle_parallel(x, opts, seeds, h, off)
    judge("c5", w, ids, stats_np(st), ora, ost, from_dev_rng(rng), orng)


# Full-size rows on the other paths: the staged cluster kernel (full
# vocabulary with min-p and a penalty, several waves of 37 resident rows),
# large top-k (certified top-m slices, k up to 256), the streaming path at a
# sharper temperature (fewer, heavier members per cell) and the streaming
# path with min-p (src/sampler.cpp:86-91) where min-p cuts the kept prefix
# first, where top-p does, and without top-p.
EXTRA = {
    "general_minp_penalty": ("c4", 1024, dict(temp=1.0, top_k=0, top_p=0.95, min_p=0.02, repeat=1.1), 64),
    "topk_128": ("c3", 1024, dict(top_k=128), None),
    "topk_256": ("c5", 512, dict(top_k=256, min_p=0.0), None),
    "nucleus_sharp": ("c4", 2048, dict(temp=0.4, top_p=0.9), None),
    "nucleus_minp_first": ("c4", 1024, dict(temp=1.0, top_p=0.99, min_p=0.3), None),
    "nucleus_topp_first": ("c4", 1024, dict(temp=1.0, top_p=0.8, min_p=0.02), None),
    "nucleus_minp_only": ("c4", 1024, dict(temp=0.7, top_p=1.0, min_p=0.1), None),
}


@pytest.mark.parametrize("name", list(EXTRA))
def test_other_paths_full_size(name):
    import verbo_b200 as vb
    from verbo_b200 import workloads as wl

    cfg, rows, over, hist_len = EXTRA[name]
    w = wl.WORKLOADS[cfg].with_rows(rows)
    x = wl.make_rows_np(w, rows)
    opts = w.sampling_kwargs()
    opts.update(over)
    if hist_len is not None:
        g = np.random.default_rng(rows + hist_len)
        h = g.integers(0, w.vocab, size=rows * hist_len).astype(np.int32)
        off = np.arange(rows + 1, dtype=np.int64) * hist_len
        opts["repeat_last"] = hist_len
    elif opts.get("repeat", 1.0) != 1.0:
        h, off = wl.make_hist_np(w, rows)
    else:
        h = off = None
    seeds = w.sampler_seeds(0, rows)
    dx = torch.from_numpy(x).cuda()
    dh = None if h is None else torch.from_numpy(h).cuda()
    do = None if off is None else torch.from_numpy(off).cuda()
    rng = to_dev_rng(po.seed_states(seeds))
    st = torch.zeros(rows * vb.ROW_STATS_BYTES, dtype=torch.uint8, device="cuda")
    ids = vb.sample(dx, vb.Sampling(**opts), rng=rng, hist=dh, hist_off=do, stats=st).cpu().numpy()
    vb.check()
    del dx
    ora, ost, orng = oracle_parallel(x, opts, seeds, h, off)
    from dataclasses import replace

    ws = replace(w, name=name, temp=opts["temp"], top_k=opts["top_k"], top_p=opts["top_p"], min_p=opts["min_p"],
                 repeat=opts["repeat"], hist_len=0 if h is None else int(off[1] - off[0]), shards=1)
    fb = vb.full_vocab_fallbacks() if name.startswith("nucleus") else None
    judge(name, ws, ids, stats_np(st), ora, ost, from_dev_rng(rng), orng, fb)
    if fb is not None and name.startswith("nucleus_minp"):  # the streaming kernel settles (almost) every row
        assert fb <= rows // 100, f"{fb} of {rows} rows went to the staged kernel"
    if name.startswith("nucleus_minp") or name == "nucleus_topp_first":
        # the kept count is the reference's, min(min-p prefix, top-p prefix),
        # except where the cut itself is a boundary decision
        bad = (stats_np(st)["keep"] != ost["keep"]) & ~(ost["cut_margin"] < BOUNDARY)
        assert not bad.any(), f"{name}: kept counts differ in {int(bad.sum())} rows"
