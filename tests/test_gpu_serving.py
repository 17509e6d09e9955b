"""Request batching (verbo_cuda_server_* through verbo_b200.serving.BatchServer)
against verbo::generate.

Seven requests share three slots (and, in the mixed test, nine requests with
three option sets share four).  A deterministic stand-in model gives each
request's t-th logits row from (request id, t), with stop ids planted so that
some requests end early.  Each request is then replayed on the oracle as the
reference's generate loop would run it alone (src/sampler.cpp:111-181): a
Sampler seeded with the request's seed, accept(prompt), then pick / stop check
/ accept, the history being the prompt plus the tokens the request really got.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import pyoracle as po

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

V = 4096
STOP = (7, 11)


def model_row(rid: int, t: int) -> np.ndarray:
    g = np.random.default_rng([rid, t])
    row = (g.standard_normal(V) * 2.0).astype(np.float32)
    if rid % 3 == 1 and t == 2 + rid % 4:
        row[STOP[rid % 2]] = 50.0  # this request meets a stop id here
    return row


def stand_in_model(active, out):
    rows = np.zeros((len(active), V), dtype=np.float32)
    for s, r in enumerate(active):
        if r is not None:
            rows[s] = model_row(r.rid, len(r.tokens))
    out.copy_(torch.from_numpy(rows))


@pytest.mark.parametrize("opts", [dict(temp=0.0, repeat=1.3, repeat_last=32),
                                  dict(temp=0.8, top_k=40, top_p=0.9, min_p=0.02, repeat=1.15, repeat_last=48)],
                         ids=["greedy", "top-k"])
def test_batch_server_matches_one_generate_per_request(cuda_lib, opts):
    if not torch.cuda.is_available():
        pytest.fail("gpu tests need a CUDA device")
    import verbo_b200 as vb
    from verbo_b200.serving import BatchServer

    g = np.random.default_rng(31)
    srv = BatchServer(vb.Sampling(**opts), slots=3, vocab=V, model=stand_in_model, stop_ids=STOP)
    reqs = []
    for i in range(7):
        prompt = g.integers(0, V, size=int(g.integers(0, 80))).tolist()
        reqs.append((srv.submit(prompt, max_tokens=int(g.integers(3, 10)), seed=1000 + i), prompt))
    done = srv.run()
    assert sorted(done) == [rid for rid, _ in reqs]
    assert replay(done, [(rid, prompt, opts) for rid, prompt in reqs]) >= 1  # the planted stops were met


MIXED = [dict(temp=0.0, repeat=1.3, repeat_last=32),
         dict(temp=0.8, top_k=40, top_p=0.9, min_p=0.02, repeat=1.15, repeat_last=48),
         dict(temp=1.0, top_k=0, top_p=0.95, repeat=1.0)]


def test_batch_server_mixed_options(cuda_lib):
    """Requests with different options in flight together: each is sampled
    with its own (one launch chain per option set over contiguous rows, the
    rows re-packed as requests come and go) and matches its own generate."""
    if not torch.cuda.is_available():
        pytest.fail("gpu tests need a CUDA device")
    import verbo_b200 as vb
    from verbo_b200.serving import BatchServer

    g = np.random.default_rng(77)
    srv = BatchServer(vb.Sampling(), slots=4, vocab=V, model=stand_in_model, stop_ids=STOP)
    reqs = []
    for i in range(9):
        opts = MIXED[i % 3]
        prompt = g.integers(0, V, size=int(g.integers(0, 60))).tolist()
        rid = srv.submit(prompt, max_tokens=int(g.integers(2, 9)), seed=500 + i, opts=vb.Sampling(**opts))
        reqs.append((rid, prompt, opts))
    done = srv.run()
    assert sorted(done) == [rid for rid, _, _ in reqs]
    replay(done, reqs)


def replay(done, reqs):
    """Each request on the oracle as generate would run it alone; returns how
    many ended on a stop id."""
    stopped = 0
    for rid, prompt, opts in reqs:
        o = po.sampling(**opts)
        r = done[rid]
        st = po.seed_states(np.array([r.seed], dtype=np.uint64))
        hist = list(prompt)
        picks = list(r.tokens) + ([None] if r.stopped else [])
        for t, got in enumerate(picks):
            h = np.array(hist, dtype=np.int32)
            ids, ost = po.sample_rows(model_row(rid, t)[None], o, st, h, np.array([0, len(h)], dtype=np.int64))
            want = int(ids[0])
            if got is None:  # the request ended on a stop id
                assert want in STOP, (rid, t, want)
                break
            if got != want:
                margin = min(float(ost["draw_margin"][0]), float(ost["cut_margin"][0]))
                assert margin < 1e-6, (rid, t, got, want, margin)
            assert got not in STOP
            hist.append(got)
        else:
            assert len(r.tokens) == r.max_tokens, (rid, len(r.tokens))
        stopped += r.stopped
    return stopped
