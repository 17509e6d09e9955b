"""Pins the C oracle (oracle/sampler_oracle.c) before it is trusted as the checker.

1. The reference's own known-answer tests for the sampler
   (tests/test_core.cpp:454-496), restated against the oracle.
2. The golden fixtures made by running the reference's compiled Sampler.
3. A live cross-check against that compiled Sampler (oracle/_ref), when it
   was built in this checkout.
4. The vocab-sharded decomposition: merging per-shard top-k candidates gives
   the unsharded pick.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import pyoracle as po
from tests import golden_io
from verbo_b200 import workloads as wl

LG = np.array([[0.1, 3.0, 2.9, -1.0, 0.0]], dtype=np.float32)


def picks(opts, seed, n, logits=LG):
    st = po.seed_states(np.array([seed], dtype=np.uint64))
    return np.array([po.sample_rows(logits, opts, st)[0][0] for _ in range(n)])


def test_kat_greedy():
    # test_core.cpp:457-458
    ids, _ = po.sample_rows(LG, po.sampling(temp=0.0))
    assert ids[0] == 1


def test_kat_topk2_seeded_statistics():
    # test_core.cpp:459-470: two samplers agree, ids in {1,2}, 150 < #1 < 300
    o = po.sampling(seed=42, top_k=2, top_p=1.0)
    a = picks(o, 42, 400)
    b = picks(o, 42, 400)
    assert np.array_equal(a, b)
    assert set(a.tolist()) <= {1, 2}
    assert 150 < int((a == 1).sum()) < 300


def test_kat_top_p_half():
    # test_core.cpp:472-477
    assert (picks(po.sampling(seed=1, top_k=0, top_p=0.5), 1, 100) == 1).all()


def test_kat_min_p():
    # test_core.cpp:478-487
    ids = picks(po.sampling(seed=1, top_k=0, top_p=1.0, min_p=0.5), 1, 100)
    assert set(ids.tolist()) <= {1, 2}


def test_kat_repeat_penalty():
    # test_core.cpp:488-495: accept(1) then greedy with repeat 2 -> 2; reset -> 1
    o = po.sampling(temp=0.0, repeat=2.0)
    ids, _ = po.sample_rows(LG, o, hist=np.array([1], np.int32), hist_off=np.array([0, 1], np.int64))
    assert ids[0] == 2
    ids, _ = po.sample_rows(LG, o)
    assert ids[0] == 1


def test_rng_stream_known_values():
    # splitmix64 + xoroshiro128+ (sampler.cpp:11-41) for seed 42: first uniforms.
    st = po.seed_states(np.array([42], dtype=np.uint64))
    lib = po.oracle_lib()
    u = [lib.oracle_unit(st[0].ctypes.data) for _ in range(3)]
    assert all(0.0 <= x < 1.0 for x in u)
    st2 = po.seed_states(np.array([42], dtype=np.uint64))
    assert [lib.oracle_unit(st2[0].ctypes.data) for _ in range(3)] == u


@pytest.mark.parametrize("case", golden_io.small_cases(), ids=lambda c: c.name)
def test_oracle_matches_golden_small(case):
    st = po.seed_states(case.seeds)
    steps = case.ids.shape[1]
    got = np.stack([po.sample_rows(case.logits, po.sampling(**case.opts), st, case.hist, case.off)[0]
                    for _ in range(steps)], axis=1)
    assert np.array_equal(got, case.ids)


def test_oracle_matches_golden_configs():
    for w, x, h, off, seeds, ids in golden_io.config_cases():
        st = po.seed_states(seeds)
        got = np.stack([po.sample_rows(x, po.sampling(**w.sampling_kwargs()), st, h, off)[0]
                        for _ in range(ids.shape[1])], axis=1)
        assert np.array_equal(got, ids), w.name


@pytest.mark.skipif(not po.ref_available(), reason="reference harness not built in this checkout")
@pytest.mark.parametrize("seed", [3, 11])
def test_oracle_matches_reference_live(seed):
    g = np.random.default_rng(seed)
    for V in (7, 64, 999, 5000):
        x = (g.standard_normal((6, V)) * g.uniform(0.2, 5)).astype(np.float32)
        x[:, g.integers(0, V, size=V // 5)] = np.round(x[:, :1], 1)  # ties
        h = g.integers(-3, V + 3, size=6 * 9).astype(np.int32)
        off = np.arange(7, dtype=np.int64) * 9
        for opts in (dict(temp=0.0, repeat=1.4), dict(temp=0.9, top_k=3, top_p=0.8, min_p=0.1, repeat=1.2, repeat_last=4),
                     dict(temp=1.3, top_k=0, top_p=0.7), dict(temp=0.4, top_k=V, top_p=0.99, min_p=0.02)):
            o = po.sampling(**opts)
            seeds = np.arange(6, dtype=np.uint64) + np.uint64(100 * seed + 1)
            ref = po.ref_sample_rows(x, o, seeds, h, off, steps=4)
            st = po.seed_states(seeds)
            got = np.stack([po.sample_rows(x, o, st, h, off)[0] for _ in range(4)], axis=1)
            assert np.array_equal(got, ref), (V, opts)


@pytest.mark.parametrize("name", ["c5", "c3"])
def test_shard_merge_equals_unsharded(name):
    w = wl.WORKLOADS[name].with_rows(5)
    x = wl.make_rows_np(w)
    h, off = wl.make_hist_np(w)
    o = po.sampling(**w.sampling_kwargs())
    shards = 8
    cols = w.vocab // shards
    k = 64
    vals, ids = [], []
    for s in range(shards):
        v, i = po.shard_topk(x[:, s * cols:(s + 1) * cols], s * cols, w.vocab, o, k, h, off)
        vals.append(v)
        ids.append(i)
    seeds = w.sampler_seeds(0, 5)
    st_a, st_b = po.seed_states(seeds), po.seed_states(seeds)
    merged, _ = po.merge_sample(np.stack(vals), np.stack(ids), w.vocab, o, st_a)
    direct, _ = po.sample_rows(x, o, st_b, h, off)
    assert np.array_equal(merged, direct)
