"""The decode-loop fixture (tests/golden/decode_models.npz) against the oracle.

Each case holds B concurrent generations, each an independent verbo::generate
run of the reference (src/sampler.cpp:111-181) on one of its tiny checkpoints,
with every pick's id and the hidden row its logits came from.  Stepping the B
generations together through the oracle's logits tail (the reference's final
rmsnorm + head, scalar build) and the oracle's Sampler::pick - histories of
prompt + accepted ids, one RNG state per generation seeded as Sampler(cfg) -
must give exactly the reference's ids.  This pins the composition that
verbo_cuda_batch_decode runs on the device.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import pyoracle as po
from tests.decode_fixture import load_cases

CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_steps_reproduce_reference_generations(case):
    assert case.B >= 2
    o = po.sampling(**case.opts)
    states = po.seed_states(case.seeds)
    hist = [list(p) for p in case.prompts]
    for j in range(case.steps):
        act = [b for b in range(case.B) if j < case.npicks[b]]
        logits, _, _ = po.logits_tail(case.head_dtype, case.q, case.s, case.norm, case.eps, case.x[act, j])
        h = np.concatenate([np.array(hist[b], dtype=np.int32) for b in act])
        off = np.cumsum([0] + [len(hist[b]) for b in act]).astype(np.int64)
        st = np.ascontiguousarray(states[act])
        ids, _ = po.sample_rows(logits, o, st, h, off)
        states[act] = st
        assert ids.tolist() == case.ids[act, j].tolist(), (case.name, j)
        for b, i in zip(act, ids.tolist()):
            hist[b].append(i)
    # the fixture covers stops and full-length generations
    assert (case.npicks >= 1).all()


def test_fixture_spans_the_sampling_modes():
    names = {c.name for c in CASES}
    kinds = {("greedy" if c.opts["temp"] <= 0 else "topk" if 0 < c.opts["top_k"] < 400 else "full") for c in CASES}
    assert kinds == {"greedy", "topk", "full"}, names
    assert any(c.stopped.any() for c in CASES)
    assert {c.head_dtype for c in CASES} >= {"f32", "q8"}
