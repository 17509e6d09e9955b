"""Batched generation streams (verbo_cuda_batch_*) against the oracle.

The reference's generate loop (src/sampler.cpp:111-181) keeps one Sampler per
generation: accept() the prompt, then pick() and accept() each token.  Here
B streams share one device step.  The oracle replays each stream as its own
Sampler over the same logits, with the history the stream really has (its
prompt plus the ids the GPU sampled so far), so every step is judged on its
own: ids equal except where the oracle's uniform or cutoff is within the
boundary margin.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import pyoracle as po
from tests.gpu_util import compare, stats_np

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def vb(cuda_lib):
    if not torch.cuda.is_available():
        pytest.fail("gpu tests need a CUDA device")
    import verbo_b200

    return verbo_b200


CASES = [
    (151936, dict(temp=0.0, repeat=1.3, repeat_last=64)),                          # split greedy
    (151936, dict(temp=0.8, top_k=50, top_p=0.95, repeat=1.1, repeat_last=64)),    # split top-k
    (49152, dict(temp=1.2, top_k=0, top_p=0.9, repeat=1.2, repeat_last=37)),       # full vocabulary
    (1000, dict(temp=0.7, top_k=40, top_p=1.0, min_p=0.05, repeat=0.8, repeat_last=5)),
    (8192, dict(temp=0.9, top_k=20, top_p=0.9)),                                   # no penalty, no windows
]


def _csr(hist):
    off = np.zeros(len(hist) + 1, dtype=np.int64)
    off[1:] = np.cumsum([len(h) for h in hist])
    flat = np.concatenate([np.asarray(h, dtype=np.int32) for h in hist]) if off[-1] else np.zeros(0, np.int32)
    return flat, off


@pytest.mark.parametrize("V,opts", CASES, ids=["greedy", "topk", "full-vocab", "min-p", "no-penalty"])
def test_batch_matches_sequential_samplers(vb, V, opts):
    g = np.random.default_rng([V, len(opts)])
    B, T = 5, 6
    seeds = np.array([11, 22, 33, 44, 55], dtype=np.uint64) + np.uint64(V)
    prompts = [g.integers(-2, V + 2, size=L).tolist() for L in (0, 3, 64, 300, 1)]  # wider than the windows
    b = vb.Batch(vb.Sampling(**opts), B)
    for i in range(B):
        b.reset(i, int(seeds[i]))
        b.accept(i, prompts[i])
    hist = [list(p) for p in prompts]
    states = po.seed_states(seeds)
    o = po.sampling(**opts)
    stats = torch.zeros(B * vb.ROW_STATS_BYTES, dtype=torch.uint8, device="cuda")
    for t in range(T):
        if t == 3:  # a new request takes slot 2
            b.reset(2, 777)
            prompts2 = g.integers(0, V, size=9).tolist()
            b.accept(2, prompts2)
            states[2] = po.seed_states(np.array([777], dtype=np.uint64))[0]
            hist[2] = list(prompts2)
        x = (g.standard_normal((B, V)) * 2.0).astype(np.float32)
        x[1, g.integers(0, V, size=V // 20)] = x[1].max()  # ties at the top of row 1
        if hist[0]:
            x[0, [h for h in hist[0] if 0 <= h < V]] += 3.0  # make the penalty decide
        ids = b.step(torch.from_numpy(x).cuda(), stats=stats).cpu().numpy()
        h, off = _csr(hist)
        ora, ost = po.sample_rows(x, o, states, h, off)
        compare(ids[:, None], ora[:, None], ost[:, None], f"step {t} {opts}")
        if opts["temp"] > 0:
            np.testing.assert_allclose(stats_np(stats)["sum"], ost["sum"], rtol=1e-5)
        for i in range(B):
            hist[i].append(int(ids[i]))
    vb.check()


def test_batch_steps_replay_in_a_cuda_graph(vb):
    # A decode loop captures its step once: the rings and RNG states advance
    # on the device, replay after replay, exactly as eager steps do.
    V, B = 151936, 8
    opts = dict(temp=0.8, top_k=50, top_p=0.95, repeat=1.1, repeat_last=64)
    g = np.random.default_rng(5)
    x = torch.from_numpy((g.standard_normal((B, V)) * 2).astype(np.float32)).cuda()
    eager, graphed = vb.Batch(vb.Sampling(**opts), B), vb.Batch(vb.Sampling(**opts), B)
    for i in range(B):
        for bb in (eager, graphed):
            bb.reset(i, 100 + i)
            bb.accept(i, [i, 2 * i])
    want = [eager.step(x).cpu().numpy() for _ in range(5)]
    out = torch.empty(B, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        graphed.step(x, out=out, cuda_stream=s)  # warm-up: scratch and launch state exist before capture
    s.synchronize()
    got = [out.cpu().numpy().copy()]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        graphed.step(x, out=out, cuda_stream=s)
    for _ in range(4):
        graph.replay()
        torch.cuda.synchronize()
        got.append(out.cpu().numpy().copy())
    assert all(np.array_equal(a, w) for a, w in zip(got, want))
