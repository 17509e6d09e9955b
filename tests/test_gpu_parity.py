"""Parity of the CUDA sampler with the oracle and the reference's golden ids.

Every test calls the CUDA library through its C ABI (via verbo_b200's ctypes
binding) on device-resident rows and compares with the C oracle, which
tests/test_oracle.py pins against the reference's compiled Sampler.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import pyoracle as po
from tests import golden_io
from tests.gpu_util import compare, run_gpu, run_oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

LG = np.array([[0.1, 3.0, 2.9, -1.0, 0.0]], dtype=np.float32)


@pytest.fixture(scope="module", autouse=True)
def _lib(cuda_lib):
    if not torch.cuda.is_available():
        pytest.fail("gpu tests need a CUDA device")
    yield


# ------------------------------------------------ reference known answers ----
def test_kat_greedy():
    ids, _, _ = run_gpu(LG, dict(temp=0.0))
    assert ids[0, 0] == 1


def test_kat_topk2_400_draws():
    # tests/test_core.cpp:459-470 with the rng advancing in place on the device
    seeds = np.array([42], dtype=np.uint64)
    opts = dict(temp=0.7, top_k=2, top_p=1.0)
    ids, _, _ = run_gpu(LG, opts, seeds, steps=400)
    ora, _, _ = run_oracle(LG, opts, seeds, steps=400)
    assert np.array_equal(ids, ora)
    assert 150 < int((ids == 1).sum()) < 300


def test_kat_top_p_and_min_p():
    ids, _, _ = run_gpu(LG, dict(temp=0.7, top_k=0, top_p=0.5), np.array([1], np.uint64), steps=100)
    assert (ids == 1).all()
    ids, _, _ = run_gpu(LG, dict(temp=0.7, top_k=0, top_p=1.0, min_p=0.5), np.array([1], np.uint64), steps=100)
    assert set(ids.ravel().tolist()) <= {1, 2}
    ora, _, _ = run_oracle(LG, dict(temp=0.7, top_k=0, top_p=1.0, min_p=0.5), np.array([1], np.uint64), steps=100)
    assert np.array_equal(ids, ora)


def test_kat_repeat_penalty():
    h, off = np.array([1], np.int32), np.array([0, 1], np.int64)
    ids, _, _ = run_gpu(LG, dict(temp=0.0, repeat=2.0), hist=h, off=off)
    assert ids[0, 0] == 2
    ids, _, _ = run_gpu(LG, dict(temp=0.0, repeat=2.0))
    assert ids[0, 0] == 1


def test_sampler_object_kat():
    # the verbo::Sampler interface: host and device logits, accept, reset
    import verbo_b200 as vb

    s = vb.Sampler(vb.Sampling(temp=0.0, repeat=2.0))
    assert s.pick(LG[0]) == 1
    s.accept(1)
    assert s.pick(LG[0]) == 2
    assert s.pick(torch.from_numpy(LG[0]).cuda()) == 2
    s.reset()
    assert s.pick(LG[0]) == 1
    assert s.cfg().repeat == 2.0
    a, b = vb.Sampler(vb.Sampling(seed=42, top_k=2, top_p=1.0)), vb.Sampler(vb.Sampling(seed=42, top_k=2, top_p=1.0))
    xs = [a.pick(LG[0]) for _ in range(100)]
    assert xs == [b.pick(LG[0]) for _ in range(100)]
    ora, _, _ = run_oracle(LG, dict(temp=0.7, top_k=2, top_p=1.0), np.array([42], np.uint64), steps=100)
    assert xs == ora[0].tolist()


# -------------------------------------------------------- golden fixtures ----
@pytest.mark.parametrize("case", golden_io.small_cases(), ids=lambda c: c.name)
def test_golden_small(case):
    steps = case.ids.shape[1]
    ids, _, _ = run_gpu(case.logits, case.opts, case.seeds, case.hist, case.off, steps=steps)
    _, ostats, _ = run_oracle(case.logits, case.opts, case.seeds, case.hist, case.off, steps=steps)
    compare(ids, case.ids, ostats, case.name)


def test_golden_configs():
    for w, x, h, off, seeds, ref_ids in golden_io.config_cases():
        ids, _, _ = run_gpu(x, w.sampling_kwargs(), seeds, h, off, steps=ref_ids.shape[1])
        _, ostats, _ = run_oracle(x, w.sampling_kwargs(), seeds, h, off, steps=ref_ids.shape[1])
        compare(ids, ref_ids, ostats, w.name)


# ---------------------------------------------------- randomized coverage ----
OPTION_SETS = [
    dict(temp=0.0, repeat=1.3, repeat_last=16),                                   # greedy
    dict(temp=0.7, top_k=40, top_p=0.9, min_p=0.05, repeat=1.1, repeat_last=64),  # streaming top-k
    dict(temp=1.2, top_k=1, top_p=0.9),                                           # top-1
    dict(temp=0.9, top_k=700, top_p=0.97, min_p=0.0, repeat=1.2),                 # large k, streaming kernel
    dict(temp=1.5, top_k=0, top_p=0.99),                                          # full-vocab nucleus
    dict(temp=1.0, top_k=0, top_p=1.0, min_p=0.1, repeat=0.9, repeat_last=0),     # full vocab, min-p only
    dict(temp=0.6, top_k=3000, top_p=0.8, min_p=0.0),                             # k above the streaming range
]


@pytest.mark.parametrize("V", [5, 33, 400, 1001, 8192, 8193, 49152, 151936, 262144])
@pytest.mark.parametrize("oi", range(len(OPTION_SETS)))
def test_random_parity(V, oi):
    opts = OPTION_SETS[oi]
    g = np.random.default_rng([V, oi])
    rows = 6 if V < 100000 else 3
    x = (g.standard_normal((rows, V)) * g.uniform(0.3, 4.0)).astype(np.float32)
    x[0, g.integers(0, V, size=max(1, V // 10))] = x[0, 0]                     # ties in row 0
    H = 37
    hist = g.integers(-2, V + 2, size=rows * H).astype(np.int32)
    off = np.arange(rows + 1, dtype=np.int64) * H
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(V * 31 + oi + 1)
    ids, st, _ = run_gpu(x, opts, seeds, hist, off, steps=2)
    ora, ost, _ = run_oracle(x, opts, seeds, hist, off, steps=2)
    compare(ids, ora, ost, f"V={V} opts={opts}")
    if opts["temp"] > 0:
        # probabilities: softmax normaliser and kept mass of the last pick
        o = ost[:, -1]
        np.testing.assert_allclose(st["sum"], o["sum"], rtol=1e-5)
        same = ids[:, -1] == ora[:, -1]
        np.testing.assert_allclose(st["tot"][same], o["tot"][same], rtol=1e-5)
        assert np.array_equal(st["keep"][same], o["keep"][same]) or (st["keep"][same] - o["keep"][same] != 0).sum() <= 1


def test_unaligned_leading_dimension():
    g = np.random.default_rng(7)
    for V, ld in ((1000, 1003), (4099, 4101), (151936, 151939)):
        x = g.standard_normal((4, V)).astype(np.float32)
        for opts in (dict(temp=0.0, repeat=1.2), dict(temp=0.8, top_k=50, top_p=0.95), dict(temp=1.1, top_k=0, top_p=0.9)):
            hist = g.integers(0, V, size=4 * 10).astype(np.int32)
            off = np.arange(5, dtype=np.int64) * 10
            seeds = np.arange(4, dtype=np.uint64) + np.uint64(77)
            ids, _, _ = run_gpu(x, opts, seeds, hist, off, ld=ld)
            ora, ost, _ = run_oracle(x, opts, seeds, hist, off)
            compare(ids, ora, ost, f"V={V} ld={ld}")


def test_nonfinite_rows():
    V = 3000
    g = np.random.default_rng(3)
    x = g.standard_normal((5, V)).astype(np.float32)
    x[0, :] = -np.inf                        # fully masked row
    x[1, [5, 900]] = np.inf                  # +inf logits
    x[2, : V - 3] = -np.inf                  # three finite values
    x[3, ::2] = -np.inf                      # half masked
    x[4, 17] = np.inf
    x[4, 2000] = np.inf
    for opts in (dict(temp=0.0), dict(temp=0.7, top_k=40, top_p=0.9), dict(temp=0.7, top_k=40, top_p=0.9, min_p=0.1),
                 dict(temp=1.0, top_k=0, top_p=0.9), dict(temp=1.0, top_k=0, top_p=0.95, min_p=0.2),
                 dict(temp=1.0, top_k=2000, top_p=1.0)):
        seeds = np.arange(5, dtype=np.uint64) + np.uint64(5)
        ids, _, _ = run_gpu(x, opts, seeds, steps=2)
        ora, ost, _ = run_oracle(x, opts, seeds, steps=2)
        compare(ids, ora, ost, str(opts))


def test_greedy_nan_first_element():
    # std::max_element keeps a NaN element 0 (nothing compares greater)
    x = np.array([[np.nan, 1.0, 5.0, 2.0], [1.0, np.nan, 5.0, 5.0]], dtype=np.float32)
    ids, _, _ = run_gpu(x, dict(temp=0.0))
    ora, _, _ = run_oracle(x, dict(temp=0.0))
    assert ids[:, 0].tolist() == ora[:, 0].tolist() == [0, 2]
    # ... also when element 0 (or the maximum) is in the penalty window, for
    # short rows and for rows long enough for several slices
    for V in (16, 151936):
        g = np.random.default_rng(V)
        x = (g.standard_normal((4, V)) * 2).astype(np.float32)
        x[0, 0] = np.nan
        x[1, 0] = np.nan
        x[2, 7] = 40.0
        x[3, 0] = 40.0
        hist = np.array([0, 3, 0, 1, 7, 2, 0, 2], dtype=np.int32)
        off = np.array([0, 2, 4, 6, 8], dtype=np.int64)
        for opts in (dict(temp=0.0, repeat=1.5, repeat_last=8), dict(temp=0.0, repeat=0.5, repeat_last=2)):
            ids, _, _ = run_gpu(x, opts, hist=hist, off=off)
            ora, _, _ = run_oracle(x, opts, hist=hist, off=off)
            assert ids[:, 0].tolist() == ora[:, 0].tolist(), (V, opts)


def test_history_windows():
    V = 9000
    g = np.random.default_rng(11)
    x = (g.standard_normal((4, V)) * 2).astype(np.float32)
    top = np.argsort(-x, axis=1)[:, :6]
    # histories made of each row's best ids, with duplicates and ragged lengths
    parts = [np.repeat(top[r], r + 1).astype(np.int32) for r in range(4)]
    hist = np.concatenate(parts)
    off = np.concatenate([[0], np.cumsum([len(p) for p in parts])]).astype(np.int64)
    for rl in (0, 1, 3, 64):
        for opts in (dict(temp=0.0, repeat=3.0, repeat_last=rl), dict(temp=0.5, top_k=20, top_p=0.9, repeat=3.0, repeat_last=rl)):
            seeds = np.arange(4, dtype=np.uint64) + np.uint64(rl + 9)
            ids, _, _ = run_gpu(x, opts, seeds, hist, off, steps=3)
            ora, ost, _ = run_oracle(x, opts, seeds, hist, off, steps=3)
            compare(ids, ora, ost, str(opts))


# ------------------------------------------------------------- sharded path ----
@pytest.mark.parametrize("nshards", [1, 2, 8])
def test_shard_topk_and_merge(nshards):
    import verbo_b200 as vb
    from verbo_b200 import workloads as wl

    w = wl.WORKLOADS["c5"].with_rows(24)
    x = wl.make_rows_np(w)
    h, off = wl.make_hist_np(w)
    opts = w.sampling_kwargs()
    o = vb.Sampling(**opts)
    k = 64
    cols = w.vocab // nshards
    dx = torch.from_numpy(x).cuda()
    dh, do = torch.from_numpy(h).cuda(), torch.from_numpy(off).cuda()
    cv = torch.empty(nshards, w.rows, k, dtype=torch.float32, device="cuda")
    ci = torch.empty(nshards, w.rows, k, dtype=torch.int32, device="cuda")
    for s in range(nshards):
        vb.shard_topk(dx[:, s * cols:(s + 1) * cols], s * cols, w.vocab, o, k, dh, do, cand_val=cv[s], cand_id=ci[s])
        ov, oi = po.shard_topk(x[:, s * cols:(s + 1) * cols], s * cols, w.vocab, po.sampling(**opts), k, h, off)
        assert np.array_equal(ci[s].cpu().numpy(), oi)
        assert np.array_equal(cv[s].cpu().numpy(), ov)
    seeds = w.sampler_seeds(0, w.rows)
    from tests.gpu_util import to_dev_rng
    rng = to_dev_rng(po.seed_states(seeds))
    got = vb.merge_sample(cv, ci, w.vocab, o, rng=rng).cpu().numpy()
    vb.check()
    ora, ost, _ = run_oracle(x, opts, seeds, h, off)
    compare(got[:, None], ora, ost, f"merge nshards={nshards}")
    # greedy through the sharded path
    g = vb.merge_sample(cv, ci, w.vocab, vb.Sampling(temp=0.0)).cpu().numpy()
    assert np.array_equal(g, run_oracle(x, dict(temp=0.0, repeat=opts["repeat"], repeat_last=opts["repeat_last"]),
                                        None, h, off)[0][:, 0])


def test_shard_topk_small_shards_pad():
    import verbo_b200 as vb

    g = np.random.default_rng(5)
    x = g.standard_normal((3, 50)).astype(np.float32)
    cv, ci = vb.shard_topk(torch.from_numpy(x).cuda(), 100, 1000, vb.Sampling(), 64)
    ov, oi = po.shard_topk(x, 100, 1000, po.sampling(), 64)
    assert np.array_equal(ci.cpu().numpy(), oi)
    assert (ci.cpu().numpy()[:, 50:] == -1).all()


@pytest.mark.parametrize("form", ["sorted", "shuffled", "holes", "duplicates"])
@pytest.mark.parametrize("nshards,k", [(1, 64), (3, 50), (16, 256), (16, 1), (2, 256)])
def test_merge_candidate_lists(form, nshards, k):
    # merge_sample on lists made directly: in step 1's order (the merge of
    # sorted lists), shuffled, with missing slots between real ones, and with
    # the same candidate in two shards; 16 x 256 is the largest merge
    import verbo_b200 as vb
    from tests.gpu_util import to_dev_rng

    g = np.random.default_rng(nshards * 1000 + k)
    rows, vocab = 6, 200000
    ids = np.stack([g.choice(vocab, size=(nshards, k), replace=False) for _ in range(rows)], axis=1)
    val = g.standard_normal((nshards, rows, k)).astype(np.float32) * 2
    val[:, 0, : k // 2] = 1.25                     # ties broken by id
    ids = ids.astype(np.int32)
    if form == "duplicates" and nshards > 1:
        ids[1, :, :5], val[1, :, :5] = ids[0, :, :5], val[0, :, :5]
    for s in range(nshards):
        for r in range(rows):
            o = np.lexsort((ids[s, r], -val[s, r]))
            ids[s, r], val[s, r] = ids[s, r][o], val[s, r][o]
    if form == "holes":
        ids[:, :, 1::3] = -1
        val[:, :, 1::3] = -np.inf
    elif form == "shuffled":
        for s in range(nshards):
            for r in range(rows):
                p = g.permutation(k)
                ids[s, r], val[s, r] = ids[s, r][p], val[s, r][p]
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(17)
    dv, di = torch.from_numpy(val).cuda(), torch.from_numpy(ids).cuda()
    for opts in (dict(temp=0.8, top_k=k, top_p=0.9, min_p=0.02), dict(temp=1.1, top_k=min(k, 40), top_p=1.0),
                 dict(temp=0.0)):
        st = po.seed_states(seeds)
        rng = to_dev_rng(st)
        got = vb.merge_sample(dv, di, vocab, vb.Sampling(**opts), rng=rng).cpu().numpy()
        vb.check()
        ora, ost = po.merge_sample(val, ids, vocab, po.sampling(**opts), st)
        compare(got[:, None], ora[:, None], ost[:, None], f"{form} {nshards}x{k} {opts}")


def test_min_p_extremes_keep_first():
    # keep starts at 1 (src/sampler.cpp:89): min_p >= 1 keeps the maximum (and its ties)
    g = np.random.default_rng(21)
    V = 5000
    x = g.standard_normal((4, V)).astype(np.float32)
    x[1, [10, 20, 30]] = x[1].max() + 1.0          # tied maxima
    for top_k in (0, 40, 600):
        for mp in (1.0, 1.5, 0.999):
            opts = dict(temp=0.9, top_k=top_k, top_p=0.9, min_p=mp)
            seeds = np.arange(4, dtype=np.uint64) + np.uint64(3)
            ids, _, _ = run_gpu(x, opts, seeds, steps=3)
            ora, ost, _ = run_oracle(x, opts, seeds, steps=3)
            compare(ids, ora, ost, str(opts))


def test_crowded_bins_use_exact_fallback():
    # rows whose values pile into a few value bins: the nucleus kernel's
    # gather overflows and the exact radix selection takes over
    g = np.random.default_rng(8)
    V = 151936
    x = np.round(g.standard_normal((3, V)) * 2).astype(np.float32) / 4   # ~30 distinct values
    x[2] = 0.75
    for opts in (dict(temp=1.0, top_k=0, top_p=0.9), dict(temp=0.7, top_k=0, top_p=1.0, min_p=0.3),
                 dict(temp=2.0, top_k=0, top_p=0.5)):
        seeds = np.arange(3, dtype=np.uint64) + np.uint64(40)
        ids, st, _ = run_gpu(x, opts, seeds, steps=2)
        ora, ost, _ = run_oracle(x, opts, seeds, steps=2)
        compare(ids, ora, ost, str(opts))
        np.testing.assert_allclose(st["sum"], ost[:, -1]["sum"], rtol=1e-9)


@pytest.mark.parametrize("temp", [0.05, 0.4, 1.0, 1.5, 6.0])
def test_full_vocab_weights_match_reference_sums(temp):
    # The reference sums glibc exp() values one by one in sorted order, whose
    # own rounding is bounded by about N * eps = 151936 * 2^-53 = 1.7e-11
    # relative.  Two kernels compute the normaliser, each with its own bound:
    #  * the streaming kernel (top_k 0, top-p and / or min-p, no penalty;
    #    nucleus.cu) sums per-cell masses exp(-j 2^-K) (1 + e(r)) with e(r) in
    #    fp32 and fixed point: within 4e-9 relative (its kDelta), about 1e-9
    #    when the cells are at their widest (2^-6, temp 0.05 over N(0, 3^2)
    #    below);
    #  * the staged cluster kernel (top_k above 256 and below the vocabulary
    #    here) sums fixed-point masses of a table-driven fp64 exponential:
    #    within 5e-11.
    # Both far inside the 1e-5 of the parity criteria; an error in either
    # exponential would show at 1e-3.  The ranges go from nearly all-underflow
    # (temp 0.05 over N(0, 3^2)) to a narrow band (temp 6).  Sampled ids agree
    # away from boundaries.
    g = np.random.default_rng(int(temp * 100))
    V = 151936
    x = np.stack([g.standard_normal(V) * 3, g.standard_normal(V) * 0.5, g.uniform(-20, 0, V)]).astype(np.float32)
    seeds = np.arange(3, dtype=np.uint64) + np.uint64(4000 + int(temp * 100))
    for opts, rtol in ((dict(temp=temp, top_k=0, top_p=0.99), 4e-9),
                       (dict(temp=temp, top_k=0, top_p=1.0, min_p=0.01), 4e-9),
                       (dict(temp=temp, top_k=0, top_p=0.9, min_p=0.05), 4e-9),
                       (dict(temp=temp, top_k=100000, top_p=1.0, min_p=0.01), 5e-11)):
        ids, st, _ = run_gpu(x, opts, seeds, steps=2)
        ora, ost, _ = run_oracle(x, opts, seeds, steps=2)
        compare(ids, ora, ost, f"temp={temp} {opts}")
        np.testing.assert_allclose(st["sum"], ost[:, -1]["sum"], rtol=rtol)


@pytest.mark.parametrize("k", [32, 50, 64, 100, 128, 200, 256])
def test_topk_concentrated_in_few_slices(k):
    # For 32 <= k <= 256 a slice emits only its top-m (m = max(16,
    # ceil(k / 14), ceil(k / 4)) at V = 151936: 15 slices) and the merge
    # checks each slice's threshold against the k-th value found.  Rows whose
    # k best sit in one or two slices (slices are 10240 columns) fail that
    # check for those slices, which the merge then resolves exactly; the ids
    # must not notice.
    g = np.random.default_rng(k + 7)
    V, S = 151936, 10240
    x = g.standard_normal((6, V)).astype(np.float32)
    x[0, :S] += 6.0                                   # all in slice 0
    x[1, V - 3000:] += 6.0                            # all in the last (short) slice
    x[2, 3 * S:4 * S] += 6.0
    x[2, 9 * S:10 * S] += 6.0                         # split over two slices
    x[3] = np.sort(x[3])                              # ascending: the k best at the end
    x[4, S:S + 40] = 9.0                              # a block of equal values across the k-th
    # row 5: no concentration
    hist = np.concatenate([g.integers(0, S, size=48), g.integers(V - 3000, V, size=48)] * 6).astype(np.int32)
    off = np.arange(7, dtype=np.int64) * 96
    seeds = np.arange(6, dtype=np.uint64) + np.uint64(700 + k)
    for opts in (dict(temp=0.8, top_k=k, top_p=0.95, repeat=1.2, repeat_last=64),
                 dict(temp=1.0, top_k=k, top_p=1.0, min_p=0.01, repeat=1.3, repeat_last=0),  # whole history (CSR)
                 dict(temp=0.7, top_k=k, top_p=0.9)):
        ids, st, _ = run_gpu(x, opts, seeds, hist, off, steps=2)
        ora, ost, _ = run_oracle(x, opts, seeds, hist, off, steps=2)
        compare(ids, ora, ost, f"k={k} {opts}")
        np.testing.assert_allclose(st["sum"], ost[:, -1]["sum"], rtol=1e-9)
        assert np.array_equal(st["k"], ost[:, -1]["k"])


@pytest.mark.parametrize("k", [1, 2, 31, 33, 50, 64, 128, 255, 256])
def test_split_topk_bounds(k):
    # The split top-k kernels bound each slice (and then the union) by the
    # q-th largest lane maximum of every full warp; rows with ties at the
    # bound, coarse values (the exact fallbacks), a short last slice and
    # masked stretches must still give the reference's top-k.
    g = np.random.default_rng(k)
    V = 151936
    x = (g.standard_normal((5, V)) * 2).astype(np.float32)
    x[1] = np.round(x[1] * 2) / 4                       # ~40 distinct values: every slice overflows
    x[2, g.integers(0, V, size=3000)] = x[2].max()      # many ties at the top
    x[3, : V - 5000] = -np.inf                          # only the last slices hold finite values
    x[4, ::3] = -np.inf
    hist = g.integers(0, V, size=5 * 64).astype(np.int32)
    off = np.arange(6, dtype=np.int64) * 64
    seeds = np.arange(5, dtype=np.uint64) + np.uint64(900 + k)
    for opts in (dict(temp=0.8, top_k=k, top_p=0.95, repeat=1.1), dict(temp=1.3, top_k=k, top_p=1.0, min_p=0.02)):
        ids, st, _ = run_gpu(x, opts, seeds, hist, off, steps=2)
        ora, ost, _ = run_oracle(x, opts, seeds, hist, off, steps=2)
        compare(ids, ora, ost, f"k={k} {opts}")
        assert np.array_equal(st["k"], ost[:, -1]["k"])
        np.testing.assert_allclose(st["sum"], ost[:, -1]["sum"], rtol=1e-9)


def test_cpp_header_known_answers(tmp_path):
    from tests.test_capi import _build_hpp_kat

    exe = _build_hpp_kat(tmp_path)
    import subprocess

    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
