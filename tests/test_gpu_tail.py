"""The CUDA logits tail (verbo_cuda_tail_*) against the oracle, bit for bit.

The oracle restates the reference's scalar build and reproduces the reference
Session's logits on its tiny checkpoints (tests/test_tail_oracle.py), so the
bar here is exact equality of every logit:
* the golden fixture's hidden rows -> the reference session's logits;
* seeded heads of every dtype over shapes that reach every token tile (8, 16,
  32, 64 and several 64-tiles), partial K chunks (dim not a multiple of 128),
  ragged vocab tiles and strided rows;
* the full Qwen2 vocabulary (151936 x 896): a few rows against the oracle,
  and 256 rows through size-independent properties (each row equals the same
  row computed alone; a slice of vocab ids equals the oracle on that slice of
  the head);
* the logits feed the sampler unchanged (greedy ids from the device tail
  equal the oracle's on the reference logits).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import pyoracle as po

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

GOLDEN = Path(__file__).resolve().parent / "golden" / "tail_models.npz"


def need_gpu():
    if not torch.cuda.is_available():
        pytest.fail("gpu tests need a CUDA device")


def run_tail(vb, dtype, q, s, norm, eps, x, ldx=None, ld=None):
    t = vb.Tail(dtype, q, s, norm, eps)
    n, dim = x.shape
    ldx = dim if ldx is None else ldx
    xd = torch.zeros(n, ldx, dtype=torch.float32, device="cuda")
    xd[:, :dim] = torch.from_numpy(x).cuda()
    ld = t.vocab if ld is None else ld
    out = torch.full((n, ld), -7.0, dtype=torch.float32, device="cuda")
    t.logits(xd[:, :dim], out=out[:, :t.vocab] if ld != t.vocab else out)
    vb.check()
    got = out.cpu().numpy()
    if ld != t.vocab:
        assert np.all(got[:, t.vocab:] == -7.0), "columns past vocab were written"
    t.close()
    return got[:, :t.vocab]


def test_golden_hidden_rows_give_the_reference_session_logits(cuda_lib):
    need_gpu()
    import verbo_b200 as vb

    z = np.load(GOLDEN)
    for i in range(int(z["ncases"])):
        dtype = str(z[f"t{i}_dtype"])
        got = run_tail(vb, dtype, z[f"t{i}_q"], z.get(f"t{i}_s"), z[f"t{i}_norm"], float(z[f"t{i}_eps"]),
                       z[f"t{i}_x"])
        assert np.array_equal(got.view(np.uint32), z[f"t{i}_logits"].view(np.uint32)), str(z[f"t{i}_name"])


SHAPES = [(1, 32, 1), (3, 96, 129), (8, 896, 300), (9, 1056, 257), (16, 64, 1000), (17, 160, 513),
          (33, 128, 700), (64, 896, 129), (65, 1056, 300), (130, 96, 4099), (192, 896, 385), (256, 1056, 1500)]


@pytest.mark.parametrize("dtype", ["q8", "q4", "f32"])
@pytest.mark.parametrize("n,dim,vocab", SHAPES)
def test_tail_matches_oracle(cuda_lib, dtype, n, dim, vocab):
    need_gpu()
    import verbo_b200 as vb

    g = np.random.default_rng(n * 1000 + dim + vocab)
    q, s = po.random_head(dtype, vocab, dim, seed=vocab + dim)
    norm = (1 + 0.25 * g.standard_normal(dim)).astype(np.float32)
    x = (g.standard_normal((n, dim)) * 3.0).astype(np.float32)
    want, _, _ = po.logits_tail(dtype, q, s, norm, 1e-6, x)
    got = run_tail(vb, dtype, q, s, norm, 1e-6, x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


TC_SHAPES = [(33, 128, 700), (64, 896, 129), (65, 1056, 300), (130, 96, 4099), (192, 896, 385), (256, 1056, 1500)]


@pytest.mark.parametrize("n,dim,vocab", TC_SHAPES)
def test_tcgen05_tail_matches_oracle(cuda_lib, monkeypatch, n, dim, vocab):
    """The tcgen05 head kernel (Q8, more than 32 tokens; selected by
    VERBO_CUDA_TAIL_TCGEN05=1) bit for bit against the oracle: ragged vocab
    tiles, partial K chunks (dim 1056, 96) and several token tiles."""
    need_gpu()
    import verbo_b200 as vb

    monkeypatch.setenv("VERBO_CUDA_TAIL_TCGEN05", "1")
    g = np.random.default_rng(n * 1000 + dim + vocab + 7)
    q, s = po.random_head("q8", vocab, dim, seed=vocab + dim + 7)
    norm = (1 + 0.25 * g.standard_normal(dim)).astype(np.float32)
    x = (g.standard_normal((n, dim)) * 3.0).astype(np.float32)
    want, _, _ = po.logits_tail("q8", q, s, norm, 1e-6, x)
    got = run_tail(vb, "q8", q, s, norm, 1e-6, x)
    vb.check()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_tcgen05_tail_full_vocab(cuda_lib, monkeypatch, qwen_head):
    """256 rows at V = 151936 on the tcgen05 kernel equal the mma.sync
    kernel's logits bit for bit, and a slice of vocab ids equals the oracle."""
    need_gpu()
    import verbo_b200 as vb

    q, s, norm = qwen_head
    x = (np.random.default_rng(14).standard_normal((256, 896)) * 3.0).astype(np.float32)
    t = vb.Tail("q8", q, s, norm, 1e-6)
    xd = torch.from_numpy(x).cuda()
    base = t.logits(xd).cpu().numpy()
    monkeypatch.setenv("VERBO_CUDA_TAIL_TCGEN05", "1")
    tc = t.logits(xd).cpu().numpy()
    vb.check()
    assert np.array_equal(tc.view(np.uint32), base.view(np.uint32))
    ids = np.r_[0:300, 151936 - 300:151936]
    want, _, _ = po.logits_tail("q8", q[ids], s[ids], norm, 1e-6, x)
    assert np.array_equal(tc[:, ids].view(np.uint32), want.view(np.uint32))


def test_tail_strided_rows_and_extreme_codes(cuda_lib):
    need_gpu()
    import verbo_b200 as vb

    g = np.random.default_rng(5)
    n, dim, vocab = 20, 224, 333
    q, s = po.random_head("q8", vocab, dim, seed=1)
    q[::7, ::3] = -128  # outside quant_rows' range, still a valid int8 code
    q[1::7, ::5] = 127
    norm = (1 + 0.25 * g.standard_normal(dim)).astype(np.float32)
    x = (g.standard_normal((n, dim)) * 3.0).astype(np.float32)
    x[3, :] = 0.0  # an all-zero row: rmsnorm of zeros, zero scales
    x[4, 5] = 1e30  # one huge element dominates its block
    want, _, _ = po.logits_tail("q8", q, s, norm, 1e-6, x)
    got = run_tail(vb, "q8", q, s, norm, 1e-6, x, ldx=dim + 40, ld=vocab + 13)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_tail_zero_rows_is_a_no_op(cuda_lib):
    need_gpu()
    import verbo_b200 as vb

    q, s = po.random_head("q8", 64, 64)
    t = vb.Tail("q8", q, s, np.ones(64, np.float32), 1e-6)
    out = torch.full((0, 64), 1.0, device="cuda")
    t.logits(torch.zeros(0, 64, device="cuda"), out=out)
    vb.check()


@pytest.fixture(scope="module")
def qwen_head():
    vocab, dim = 151936, 896
    q, s = po.random_head("q8", vocab, dim, seed=2026)
    g = np.random.default_rng(11)
    norm = (1 + 0.25 * g.standard_normal(dim)).astype(np.float32)
    return q, s, norm


def test_full_vocab_rows_match_oracle(cuda_lib, qwen_head):
    need_gpu()
    import verbo_b200 as vb

    q, s, norm = qwen_head
    x = (np.random.default_rng(12).standard_normal((3, 896)) * 3.0).astype(np.float32)
    want, _, _ = po.logits_tail("q8", q, s, norm, 1e-6, x)
    got = run_tail(vb, "q8", q, s, norm, 1e-6, x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_full_vocab_batch_properties(cuda_lib, qwen_head):
    """256 rows at V = 151936: each row equals itself computed alone, and a
    slice of vocab ids equals the oracle run on that slice of the head."""
    need_gpu()
    import verbo_b200 as vb

    q, s, norm = qwen_head
    x = (np.random.default_rng(13).standard_normal((256, 896)) * 3.0).astype(np.float32)
    t = vb.Tail("q8", q, s, norm, 1e-6)
    xd = torch.from_numpy(x).cuda()
    big = t.logits(xd).cpu().numpy()
    for r in (0, 63, 64, 200, 255):
        one = t.logits(xd[r:r + 1]).cpu().numpy()
        assert np.array_equal(one[0].view(np.uint32), big[r].view(np.uint32))
    vb.check()
    ids = np.r_[0:700, 75000:75300, 151936 - 500:151936]
    want, _, _ = po.logits_tail("q8", q[ids], s[ids], norm, 1e-6, x)
    assert np.array_equal(big[:, ids].view(np.uint32), want.view(np.uint32))


def test_tail_feeds_the_sampler(cuda_lib):
    """Device tail -> device sampler without a host round trip: greedy and
    top-k picks equal the oracle's on the reference session's logits."""
    need_gpu()
    import verbo_b200 as vb

    z = np.load(GOLDEN)
    x, logits = z["t0_x"], z["t0_logits"]
    t = vb.Tail("q8", z["t0_q"], z["t0_s"], z["t0_norm"], float(z["t0_eps"]))
    dev = t.logits(torch.from_numpy(x).cuda())
    seeds = np.arange(x.shape[0], dtype=np.uint64) + np.uint64(77)
    for opts in (dict(temp=0.0), dict(temp=0.8, top_k=20, top_p=0.9)):
        rng = torch.from_numpy(po.seed_states(seeds).view(np.int64).copy()).cuda()
        ids = vb.sample(dev, vb.Sampling(**opts), rng=rng).cpu().numpy()
        vb.check()
        ref, _ = po.sample_rows(logits, po.sampling(**opts), po.seed_states(seeds))
        assert np.array_equal(ids, ref), opts
