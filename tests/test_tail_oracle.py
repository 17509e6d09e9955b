"""The logits-tail oracle (oracle/tail_oracle.c) against the reference.

Three pins, all on the CPU:
* the golden fixture tests/golden/tail_models.npz: hidden rows read out of the
  reference's own Session on its two tiny checkpoints, with the head and norm
  that Model::load built and the session's logits (scalar build) - the oracle
  must reproduce those logits bit for bit;
* the reference's rmsnorm / quant_act / matmul compiled from its sources
  (oracle/_ref), on seeded heads of every dtype and dims with partial chunks:
  bit-exact against the VERBO_SCALAR build; against the default AVX2 build,
  which adds each row's block terms in another order, within the bound of
  that reordering;
* the C ABI rejects bad tail arguments before touching a device.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from oracle import pyoracle as po

GOLDEN = Path(__file__).resolve().parent / "golden" / "tail_models.npz"


def fixture_cases():
    z = np.load(GOLDEN)
    for i in range(int(z["ncases"])):
        yield (str(z[f"t{i}_name"]), str(z[f"t{i}_dtype"]), z[f"t{i}_q"], z.get(f"t{i}_s"), z[f"t{i}_norm"],
               float(z[f"t{i}_eps"]), z[f"t{i}_x"], z[f"t{i}_logits"], z[f"t{i}_logits_avx2"])


def term_bound(dtype, q, s, x_norm_q, xs):
    """Per (row, id): sum over blocks of |scale_w * scale_x| * sum |w_k * x_k|,
    which bounds every partial sum of any order of the terms (the AVX2 build
    splits each block into 8 lane sums of 4 products)."""
    w = s.view(np.float16).astype(np.float64)
    nb = w.shape[1]
    if dtype == "q8":
        qq = q.astype(np.int64)
    else:
        lo = (q & 0x0F).astype(np.int64) - 8
        hi = (q >> 4).astype(np.int64) - 8
        qq = np.concatenate([np.concatenate([lo[:, b * 16:(b + 1) * 16], hi[:, b * 16:(b + 1) * 16]], 1)
                             for b in range(nb)], 1)
    out = np.zeros((x_norm_q.shape[0], q.shape[0]))
    for b in range(nb):
        sb = np.abs(x_norm_q[:, b * 32:(b + 1) * 32].astype(np.int64)) @ np.abs(qq[:, b * 32:(b + 1) * 32]).T
        out += sb * np.abs(xs[:, b:b + 1] * w[None, :, b])
    return out


def test_golden_fixture_is_the_reference_session():
    cases = list(fixture_cases())
    assert [c[0] for c in cases] == ["tiny-qwen2/q8", "tiny-llama/q8", "tiny-llama/f32"]
    for name, dtype, q, s, norm, eps, x, logits, logits_avx2 in cases:
        got, xq, xs = po.logits_tail(dtype, q, s, norm, eps, x)
        assert np.array_equal(got.view(np.uint32), logits.view(np.uint32)), name
        # the AVX2 build differs only by the order of its sums
        assert np.allclose(logits_avx2, logits, rtol=0, atol=4e-6 * max(1.0, float(np.abs(logits).max()))), name


CASES = [("q8", 32, 17, 1), ("q8", 96, 513, 4), ("q8", 1056, 300, 3), ("q4", 64, 129, 2), ("q4", 1056, 200, 5),
         ("f32", 32, 17, 1), ("f32", 160, 257, 3)]


@pytest.mark.skipif(not po.ref_tail_available("scalar"), reason="reference tail harness not built")
@pytest.mark.parametrize("dtype,dim,vocab,n", CASES)
def test_oracle_is_the_scalar_reference(dtype, dim, vocab, n):
    g = np.random.default_rng(dim * 7 + n)
    q, s = po.random_head(dtype, vocab, dim, seed=dim + vocab)
    norm = (1 + 0.2 * g.standard_normal(dim)).astype(np.float32)
    x = (g.standard_normal((n, dim)) * 2.5).astype(np.float32)
    got, xq, xs = po.logits_tail(dtype, q, s, norm, 1e-5, x)
    want, rq, rs = po.ref_logits_tail(dtype, q, s, norm, 1e-5, x, build="scalar")
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    if dtype != "f32":
        assert np.array_equal(xq, rq) and np.array_equal(xs.view(np.uint32), rs.view(np.uint32))


@pytest.mark.skipif(not po.ref_tail_available("avx2"), reason="reference tail harness not built")
@pytest.mark.parametrize("dtype,dim,vocab,n", [c for c in CASES if c[0] != "f32"])
def test_oracle_within_reordering_of_the_avx2_reference(dtype, dim, vocab, n):
    g = np.random.default_rng(dim + n)
    q, s = po.random_head(dtype, vocab, dim, seed=dim)
    norm = (1 + 0.2 * g.standard_normal(dim)).astype(np.float32)
    x = (g.standard_normal((n, dim)) * 2.5).astype(np.float32)
    got, xq, xs = po.logits_tail(dtype, q, s, norm, 1e-5, x)
    want, rq, rs = po.ref_logits_tail(dtype, q, s, norm, 1e-5, x, build="avx2", threads=2)
    # the activations are quantised by the same scalar code in both builds
    assert np.array_equal(xq, rq) and np.array_equal(xs.view(np.uint32), rs.view(np.uint32))
    # the same terms added in two orders (nb fused steps per lane, 8 lanes):
    # each result is within (nb + 4) * 2^-24 * term_bound of the exact sum
    nb = dim // 32
    bound = 2 * (nb + 4) * 2.0 ** -24 * term_bound(dtype, q, s, xq, xs)
    assert np.all(np.abs(got.astype(np.float64) - want) <= bound + 1e-30)


def test_oracle_rejects_bad_arguments():
    q, s = po.random_head("q8", 8, 32)
    with pytest.raises(ValueError):
        po.logits_tail("q8", q[:, :24], s, np.ones(24, np.float32), 1e-5, np.ones((1, 24), np.float32))


def test_tail_abi_validates_before_any_device_work():
    import verbo_b200 as vb

    lib = vb.load_library()
    q = np.zeros((4, 64), dtype=np.int8)
    s = np.zeros((4, 2), dtype=np.uint16)
    norm = np.ones(64, dtype=np.float32)
    for dtype, vocab, dim, sp in ((3, 4, 64, s), (1, 0, 64, s), (1, 4, 48, s), (1, 4, 64, None),
                                  (0, 4, 16384 + 32, None)):
        h = lib.verbo_cuda_tail_new(dtype, vocab, dim, q.ctypes.data, None if sp is None else sp.ctypes.data,
                                    norm.ctypes.data, ctypes.c_float(1e-5), 0)
        assert not h
        assert lib.verbo_cuda_last_error().decode().startswith("verbo_cuda: ")
    assert lib.verbo_cuda_tail_logits(None, None, 1, 64, None, 4, None) == -1
    assert "tail is NULL" in lib.verbo_cuda_last_error().decode()
