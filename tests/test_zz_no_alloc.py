"""The allocation-free entry point, verbo_cuda_sample_noalloc.

It exists for callers that cannot let the library allocate device memory:
a serving engine that has reserved almost all HBM for its own pool, or a
decode loop that cannot take the device-wide synchronisation of cudaMalloc.
Its scratch is a fixed array inside the library, so these tests check, through
the C ABI, that it returns exactly what verbo_cuda_sample returns, on two
calls in a row (the second call finds the previous call's contents in the
shared array), and that it allocates no device memory while doing so.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import pyoracle as po
from tests.gpu_util import compare

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def vb(cuda_lib):
    if not torch.cuda.is_available():
        pytest.fail("gpu tests need a CUDA device")
    import verbo_b200

    return verbo_b200


CASES = [
    (151936, 200, dict(temp=0.0, repeat=1.2, repeat_last=128)),
    (151936, 64, dict(temp=0.8, top_k=50, top_p=0.95, repeat=1.1, repeat_last=256)),
    (49152, 17, dict(temp=0.7, top_k=40, top_p=0.9, min_p=0.05, repeat=1.1, repeat_last=64)),
    (400, 8, dict(temp=1.2, top_k=256, top_p=0.97, min_p=0.0)),
]


@pytest.mark.parametrize("vocab,rows,opts", CASES, ids=["greedy", "topk50", "c1-like", "small-vocab"])
def test_noalloc_matches_sample_on_two_calls(vb, vocab, rows, opts):
    g = np.random.default_rng([vocab, rows])
    x = torch.from_numpy((g.standard_normal((rows, vocab)) * 2).astype(np.float32)).cuda()
    H = 48
    hist = torch.from_numpy(g.integers(0, vocab, size=rows * H).astype(np.int32)).cuda()
    off = torch.arange(rows + 1, dtype=torch.int64, device="cuda") * H
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(vocab)
    states = po.seed_states(seeds).view(np.int64)
    rng_a = torch.from_numpy(states.copy()).cuda()
    rng_b = torch.from_numpy(states.copy()).cuda()
    o = vb.Sampling(**opts)
    want = torch.empty(rows, dtype=torch.int32, device="cuda")
    got = torch.empty(rows, dtype=torch.int32, device="cuda")
    vb.sample(x, o, rng=rng_a, hist=hist, hist_off=off, out=want)  # the allocating entry point sets up first
    rng_a.copy_(rng_b)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for call in range(2):
        vb.sample(x, o, rng=rng_a, hist=hist, hist_off=off, out=want)
        vb.sample_noalloc(x, o, rng=rng_b, hist=hist, hist_off=off, out=got)
        vb.check()
        assert torch.equal(got, want), f"call {call}: ids differ"
        assert torch.equal(rng_a, rng_b), f"call {call}: rng states differ"
        if call == 0:
            # and the first call's ids against the oracle (the reference's
            # Sampler restated), on the same rows, histories and seeds
            xh, hh, oh = x.cpu().numpy(), hist.cpu().numpy(), off.cpu().numpy()
            ora, ost = po.sample_rows(xh, po.sampling(**opts), po.seed_states(seeds), hh, oh)
            compare(got.cpu().numpy()[:, None], ora[:, None], ost[:, None], "noalloc vs oracle")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before


def test_noalloc_first_call_in_a_fresh_process(vb):
    """The allocation-free entry point as the first call of the library in a
    process.  CUDA loads the library's module lazily, so this first call is
    where the module's device memory (the fixed scratch array and the code)
    is placed: the worker reports that cost, and checks that the calls after
    it change the device's free memory by nothing."""
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    env = dict(os.environ)
    env.pop("CUDA_MODULE_LOADING", None)
    r = subprocess.run([sys.executable, str(root / "tests" / "noalloc_first_call.py")], capture_output=True,
                       text=True, timeout=300, env=env, cwd=str(root))
    assert r.returncode == 0, r.stdout + r.stderr
    rep = json.loads(r.stdout.strip().splitlines()[-1])
    print("first allocation-free call:", rep)
    assert rep["ids_equal"] and rep["later_calls_bytes"] == 0
    # what the first call placed: the library's module (the 8 MiB array plus
    # code and small globals), or nothing if the module was loaded eagerly
    assert rep["first_call_bytes"] <= 64 << 20


def test_noalloc_rejects_sizes_beyond_the_scratch(vb):
    one = torch.zeros(1, device="cuda")
    ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib = vb.load_library()
    # greedy keeps one key per item, top-k up to 256: their limits differ
    for rows, o in ((100000, vb.Sampling(temp=0.0)._c()), (4096, vb.Sampling(temp=0.8, top_k=50)._c())):
        rc = lib.verbo_cuda_sample_noalloc(one.data_ptr(), rows, 151936, 151936, None, None, ctypes.byref(o),
                                           ids.data_ptr(), ids.data_ptr(), None, None)
        assert rc == -1
        msg = lib.verbo_cuda_last_error().decode()
        assert "fixed scratch" in msg and "rows at vocab 151936" in msg


def test_noalloc_rejects_options_outside_its_kernel(vb):
    x = torch.zeros(2, 1000, device="cuda")
    with pytest.raises(vb.VerboCudaError, match="allocation-free"):
        vb.sample_noalloc(x, vb.Sampling(temp=1.0, top_k=0, top_p=0.9), rng=torch.zeros(2, 2, dtype=torch.int64,
                                                                                         device="cuda"))
