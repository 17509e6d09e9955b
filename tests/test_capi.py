"""CPU tests of the C ABI boundary (no kernel launches).

* the library loads and exports exactly the functions include/verbo_cuda.h
  declares;
* the host-side RNG (Sampler::reset / Sampler::unit) equals the oracle's;
* argument validation fails before touching the GPU, with the reference
  C ABI's convention: -1 and a message in verbo_cuda_last_error().
"""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import verbo_b200 as vb
from oracle import pyoracle as po
from verbo_b200 import build

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "verbo_cuda.h"


@pytest.fixture(scope="module")
def lib():
    build.build()
    return vb.load_library()


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"VERBO_CUDA_API\s+[^;(]*?\b(verbo_cuda_\w+)\s*\(", text)))


def test_exports_match_header(lib):
    declared = declared_functions()
    assert len(declared) == 38
    out = subprocess.run(["nm", "-D", "--defined-only", str(build.LIB)], capture_output=True, text=True,
                         check=True).stdout
    exported = sorted(ln.split()[-1] for ln in out.splitlines() if ln.split()[-1].startswith("verbo_cuda_"))
    assert exported == declared
    for name in declared:
        assert getattr(lib, name) is not None


def test_version_and_defaults(lib):
    assert vb.version().startswith("0.1.0")
    d = lib.verbo_cuda_default_sampling()
    # include/verbo/verbo.hpp:56-64
    assert (round(d.temp, 6), d.top_k, round(d.top_p, 6), d.min_p, d.repeat, d.repeat_last, d.seed) == \
        (0.7, 40, 0.9, 0.0, 1.0, 64, 0)


def test_rng_matches_oracle(lib):
    for seed in (1, 42, 2**63 + 5, 123456789):
        st = (ctypes.c_ulonglong * 2)()
        assert lib.verbo_cuda_rng_seed(seed, st) == 0
        ost = po.seed_states(np.array([seed], dtype=np.uint64))
        assert [st[0], st[1]] == [int(ost[0, 0]), int(ost[0, 1])]
        olib = po.oracle_lib()
        for _ in range(5):
            assert lib.verbo_cuda_rng_unit(st) == olib.oracle_unit(ost[0].ctypes.data)


def test_seed_zero_uses_clock(lib):
    a, b = vb.seed_states([0])[0], vb.seed_states([0])[0]
    assert a != [0, 0] and b != [0, 0]


def _sample(lib, **kw):
    args = dict(logits=1, rows=1, vocab=8, ld=8, hist=None, hist_off=None, opts=vb.Sampling(), rng=1, out=1,
                stats=None, stream=None)
    args.update(kw)
    o = args["opts"]._c() if args["opts"] is not None else None
    return lib.verbo_cuda_sample(args["logits"], args["rows"], args["vocab"], args["ld"], args["hist"],
                                 args["hist_off"], ctypes.byref(o) if o is not None else None, args["rng"],
                                 args["out"], args["stats"], args["stream"])


@pytest.mark.parametrize("kw,msg", [
    (dict(opts=None), "opts is NULL"),
    (dict(rows=-1), "rows"),
    (dict(vocab=0), "vocab"),
    (dict(vocab=400000, ld=400000), "vocab"),
    (dict(ld=4), "ld"),
    (dict(hist=1), "hist"),
    (dict(opts=vb.Sampling(temp=float("nan"))), "temp"),
    (dict(opts=vb.Sampling(temp=float("inf"))), "temp"),
    (dict(rng=None), "rng"),
    (dict(logits=None), "NULL"),
])
def test_sample_validation(lib, kw, msg):
    assert _sample(lib, **kw) == -1
    assert msg in lib.verbo_cuda_last_error().decode()


def test_zero_rows_is_a_noop(lib):
    assert _sample(lib, rows=0, logits=None, out=None) == 0
    assert lib.verbo_cuda_last_error().decode() == ""


def test_shard_and_merge_validation(lib):
    o = vb.Sampling()._c()
    assert lib.verbo_cuda_shard_topk(1, 2, 100, 100, 0, 1000, None, None, ctypes.byref(o), 0, 1, 1, None) == -1
    assert "k must" in lib.verbo_cuda_last_error().decode()
    assert lib.verbo_cuda_shard_topk(1, 2, 100, 100, 950, 1000, None, None, ctypes.byref(o), 8, 1, 1, None) == -1
    assert "shard" in lib.verbo_cuda_last_error().decode()
    bad = vb.Sampling(top_k=0)._c()
    assert lib.verbo_cuda_merge_sample(1, 1, 2, 8, 64, 1000, ctypes.byref(bad), 1, 1, None, None) == -1
    assert "top_k" in lib.verbo_cuda_last_error().decode()
    big = vb.Sampling(top_k=10)._c()
    assert lib.verbo_cuda_merge_sample(1, 1, 2, 8, 1024, 1000, ctypes.byref(big), 1, 1, None, None) == -1
    assert "nshards * k" in lib.verbo_cuda_last_error().decode()


def test_batch_validation(lib):
    """Arguments are checked before any device is touched."""
    assert lib.verbo_cuda_batch_new(None, 4, 0) is None
    assert "cfg is NULL" in lib.verbo_cuda_last_error().decode()
    o = vb.Sampling()._c()
    assert lib.verbo_cuda_batch_new(ctypes.byref(o), 0, 0) is None
    assert "streams" in lib.verbo_cuda_last_error().decode()
    for rl in (0, 4096):
        bad = vb.Sampling(repeat=1.1, repeat_last=rl)._c()
        assert lib.verbo_cuda_batch_new(ctypes.byref(bad), 4, 0) is None
        assert "repeat_last" in lib.verbo_cuda_last_error().decode()
    assert lib.verbo_cuda_batch_step(None, 1, 10, 10, 1, None, None) == -1
    assert "batch is NULL" in lib.verbo_cuda_last_error().decode()
    assert lib.verbo_cuda_batch_reset(None, 0, 1, None) == -1
    assert lib.verbo_cuda_batch_accept(None, 0, None, 0, None) == -1


def test_error_message_is_thread_local_and_cleared(lib):
    assert _sample(lib, opts=None) == -1
    assert lib.verbo_cuda_last_error().decode() != ""
    assert _sample(lib, rows=0) == 0
    assert lib.verbo_cuda_last_error().decode() == ""


def _build_hpp_kat(tmp_path):
    exe = tmp_path / "hpp_kat"
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{ROOT / 'include'}", str(ROOT / "tests/cpp/hpp_kat.cpp"),
                    f"-L{build.LIB.parent}", "-lverbo_cuda", f"-Wl,-rpath,{build.LIB.parent}", "-o", str(exe)],
                   check=True, capture_output=True)
    return exe


def test_cpp_header_compiles_and_reports_errors(lib, tmp_path):
    """The C++ wrapper builds against the library; without a usable device the
    constructor throws with the C ABI's message instead of crashing."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("device present: covered by the gpu test")
    exe = _build_hpp_kat(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 2 and r.stdout.startswith("error verbo_cuda:"), r.stdout
