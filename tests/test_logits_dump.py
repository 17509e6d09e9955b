"""The reference's logits dump layout (cli/main.cpp:174-190) as a parity input.

tests/golden/tiny_qwen2.f32 holds the 38 real rows of the reference's
tiny-qwen2 fixture in that layout; tests/golden/dump_ids.json the ids the
reference's own Sampler picks from them (tests/golden/make_golden.py).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import pyoracle as po
from verbo_b200 import logits_dump

GOLDEN = Path(__file__).resolve().parent / "golden"


def _fixture():
    d = json.loads((GOLDEN / "dump_ids.json").read_text())
    return logits_dump.read_dump(GOLDEN / "tiny_qwen2.f32", d["vocab"]), d


def test_dump_layout_round_trip(tmp_path):
    g = np.random.default_rng(1)
    rows = g.standard_normal((7, 33)).astype(np.float32)
    f = tmp_path / "rows.bin"
    logits_dump.write_dump(f, rows)
    assert f.stat().st_size == rows.size * 4  # raw fp32, no header
    assert np.array_equal(logits_dump.read_dump(f, 33), rows)
    # two eval_all outputs appended: still rows of `vocab`
    with open(f, "ab") as fh:
        rows[:2].tofile(fh)
    assert logits_dump.read_dump(f, 33).shape == (9, 33)
    with pytest.raises(ValueError, match="whole number of rows"):
        logits_dump.read_dump(f, 32)


def test_oracle_matches_reference_on_dumped_rows():
    x, d = _fixture()
    assert x.shape == (38, 400)
    seeds = np.arange(d["rows"], dtype=np.uint64) + np.uint64(d["seed0"])
    for name, case in d["cases"].items():
        st = po.seed_states(seeds)
        got = np.stack([po.sample_rows(x, po.sampling(**case["opts"]), st)[0] for _ in range(d["steps"])], axis=1)
        assert np.array_equal(got, np.array(case["ids"])), name


@pytest.mark.gpu
def test_cuda_sampler_matches_reference_on_dumped_rows(cuda_lib):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("gpu tests need a CUDA device")
    from tests.gpu_util import compare, run_gpu, run_oracle

    x, d = _fixture()
    seeds = np.arange(d["rows"], dtype=np.uint64) + np.uint64(d["seed0"])
    for name, case in d["cases"].items():
        ids, _, _ = run_gpu(x, case["opts"], seeds, steps=d["steps"])
        _, ost, _ = run_oracle(x, case["opts"], seeds, steps=d["steps"])
        compare(ids, np.array(case["ids"], dtype=np.int32), ost, name)
