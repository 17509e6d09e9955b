"""Generates the golden fixtures of the sampling path from the REFERENCE itself.

Run where the reference checkout and its compiled harness exist:

    make -C oracle ref REF=<verbo checkout>
    python tests/golden/make_golden.py <verbo checkout>

Writes, next to this script:

* ``small.npz``    - explicit small cases (logits, histories, options, seeds)
                     with the token ids the reference's own Sampler returns for
                     3 consecutive picks per row (src/sampler.cpp:50-109).  The
                     first case uses 8 rows of real logits from the reference's
                     tiny-qwen2 fixture (tests/data/tiny-qwen2/ref_logits.bin,
                     38 x 400 fp32 produced by transformers);
* ``configs.json`` - the five benchmark configurations at a few rows each:
                     the ids of 2 picks per row from the reference, plus a
                     SHA-256 of the regenerated logits so a test can tell a
                     changed generator from a wrong sampler;
* ``tiny_qwen2.f32`` - all 38 real rows of that fixture in the reference's
                     logits dump layout (cli/main.cpp:174-190: raw fp32 rows),
                     read back through verbo_b200.logits_dump;
* ``dump_ids.json``  - the ids the reference's Sampler picks from those rows
                     (2 picks per row) under three option sets;
* ``tail_models.npz`` - the logits producer tail (src/session.cpp:163-169) on
                     the reference's two tiny checkpoints: the final hidden
                     rows read out of a reference Session after eval_all on
                     the first TAIL_ROWS ids of ref.json, the head and norm
                     that Model::load built, and the session's logits from the
                     VERBO_SCALAR build (bit-exact target) and the default
                     AVX2 build.

The reference's Sampler has no golden vectors of its own for seeded draws
(its tests check determinism and ranges only, tests/test_core.cpp:454-496),
so these files are the pin.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import pyoracle as po  # noqa: E402
from verbo_b200 import logits_dump  # noqa: E402
from verbo_b200 import workloads as wl  # noqa: E402

DUMP_OPTS = {
    "greedy": dict(temp=0.0, top_k=40, top_p=0.9, min_p=0.0, repeat=1.0, repeat_last=64),
    "default": dict(temp=0.7, top_k=40, top_p=0.9, min_p=0.0, repeat=1.0, repeat_last=64),
    "nucleus": dict(temp=1.0, top_k=0, top_p=0.95, min_p=0.02, repeat=1.0, repeat_last=64),
}

STEPS_SMALL = 3
STEPS_CFG = 2
CFG_ROWS = {"c1": 1, "c2": 6, "c3": 6, "c4": 4, "c5": 6}
TAIL_ROWS = 12
TAIL_CASES = (("tiny-qwen2", "q8"), ("tiny-llama", "q8"), ("tiny-llama", "f32"))


def opts_array(o: dict) -> np.ndarray:
    return np.array([o["temp"], o["top_k"], o["top_p"], o["min_p"], o["repeat"], o["repeat_last"]], dtype=np.float64)


def special_rows(g: np.random.Generator, V: int) -> np.ndarray:
    rows = []
    rows.append(np.round(g.standard_normal(V) * 2) / 2)                      # many ties (0.5 grid)
    r = np.full(V, -np.inf); r[g.choice(V, 20, replace=False)] = g.standard_normal(20)
    rows.append(r)                                                             # masked to 20 finite values
    r = g.standard_normal(V); r[g.choice(V, V // 3, replace=False)] = 0.0
    r[g.choice(V, V // 3, replace=False)] = -0.0
    rows.append(r)                                                             # +0 / -0 ties
    rows.append(np.sort(g.standard_normal(V)))                                 # ascending (adversarial order)
    rows.append(np.full(V, 1.25))                                              # constant row
    rows.append(g.standard_normal(V) * 8.0)                                    # wide logits
    return np.stack(rows).astype(np.float32)


def make_hist(g: np.random.Generator, rows: int, V: int, H: int):
    hist = g.integers(-5, V + 5, size=rows * H).astype(np.int32)              # includes out-of-range ids
    hist[::7] = hist[1::7][: len(hist[::7])] if rows * H > 7 else hist[::7]   # duplicates
    off = np.arange(rows + 1, dtype=np.int64) * H
    return hist, off


def small_cases(ref_dir: Path):
    g = np.random.default_rng(20240601)
    cases = []
    qwen = np.fromfile(ref_dir / "tests/data/tiny-qwen2/ref_logits.bin", dtype=np.float32).reshape(-1, 400)[:8]
    h, o = make_hist(g, 8, 400, 24)
    for opts in (
        dict(temp=0.7, top_k=40, top_p=0.9, min_p=0.0, repeat=1.0, repeat_last=64),       # defaults
        dict(temp=0.6, top_k=30, top_p=0.85, min_p=0.0, repeat=1.3, repeat_last=16),      # model defaults + penalty
        dict(temp=0.0, top_k=40, top_p=0.9, min_p=0.0, repeat=1.3, repeat_last=64),       # greedy + penalty
        dict(temp=1.0, top_k=0, top_p=0.5, min_p=0.0, repeat=1.0, repeat_last=64),        # full vocab nucleus
        dict(temp=1.2, top_k=0, top_p=1.0, min_p=0.2, repeat=1.1, repeat_last=8),         # min-p only
        dict(temp=0.9, top_k=300, top_p=0.95, min_p=0.01, repeat=1.0, repeat_last=64),
        dict(temp=0.8, top_k=399, top_p=0.99, min_p=0.0, repeat=0.8, repeat_last=0),      # repeat < 1, whole history
        dict(temp=1.5, top_k=400, top_p=0.97, min_p=0.05, repeat=1.0, repeat_last=64),    # top_k == V
    ):
        cases.append(("qwen", qwen, h, o, opts))
    V = 4096
    sp = special_rows(g, V)
    h2, o2 = make_hist(g, sp.shape[0], V, 40)
    for opts in (
        dict(temp=0.0, top_k=40, top_p=0.9, min_p=0.0, repeat=1.5, repeat_last=64),
        dict(temp=0.7, top_k=40, top_p=0.9, min_p=0.0, repeat=1.2, repeat_last=64),
        dict(temp=1.0, top_k=5, top_p=1.0, min_p=0.3, repeat=1.0, repeat_last=64),
        dict(temp=1.3, top_k=0, top_p=0.9, min_p=0.0, repeat=1.1, repeat_last=20),
        dict(temp=0.5, top_k=1500, top_p=0.8, min_p=0.0, repeat=1.0, repeat_last=64),
        dict(temp=2.0, top_k=1024, top_p=1.0, min_p=0.0, repeat=1.0, repeat_last=64),
        dict(temp=0.9, top_k=0, top_p=0.999, min_p=0.001, repeat=1.05, repeat_last=40),
    ):
        cases.append(("special", sp, h2, o2, opts))
    # odd vocabulary and an unaligned leading dimension
    V3 = 1001
    x = (g.standard_normal((5, V3)) * 3).astype(np.float32)
    h3, o3 = make_hist(g, 5, V3, 12)
    for opts in (
        dict(temp=0.0, top_k=40, top_p=0.9, min_p=0.0, repeat=1.2, repeat_last=64),
        dict(temp=0.7, top_k=40, top_p=0.9, min_p=0.05, repeat=1.1, repeat_last=64),
        dict(temp=1.1, top_k=0, top_p=0.9, min_p=0.0, repeat=1.0, repeat_last=64),
    ):
        cases.append(("odd", x, h3, o3, opts))
    return cases


def main(ref_dir: str) -> None:
    ref_dir = Path(ref_dir)
    out = {}
    for i, (tag, x, h, o, opts) in enumerate(small_cases(ref_dir)):
        rows = x.shape[0]
        seeds = (np.arange(rows, dtype=np.uint64) * np.uint64(7919) + np.uint64(1000 + i))
        ids = po.ref_sample_rows(x, po.sampling(**opts), seeds, h, o, steps=STEPS_SMALL)
        out[f"c{i}_tag"] = np.array(tag)
        out[f"in_{tag}_logits"] = x
        out[f"in_{tag}_hist"] = h
        out[f"in_{tag}_off"] = o
        out[f"c{i}_opts"] = opts_array(opts)
        out[f"c{i}_seeds"] = seeds
        out[f"c{i}_ids"] = ids
    out["ncases"] = np.array(len(small_cases(ref_dir)))
    np.savez_compressed(HERE / "small.npz", **out)

    cfg = {}
    for name, w in wl.WORKLOADS.items():
        rows = CFG_ROWS[name]
        x = wl.make_rows_np(w, rows)
        h, o = wl.make_hist_np(w, rows)
        seeds = w.sampler_seeds(0, rows)
        ids = po.ref_sample_rows(x, po.sampling(**w.sampling_kwargs()), seeds, h, o, steps=STEPS_CFG)
        cfg[name] = {
            "rows": rows,
            "steps": STEPS_CFG,
            "logits_sha256": hashlib.sha256(x.tobytes()).hexdigest(),
            "hist_sha256": None if h is None else hashlib.sha256(h.tobytes()).hexdigest(),
            "ids": ids.tolist(),
        }
    (HERE / "configs.json").write_text(json.dumps(cfg, indent=1) + "\n")

    rows = np.fromfile(ref_dir / "tests/data/tiny-qwen2/ref_logits.bin", dtype=np.float32).reshape(-1, 400)
    logits_dump.write_dump(HERE / "tiny_qwen2.f32", rows)
    back = logits_dump.read_dump(HERE / "tiny_qwen2.f32", 400)
    seeds = np.arange(back.shape[0], dtype=np.uint64) + np.uint64(9001)
    dump = {"vocab": 400, "rows": int(back.shape[0]), "seed0": 9001, "steps": STEPS_CFG, "cases": {}}
    for name, opts in DUMP_OPTS.items():
        ids = po.ref_sample_rows(back, po.sampling(**opts), seeds, None, None, steps=STEPS_CFG)
        dump["cases"][name] = {"opts": opts, "ids": ids.tolist()}
    (HERE / "dump_ids.json").write_text(json.dumps(dump, indent=1) + "\n")

    toks = json.loads((ref_dir / "tests/data/tiny-qwen2/ref.json").read_text())["ids"][:TAIL_ROWS]
    tail = {"ncases": np.array(len(TAIL_CASES)), "toks": np.array(toks, dtype=np.int32)}
    for i, (model, dtype) in enumerate(TAIL_CASES):
        r = po.ref_model_tail(ref_dir / "tests/data" / model, dtype, toks, build="scalar")
        tail[f"t{i}_name"] = np.array(f"{model}/{dtype}")
        tail[f"t{i}_dtype"] = np.array(r["dtype"])
        tail[f"t{i}_eps"] = np.array(r["eps"], dtype=np.float32)
        tail[f"t{i}_x"] = r["x"]
        tail[f"t{i}_q"] = r["q"]
        if r["s"] is not None:
            tail[f"t{i}_s"] = r["s"]
        tail[f"t{i}_norm"] = r["norm"]
        tail[f"t{i}_logits"] = r["logits"]
        # the AVX2 build's tail on the scalar build's hidden rows (its own
        # layers round differently, so its session logits are not comparable)
        tail[f"t{i}_logits_avx2"] = po.ref_logits_tail(r["dtype"], r["q"], r["s"], r["norm"], r["eps"], r["x"],
                                                       build="avx2")[0]
    np.savez_compressed(HERE / "tail_models.npz", **tail)
    print("wrote", HERE / "small.npz", HERE / "configs.json", HERE / "tiny_qwen2.f32", HERE / "dump_ids.json",
          HERE / "tail_models.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference")
