"""Generates the decode-loop fixture from the REFERENCE itself.

Run where the reference checkout and its compiled harness exist:

    make -C oracle ref REF=<verbo checkout>
    python tests/golden/make_decode_golden.py <verbo checkout>

Writes ``decode_models.npz`` next to this script: for each case, B concurrent
generations on one of the reference's tiny checkpoints (tests/data), each an
independent ``verbo::generate`` run (src/sampler.cpp:111-181) of the
reference built with its VERBO_SCALAR option, with its own prompt and seed.
Per generation the file holds the ids it picked (the stop id last when it
stopped on one) and, for every pick, the hidden row its logits came from (the
residual of the producing position before the final rmsnorm, read out of a
reference Session that replays the same loop; the harness checks that the
replay's ids equal generate's).  The head, norm weight and eps that
Model::load built complete the case.  A decode step of the GPU path takes row
j of every generation, runs the tail and the pick on the device, and must
return pick j of each.

The AVX2 build's generations are compared on the way and the count of ids
that differ from the scalar build's is printed (its matmuls round
differently, so its hidden rows differ too).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import pyoracle as po  # noqa: E402

MAX_TOKENS = 32
# name, checkpoint, weight dtype, options (verbo::Sampling fields), seeds
CASES = (
    ("qwen2_q8_topk", "tiny-qwen2", "q8",
     dict(temp=0.8, top_k=40, top_p=0.9, min_p=0.05, repeat=1.1, repeat_last=64), (11, 12, 13, 14)),
    ("qwen2_f32_greedy_penalty", "tiny-qwen2", "f32",
     dict(temp=0.0, top_k=40, top_p=0.9, min_p=0.0, repeat=1.3, repeat_last=16), (1, 2, 3)),
    ("qwen2_q4_full_vocab", "tiny-qwen2", "q4",
     dict(temp=1.0, top_k=0, top_p=0.95, min_p=0.0, repeat=1.0, repeat_last=64), (21, 22, 23, 24, 25)),
    ("llama_q8_defaults", "tiny-llama", "q8",
     dict(temp=0.7, top_k=40, top_p=0.9, min_p=0.0, repeat=1.0, repeat_last=64), (31, 32)),
)


def prompts(ref_dir: Path, count: int):
    """Chat-style prompts from the tokenizer cases of tiny-qwen2's ref.json:
    bos + the ids of the non-empty cases, in order."""
    cases = json.loads((ref_dir / "tests/data/tiny-qwen2/ref.json").read_text())["cases"]
    texts = [c["ids"] for c in cases if c["ids"]]
    return [[1] + texts[(3 * i + 2) % len(texts)] for i in range(count)]


def main(ref_dir: str) -> None:
    ref_dir = Path(ref_dir)
    out = {"cases": np.array([c[0] for c in CASES])}
    for name, model, dtype, opts, seeds in CASES:
        mdir = ref_dir / "tests/data" / model
        prs = prompts(ref_dir, len(seeds))
        runs, differ = [], 0
        for pr, seed in zip(prs, seeds):
            o = po.sampling(**opts, seed=seed)
            r = po.ref_decode(mdir, dtype, pr, o, MAX_TOKENS, build="scalar")
            a = po.ref_decode(mdir, dtype, pr, o, MAX_TOKENS, build="avx2")
            n = min(len(r["ids"]), len(a["ids"]))
            differ += int((r["ids"][:n] != a["ids"][:n]).sum()) + abs(len(r["ids"]) - len(a["ids"]))
            runs.append(r)
        head = po.ref_model_tail(mdir, dtype, [1], build="scalar")
        B, S, dim = len(runs), max(len(r["ids"]) for r in runs), head["x"].shape[1]
        ids = np.full((B, S), -1, dtype=np.int32)
        x = np.zeros((B, S, dim), dtype=np.float32)
        for b, r in enumerate(runs):
            ids[b, :len(r["ids"])] = r["ids"]
            x[b, :len(r["ids"])] = r["x"]
        off = np.cumsum([0] + [len(p) for p in prs]).astype(np.int64)
        out[f"{name}_model"] = np.array(f"{model}/{dtype}")
        out[f"{name}_opts"] = np.array([opts["temp"], opts["top_k"], opts["top_p"], opts["min_p"], opts["repeat"],
                                        opts["repeat_last"]], dtype=np.float64)
        out[f"{name}_seeds"] = np.array(seeds, dtype=np.uint64)
        out[f"{name}_prompt"] = np.concatenate([np.array(p, dtype=np.int32) for p in prs])
        out[f"{name}_prompt_off"] = off
        out[f"{name}_ids"] = ids
        out[f"{name}_npicks"] = np.array([len(r["ids"]) for r in runs], dtype=np.int32)
        out[f"{name}_stopped"] = np.array([r["stopped"] for r in runs], dtype=np.int32)
        out[f"{name}_x"] = x
        out[f"{name}_head_dtype"] = np.array(head["dtype"])
        out[f"{name}_q"] = head["q"]
        if head["s"] is not None:
            out[f"{name}_s"] = head["s"]
        out[f"{name}_norm"] = head["norm"]
        out[f"{name}_eps"] = np.array(head["eps"], dtype=np.float32)
        print(f"{name}: {B} generations, picks {out[f'{name}_npicks'].tolist()}, "
              f"stopped {out[f'{name}_stopped'].tolist()}, AVX2 build differs in {differ} ids")
    np.savez_compressed(HERE / "decode_models.npz", **out)
    print("wrote", HERE / "decode_models.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference")
