"""Readers for the golden fixtures under tests/golden/ (made by make_golden.py)."""
from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path
from typing import List, Optional

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


@dataclass
class Case:
    name: str
    logits: np.ndarray
    hist: Optional[np.ndarray]
    off: Optional[np.ndarray]
    opts: dict
    seeds: np.ndarray
    ids: np.ndarray  # (rows, steps)


def small_cases() -> List[Case]:
    z = np.load(GOLDEN / "small.npz")
    out = []
    for i in range(int(z["ncases"])):
        tag = str(z[f"c{i}_tag"])
        o = z[f"c{i}_opts"]
        opts = dict(temp=float(o[0]), top_k=int(o[1]), top_p=float(o[2]), min_p=float(o[3]), repeat=float(o[4]),
                    repeat_last=int(o[5]))
        out.append(Case(f"{i}-{tag}", z[f"in_{tag}_logits"], z[f"in_{tag}_hist"], z[f"in_{tag}_off"], opts,
                        z[f"c{i}_seeds"], z[f"c{i}_ids"]))
    return out


def config_cases():
    """(workload, logits, hist, off, seeds, expected ids) for each benchmark config."""
    from verbo_b200 import workloads as wl

    cfg = json.loads((GOLDEN / "configs.json").read_text())
    out = []
    for name, c in cfg.items():
        w = wl.WORKLOADS[name]
        x = wl.make_rows_np(w, c["rows"])
        h, off = wl.make_hist_np(w, c["rows"])
        if hashlib.sha256(x.tobytes()).hexdigest() != c["logits_sha256"]:
            raise RuntimeError(f"{name}: regenerated logits differ from the fixture's (numpy generator changed)")
        out.append((w, x, h, off, w.sampler_seeds(0, c["rows"]), np.array(c["ids"], dtype=np.int32)))
    return out
