"""Reader of tests/golden/decode_models.npz (tests/golden/make_decode_golden.py):
B concurrent generations per case, each an independent verbo::generate run of
the reference on a tiny checkpoint, with every pick's id and the hidden row
its logits came from, plus the head the tail needs."""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden" / "decode_models.npz"


@dataclass
class DecodeCase:
    name: str
    model: str
    opts: dict
    seeds: np.ndarray
    prompts: list
    ids: np.ndarray       # [B, S] picks, -1 past a generation's end
    npicks: np.ndarray    # [B]
    stopped: np.ndarray   # [B]: the last pick is a stop id
    x: np.ndarray         # [B, S, dim] hidden rows, zeros past the end
    head_dtype: str
    q: np.ndarray
    s: np.ndarray | None
    norm: np.ndarray
    eps: float

    @property
    def B(self) -> int:
        return self.ids.shape[0]

    @property
    def steps(self) -> int:
        return self.ids.shape[1]


def load_cases():
    z = np.load(GOLDEN)
    out = []
    for name in (str(c) for c in z["cases"]):
        o = z[f"{name}_opts"]
        opts = dict(temp=float(o[0]), top_k=int(o[1]), top_p=float(o[2]), min_p=float(o[3]), repeat=float(o[4]),
                    repeat_last=int(o[5]))
        off = z[f"{name}_prompt_off"]
        pr = z[f"{name}_prompt"]
        out.append(DecodeCase(name, str(z[f"{name}_model"]), opts, z[f"{name}_seeds"],
                              [pr[off[i]:off[i + 1]].copy() for i in range(len(off) - 1)], z[f"{name}_ids"],
                              z[f"{name}_npicks"], z[f"{name}_stopped"], z[f"{name}_x"], str(z[f"{name}_head_dtype"]),
                              z[f"{name}_q"], z[f"{name}_s"] if f"{name}_s" in z.files else None, z[f"{name}_norm"],
                              float(z[f"{name}_eps"])))
    return out
