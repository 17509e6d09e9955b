"""The reference's logits dump format as an input to the sampler.

``verbo logits --input ids.txt --out rows.bin`` (cli/main.cpp:174-190) writes,
for every line of token ids, the ``Session::eval_all`` logits of that line:
``n x vocab`` fp32 values in native byte order, lines concatenated, no header.
A dump is therefore a ``[rows, vocab]`` fp32 array once the model's vocabulary
is known.  These helpers read and write that layout so that real-model rows
can be fed to the CUDA sampler (and to the parity tests) as they come out of
the reference.
"""
from __future__ import annotations

from pathlib import Path
from typing import Union

import numpy as np

PathLike = Union[str, Path]


def read_dump(path: PathLike, vocab: int) -> np.ndarray:
    """The rows of a dump as a C-contiguous float32 array [rows, vocab]."""
    if vocab < 1:
        raise ValueError("vocab must be >= 1")
    data = np.fromfile(path, dtype=np.float32)
    if data.size % vocab:
        raise ValueError(f"{path}: {data.size} floats is not a whole number of rows of {vocab}")
    return data.reshape(-1, vocab)


def write_dump(path: PathLike, rows: np.ndarray) -> None:
    """Writes rows [n, vocab] in the dump layout (appending is the caller's choice)."""
    np.ascontiguousarray(rows, dtype=np.float32).tofile(path)


def sample_dump(path: PathLike, vocab: int, opts, rng=None, hist=None, hist_off=None, device: str = "cuda"):
    """Reads a dump and samples every row on the GPU (verbo_b200.sample)."""
    import torch

    import verbo_b200 as vb

    x = torch.from_numpy(read_dump(path, vocab)).to(device)
    return vb.sample(x, opts, rng=rng, hist=hist, hist_off=hist_off)
