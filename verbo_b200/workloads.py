"""Synthetic logits workloads for the sampling path.

The reference publishes no sampler benchmark, so the five configurations
below (C1-C5) are seeded synthetic stand-ins with the shapes, value
distributions and sampling options of the benchmark plan:

=====  ==============  ==============================================  ========================================  ==========
name   rows x vocab    logits                                          options                                   history
=====  ==============  ==============================================  ========================================  ==========
c1     1 x 49152       N(0, 3^2)                                       temp .7 top_k 40 top_p .9 min_p .05 rep 1.1  64 ids
c2     256 x 151936    N(0, 2^2)                                       greedy, repeat 1.2                        128 ids
c3     1024 x 151936   log(rank^-1.1) + N(0, .1^2), permuted per row   temp .8 top_k 50 top_p .95 rep 1.1        256 ids
c4     4096 x 151936   N(0, .5^2)                                      temp 1.5 top_k 0 top_p .99                none
c5     512 x 151936    N(0, 3^2), 8 column shards of 18992             temp .9 top_k 64 top_p .9 min_p .1 rep 1.15  1024 ids
=====  ==============  ==============================================  ========================================  ==========

History ids are uniform in [0, vocab).  The penalty window equals the history
length (repeat_last = H), so the whole history is penalised.  Row r of a
config with data seed s uses the non-zero sampler seed ``(s << 32) | (r + 1)``
(the reference seeds 0 from the clock, src/sampler.cpp:27).

Two generators produce the same *distribution*: numpy (host, for parity
tests and fixtures, exact and seeded) and torch (device, for the benchmark,
where a few GB of rows must be made quickly).
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Optional

import numpy as np


@dataclass(frozen=True)
class Workload:
    name: str
    rows: int
    vocab: int
    dist: str            # "normal" | "zipf"
    scale: float         # std of the normal, or of the zipf noise
    data_seed: int
    temp: float
    top_k: int
    top_p: float
    min_p: float
    repeat: float
    hist_len: int
    shards: int = 1

    @property
    def repeat_last(self) -> int:
        return self.hist_len if self.hist_len > 0 else 64

    def sampling_kwargs(self) -> dict:
        return dict(temp=self.temp, top_k=self.top_k, top_p=self.top_p, min_p=self.min_p,
                    repeat=self.repeat, repeat_last=self.repeat_last)

    def with_rows(self, rows: int) -> "Workload":
        return replace(self, rows=rows)

    def sampler_seeds(self, row0: int = 0, rows: Optional[int] = None) -> np.ndarray:
        rows = self.rows if rows is None else rows
        r = np.arange(row0, row0 + rows, dtype=np.uint64)
        return (np.uint64(self.data_seed) << np.uint64(32)) | (r + np.uint64(1))


WORKLOADS = {
    "c1": Workload("c1", 1, 49152, "normal", 3.0, 0, 0.7, 40, 0.9, 0.05, 1.1, 64),
    "c2": Workload("c2", 256, 151936, "normal", 2.0, 1, 0.0, 40, 0.9, 0.0, 1.2, 128),
    "c3": Workload("c3", 1024, 151936, "zipf", 0.1, 2, 0.8, 50, 0.95, 0.0, 1.1, 256),
    "c4": Workload("c4", 4096, 151936, "normal", 0.5, 3, 1.5, 0, 0.99, 0.0, 1.0, 0),
    # C5 names no top_p: the reference's default, 0.9 (include/verbo/verbo.hpp:58), applies
    "c5": Workload("c5", 512, 151936, "normal", 3.0, 4, 0.9, 64, 0.9, 0.1, 1.15, 1024, shards=8),
}


def make_rows_np(w: Workload, rows: Optional[int] = None, row0: int = 0) -> np.ndarray:
    """Host logits rows [row0, row0+rows) of workload `w` (float32, C order)."""
    rows = w.rows if rows is None else rows
    out = np.empty((rows, w.vocab), dtype=np.float32)
    for i in range(rows):
        g = np.random.default_rng([w.data_seed, row0 + i])
        if w.dist == "normal":
            out[i] = g.standard_normal(w.vocab, dtype=np.float32) * np.float32(w.scale)
        else:
            rank = np.arange(1, w.vocab + 1, dtype=np.float64)
            base = (-1.1 * np.log(rank)).astype(np.float32)
            noisy = base + g.standard_normal(w.vocab, dtype=np.float32) * np.float32(w.scale)
            out[i] = noisy[g.permutation(w.vocab)]
    return out


def make_hist_np(w: Workload, rows: Optional[int] = None, row0: int = 0):
    """CSR histories (hist int32, hist_off int64) or (None, None)."""
    rows = w.rows if rows is None else rows
    if w.hist_len <= 0:
        return None, None
    g = np.random.default_rng([w.data_seed, 1 << 20, row0])
    hist = g.integers(0, w.vocab, size=rows * w.hist_len, dtype=np.int32)
    off = np.arange(rows + 1, dtype=np.int64) * w.hist_len
    return hist, off


def make_rows_torch(w: Workload, rows: int, device, seed_offset: int = 0):
    """Device logits with the distribution of `w` (not bit-identical to numpy)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(w.data_seed * 1000003 + seed_offset)
    if w.dist == "normal":
        return torch.randn(rows, w.vocab, device=device, generator=g, dtype=torch.float32) * w.scale
    rank = torch.arange(1, w.vocab + 1, device=device, dtype=torch.float64)
    base = (-1.1 * torch.log(rank)).to(torch.float32)
    out = torch.empty(rows, w.vocab, device=device, dtype=torch.float32)
    chunk = 256
    for r0 in range(0, rows, chunk):
        n = min(chunk, rows - r0)
        perm = torch.argsort(torch.rand(n, w.vocab, device=device, generator=g), dim=1)
        noisy = base.unsqueeze(0) + torch.randn(n, w.vocab, device=device, generator=g) * w.scale
        out[r0:r0 + n] = torch.gather(noisy, 1, perm)
    return out


def make_hist_torch(w: Workload, rows: int, device, seed_offset: int = 0):
    import torch

    if w.hist_len <= 0:
        return None, None
    g = torch.Generator(device=device)
    g.manual_seed(w.data_seed * 7919 + seed_offset + 17)
    hist = torch.randint(0, w.vocab, (rows * w.hist_len,), device=device, generator=g, dtype=torch.int32)
    off = torch.arange(rows + 1, device=device, dtype=torch.int64) * w.hist_len
    return hist, off


# ------------------------------------------------------------ logits tail --
@dataclass(frozen=True)
class TailWorkload:
    """The logits producer tail (src/session.cpp:163-169) on a Qwen2-0.5B-shaped
    head: vocab x dim weights in verbo::Tensor layout (src/kernels.hpp:13-23),
    seeded synthetic values with the ranges the reference's quant_rows gives
    (Q8 codes in [-127, 127], Q4 nibbles in [0, 15], positive fp16 scales),
    a norm weight near 1 and hidden rows N(0, scale^2).  The default batch is
    one row: one decode step of the reference's generate loop."""
    name: str = "tail"
    rows: int = 1
    vocab: int = 151936
    dim: int = 896
    dtype: str = "q8"
    eps: float = 1e-6
    scale: float = 3.0
    data_seed: int = 5

    def with_rows(self, rows: int) -> "TailWorkload":
        return replace(self, rows=rows)

    def with_dtype(self, dtype: str) -> "TailWorkload":
        return replace(self, dtype=dtype)

    def head_bytes(self) -> int:
        """Bytes of the head the kernel must read once per call."""
        if self.dtype == "f32":
            return self.vocab * self.dim * 4
        q = self.vocab * self.dim if self.dtype == "q8" else self.vocab * self.dim // 2
        return q + self.vocab * (self.dim // 32) * 2

    def make_head(self):
        """(q, s, norm) host arrays of the head."""
        g = np.random.default_rng(self.data_seed)
        norm = (1.0 + 0.1 * g.standard_normal(self.dim)).astype(np.float32)
        if self.dtype == "f32":
            return (g.standard_normal((self.vocab, self.dim)) * 0.05).astype(np.float32), None, norm
        s = (np.abs(g.standard_normal((self.vocab, self.dim // 32))) * 0.004 + 1e-4).astype(np.float16)
        if self.dtype == "q8":
            q = g.integers(-127, 128, size=(self.vocab, self.dim), dtype=np.int8)
        else:
            q = g.integers(0, 256, size=(self.vocab, self.dim // 2), dtype=np.uint8)
        return q, s.view(np.uint16), norm

    def make_hidden_np(self, rows: Optional[int] = None, seed_offset: int = 0) -> np.ndarray:
        rows = self.rows if rows is None else rows
        g = np.random.default_rng(self.data_seed * 1000 + 7 + seed_offset)
        return (g.standard_normal((rows, self.dim)) * self.scale).astype(np.float32)


TAIL = TailWorkload()
