"""Request batching for a server, over the library's verbo_cuda_server_*.

The reference's server (cli/serve.cpp:139-218) runs one request at a time
behind a global mutex (:168), each through verbo::generate
(src/sampler.cpp:111-181) with the request's own Sampling (:149-157): accept
the prompt, then pick / stop check / accept until a stop id or max_tokens.
``BatchServer`` keeps up to ``slots`` requests in flight in one
``verbo_b200.Server`` instead: a request takes a free row (its Sampler seeded
with its seed, its prompt accepted), every step samples all rows from the
logits rows the caller's model produced, one launch chain per option set, and
a request leaves when it meets a stop id (not emitted, as in generate) or its
token limit, letting the next queued request in.  Only the ids cross to the
host each step; the scheduling itself is the C ABI's, so a C++ server can drive
the same object (verbo_cuda_server_prepare / _step / _result).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence


@dataclass
class Request:
    prompt: List[int]
    max_tokens: int
    seed: int
    opts: object = None
    rid: int = -1
    tokens: List[int] = field(default_factory=list)
    stopped: bool = False  # ended on a stop id (else on max_tokens)


class BatchServer:
    """Continuous batching of generation requests on one GPU.

    ``model(row_requests, out)`` fills ``out`` (CUDA float32 [slots, vocab])
    with the next logits row of each row's request (``None`` for an idle row,
    whose row may hold anything finite).  ``opts`` is the default Sampling; a
    request may bring its own.  ``stop_ids`` is the model's stop set."""

    def __init__(self, opts, slots: int, vocab: int, model: Callable, device: int = 0, stop_ids: Sequence[int] = (),
                 max_window: int = 256):
        import torch

        import verbo_b200 as vb

        self.opts, self.vocab, self.slots, self.model = opts, vocab, slots, model
        self.server = vb.Server(slots, vocab, max_window=max_window, stop_ids=stop_ids, device=device)
        self.logits = torch.zeros((slots, vocab), dtype=torch.float32, device=f"cuda:{device}")
        self.reqs: Dict[int, Request] = {}
        self.done: Dict[int, Request] = {}

    def submit(self, prompt: Sequence[int], max_tokens: int, seed: int, opts=None) -> int:
        import dataclasses

        if seed == 0:
            raise ValueError("seed 0 means the clock in the reference; give each request its own seed")
        o = dataclasses.replace(opts if opts is not None else self.opts, seed=int(seed))
        rid = self.server.submit(list(prompt), o, int(max_tokens))
        r = Request(list(prompt), int(max_tokens), int(seed), o, rid=rid)
        if r.max_tokens <= 0:
            self.server.result(rid, release=True)
            self.done[rid] = r
        else:
            self.reqs[rid] = r
        return rid

    def step(self) -> bool:
        """One sampling step over the active rows; False when nothing is left."""
        rows, n = self.server.prepare()
        if n == 0:
            return False
        active: List[Optional[Request]] = [self.reqs[int(rid)] if rid >= 0 else None for rid in rows]
        self.model(active, self.logits)
        self.server.step(self.logits)
        for r in active[:n]:
            finished, ids, stopped = self.server.result(r.rid, release=True)
            r.tokens = ids
            if finished:
                r.stopped = stopped
                self.done[r.rid] = self.reqs.pop(r.rid)
        return True

    def run(self) -> Dict[int, Request]:
        while self.step():
            pass
        return self.done
