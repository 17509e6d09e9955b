"""Request batching over the device-resident streams (verbo_cuda_batch_*).

The reference's server (cli/serve.cpp:139-218) runs one request at a time
behind a global mutex, each through verbo::generate (src/sampler.cpp:111-181):
accept the prompt, then pick / stop check / accept until a stop id or
max_tokens.  ``BatchServer`` keeps up to ``slots`` requests in one
``verbo_b200.Batch`` instead: a request takes a free slot (reset with its seed,
accept its prompt), every step samples all slots in one launch chain from the
rows the caller's model produced, and a request leaves its slot when it meets
a stop id (not emitted, as in generate) or its token limit, letting the next
queued request in.  Only the ids cross to the host each step; stop checks stay
on the host as in generate.  Idle slots are sampled too (their ids ignored).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence


@dataclass
class Request:
    prompt: List[int]
    max_tokens: int
    seed: int
    stop_ids: Sequence[int] = ()
    rid: int = -1
    tokens: List[int] = field(default_factory=list)
    stopped: bool = False  # ended on a stop id (else on max_tokens)


class BatchServer:
    """Continuous batching of generation requests on one GPU.

    ``model(slot_requests, out)`` fills ``out`` (CUDA float32 [slots, vocab])
    with the next logits row of each slot's request (``None`` for an idle slot,
    whose row may hold anything finite)."""

    def __init__(self, opts, slots: int, vocab: int, model: Callable, device: int = 0):
        import torch

        import verbo_b200 as vb

        self.vocab, self.slots, self.model = vocab, slots, model
        self.batch = vb.Batch(opts, slots, device)
        self.logits = torch.zeros((slots, vocab), dtype=torch.float32, device=f"cuda:{device}")
        self.ids = torch.empty(slots, dtype=torch.int32, device=f"cuda:{device}")
        self.active: List[Optional[Request]] = [None] * slots
        self.queue: deque = deque()
        self.done: Dict[int, Request] = {}
        self._next = 0

    def submit(self, prompt: Sequence[int], max_tokens: int, seed: int, stop_ids: Sequence[int] = ()) -> int:
        if seed == 0:
            raise ValueError("seed 0 means the clock in the reference; give each request its own seed")
        r = Request(list(prompt), int(max_tokens), int(seed), tuple(stop_ids), rid=self._next)
        self._next += 1
        if r.max_tokens <= 0:
            self.done[r.rid] = r
        else:
            self.queue.append(r)
        return r.rid

    def _admit(self) -> None:
        for s in range(self.slots):
            if self.active[s] is None and self.queue:
                r = self.queue.popleft()
                self.batch.reset(s, r.seed)
                self.batch.accept(s, r.prompt)
                self.active[s] = r

    def step(self) -> bool:
        """One sampling step over all slots; False when nothing is left to do."""
        self._admit()
        if not any(self.active):
            return False
        self.model(self.active, self.logits)
        ids = self.batch.step(self.logits, out=self.ids).cpu().numpy()
        for s, r in enumerate(self.active):
            if r is None:
                continue
            t = int(ids[s])
            if t in r.stop_ids:
                r.stopped = True
            else:
                r.tokens.append(t)
            if r.stopped or len(r.tokens) >= r.max_tokens:
                self.done[r.rid] = r
                self.active[s] = None
        return True

    def run(self) -> Dict[int, Request]:
        while self.step():
            pass
        return self.done
