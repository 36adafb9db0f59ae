"""DSpark speculative decoding behind the OpenAI server.

:class:`SpecServingEngine` gives :class:`.dspark.SpecEngine` the interface the
server's engine thread drives (``add_request`` / ``step`` / ``sched.idle`` /
``sched.cancel`` / ``stats``, as :class:`..engine.engine.Engine`):

* a request waits until a drafter row (a cache slot of the model) is free; it
  is then prefilled (chunked) and its first token is emitted;
* every step runs one draft + lossless verify round for all admitted requests
  together, and each request emits between one and ``block_size`` tokens;
* EOS, stop ids and the length cap end a request inside a round (tokens after
  the end are dropped); its row is released at once.

The reference serves DSpark one request at a time under a lock
(``tpu-v7x/deepseek_v41/server.py:44-150``, ``use_dspark``); here requests
share every verify step.  Decoding is greedy: a request asking for
``temperature > 0`` is refused, since the verify rule keeps the argmax chain.
"""

from __future__ import annotations

import itertools
from collections import deque

from ..engine.scheduler import Request


class _Queue:
    """The part of the scheduler interface the engine thread uses."""

    def __init__(self, owner: "SpecServingEngine"):
        self.o = owner

    @property
    def idle(self) -> bool:
        return not self.o.waiting and not self.o.active

    @property
    def running(self) -> list:
        return list(self.o.active.values())

    @property
    def waiting(self):
        return self.o.waiting

    @property
    def max_seqs(self) -> int:
        return self.o.spec.max_seqs

    @property
    def slots(self):
        return self

    @property
    def n_free(self) -> int:
        return len(self.o.free_rows)

    def cancel(self, req: Request) -> None:
        req.cancelled = True
        if req in self.o.waiting:
            self.o.waiting.remove(req)
            self.o._finish(req, "abort")


class SpecServingEngine:
    def __init__(self, spec, max_seq_len: int, eos_id: int | None = None):
        self.spec = spec
        self.cfg = spec.cfg
        self.max_seq_len = max_seq_len
        self.eos_id = self.cfg.eos_token_id if eos_id is None else eos_id
        self.waiting: deque[Request] = deque()
        self.active: dict[int, Request] = {}
        self.free_rows = deque(range(spec.max_seqs))
        self.sched = _Queue(self)
        self._ids = itertools.count()
        self.stats = {"steps": 0, "tokens": 0, "rounds": 0, "last_T": 0}
        spec.open_rows()

    def add_request(self, prompt: list[int], max_new_tokens: int, ignore_eos: bool = False,
                    stop_ids=(), temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                    logprobs: int | None = None, seed: int | None = None) -> Request:
        if temperature > 0:
            raise ValueError("speculative decoding (DSpark) decodes greedily; temperature > 0 is not supported")
        if logprobs is not None:
            raise ValueError("speculative decoding (DSpark) does not return logprobs")
        if not prompt:
            raise ValueError("empty prompt")
        if len(prompt) + max_new_tokens + self.spec.blk > self.max_seq_len:
            raise ValueError(f"prompt + max_tokens + draft block exceeds max_model_len {self.max_seq_len}")
        r = Request(next(self._ids), list(prompt), max_new_tokens, ignore_eos=ignore_eos, eos_id=self.eos_id,
                    stop_ids=tuple(stop_ids))
        self.waiting.append(r)
        return r

    def _finish(self, r: Request, reason: str) -> None:
        r.finished = True
        r.finish_reason = reason

    def _emit(self, r: Request, toks: list[int], events: list) -> None:
        for t in toks:
            if r.finished:
                break
            r.output.append(t)
            events.append((r, t))
            if not r.ignore_eos and r.eos_id is not None and t == r.eos_id:
                self._finish(r, "stop")
            elif t in r.stop_ids:
                self._finish(r, "stop")
            elif len(r.output) >= r.max_new_tokens:
                self._finish(r, "length")

    def step(self) -> list[tuple[Request, int | None]]:
        events: list = []
        sp = self.spec
        while self.waiting and self.free_rows:
            r = self.waiting.popleft()
            j = self.free_rows.popleft()
            r.slot = j
            self.active[j] = r
            r.n_prefilled = len(r.prompt)
            first = sp.add_sequence(j, r.prompt)
            self.stats["tokens"] += len(r.prompt)
            self._emit(r, [first], events)
        act = [j for j, r in self.active.items() if not r.finished and not r.cancelled]
        if act:
            emitted = sp.round(act, [self.active[j].max_new_tokens for j in act])
            self.stats["rounds"] += 1
            self.stats["last_T"] = len(act) * sp.blk
            self.stats["tokens"] += len(act) * sp.blk
            for j, toks in zip(act, emitted):
                self._emit(self.active[j], toks, events)
        for j in [j for j, r in self.active.items() if r.finished or r.cancelled]:
            r = self.active.pop(j)
            if not r.finished:
                self._finish(r, "abort")
            sp.release_row(j)
            self.free_rows.append(j)
        self.stats["steps"] += 1
        self.stats["spec"] = sp.stats.as_dict()
        return events
