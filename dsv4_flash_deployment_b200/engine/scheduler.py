"""Continuous batching with chunked prefill (host side, no torch).

Plays the role of the vLLM V1 scheduler the reference serves behind
(``--max-num-seqs``, ``--max-num-batched-tokens``, chunked prefill at 256/2048
tokens per step; ``KO/dsv41-flash-v6e16-serving.yaml:360-373``).  Policy per
step: every running sequence that has finished its prompt decodes one token;
the remaining token budget goes to prompt chunks, oldest request first.  A
request enters only when a cache slot is free (``max_seqs``) and its total
length fits ``max_seq_len``.  Finished requests release their slot at once.
With paged compressed caches (``kv``: models/kv_pages.py) admission also
reserves every cache block the request can touch, oldest request first (a
request that does not fit waits at the head of the queue); finishing releases them.

``preempt=True`` (with paged caches) admits optimistically instead, as vLLM's
scheduler does: a request reserves the blocks of its prompt, and a decoding
sequence grows its reservation as it crosses block boundaries.  When the pool
cannot grow one, the most recently admitted running request is preempted: its
slot and blocks are released and it goes back to the head of the queue with
its prompt and the tokens generated so far as the context to recompute
(vLLM's recompute preemption); no request is admitted in a step that
preempted.  The oldest request always progresses, since a lone request fits
the pool (checked when it is added).
"""

from __future__ import annotations

import itertools
import time
from collections import deque
from dataclasses import dataclass, field


@dataclass
class Request:
    req_id: int
    prompt: list[int]
    max_new_tokens: int
    ignore_eos: bool = False
    eos_id: int | None = None
    stop_ids: tuple[int, ...] = ()
    temperature: float = 0.0          # 0 = greedy
    top_k: int = 0                    # 0 = off
    top_p: float = 1.0                # 1.0 = off
    want_logprobs: int | None = None  # alternatives per generated token (None: no log-probabilities)
    seed: int | None = None           # samples depend on (seed, position) only
    slot: int = -1
    n_prefilled: int = 0
    output: list[int] = field(default_factory=list)
    finished: bool = False
    finish_reason: str | None = None
    t_arrival: float = field(default_factory=time.perf_counter)
    t_first_token: float | None = None
    t_done: float | None = None
    cancelled: bool = False
    # per generated token when ``want_logprobs`` is set: {"logprob": lp, "top": [(id, lp), ...]}
    logprobs: list = field(default_factory=list)
    # recompute after a preemption: the context to prefill (prompt + the tokens
    # generated before it) and how many of ``output`` it holds
    ctx: list[int] | None = None
    folded: int = 0
    kv_len: int = 0               # tokens of context the slot's cache reservation covers
    preemptions: int = 0

    @property
    def prefill(self) -> list[int]:
        """Tokens to prefill: the prompt, or after a preemption the whole context so far."""
        return self.prompt if self.ctx is None else self.ctx

    @property
    def prompt_done(self) -> bool:
        return self.n_prefilled >= len(self.prefill)

    @property
    def position(self) -> int:
        """Next position to be written."""
        new = len(self.output) - self.folded
        return self.n_prefilled + new - (1 if new > 0 else 0)


@dataclass
class ScheduledChunk:
    req: Request
    start_pos: int
    tokens: list[int]
    sample: bool


class SlotAllocator:
    def __init__(self, n: int):
        self.free = deque(range(n))

    def alloc(self) -> int | None:
        return self.free.popleft() if self.free else None

    def release(self, s: int) -> None:
        self.free.append(s)

    @property
    def n_free(self) -> int:
        return len(self.free)


class Scheduler:
    def __init__(self, max_seqs: int, max_batched_tokens: int, max_seq_len: int, chunk_size: int | None = None,
                 kv=None, preempt: bool = False):
        self.max_seqs = max_seqs
        self.budget = max_batched_tokens
        self.max_seq_len = max_seq_len
        self.chunk = chunk_size or max_batched_tokens
        self.slots = SlotAllocator(max_seqs)
        self.kv = kv                  # paged-cache reservations (fits / reserve / release) or None
        self.preempt = bool(preempt) and kv is not None
        self.n_preempted = 0
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self._ids = itertools.count()

    def add(self, prompt: list[int], max_new_tokens: int, **kw) -> Request:
        if not prompt:
            raise ValueError("empty prompt")
        if len(prompt) + max_new_tokens > self.max_seq_len:
            raise ValueError(f"prompt {len(prompt)} + {max_new_tokens} new tokens exceeds max_seq_len {self.max_seq_len}")
        if self.kv is not None and not self.kv.fits(len(prompt) + max_new_tokens):
            raise ValueError(f"prompt {len(prompt)} + {max_new_tokens} new tokens exceeds the paged cache pool")
        r = Request(next(self._ids), list(prompt), max_new_tokens, **kw)
        self.waiting.append(r)
        return r

    def cancel(self, req: Request) -> None:
        req.cancelled = True

    def schedule(self) -> list[ScheduledChunk]:
        # drop cancelled requests
        for r in [r for r in self.running if r.cancelled]:
            self._finish(r, "cancelled")
        for r in [r for r in self.waiting if r.cancelled]:
            self._finish(r, "cancelled")
        self.waiting = deque(r for r in self.waiting if not r.cancelled)
        preempted = self._grow_or_preempt() if self.preempt else 0
        out: list[ScheduledChunk] = []
        budget = self.budget
        prefilling = []
        for r in self.running:
            if r.prompt_done:
                if budget > 0:
                    out.append(ScheduledChunk(r, r.position, [r.output[-1]], True))
                    budget -= 1
            else:
                prefilling.append(r)
        # continue partially prefilled requests first, then admit new ones
        for r in prefilling:
            if budget <= 0:
                break
            pf = r.prefill
            n = min(self.chunk, budget, len(pf) - r.n_prefilled)
            out.append(ScheduledChunk(r, r.n_prefilled, pf[r.n_prefilled:r.n_prefilled + n],
                                      r.n_prefilled + n == len(pf)))
            budget -= n
        while budget > 0 and self.waiting and self.slots.n_free > 0 and not preempted:
            r = self.waiting[0]
            pf = r.prefill
            # reserve mode: every block the request can touch; preempt mode: its context
            need = len(pf) + 1 if self.preempt else len(r.prompt) + r.max_new_tokens
            slot = self.slots.alloc()
            if self.kv is not None and not self.kv.reserve(slot, need):
                self.slots.free.appendleft(slot)
                break
            self.waiting.popleft()
            r.slot = slot
            r.kv_len = need
            self.running.append(r)
            n = min(self.chunk, budget, len(pf))
            out.append(ScheduledChunk(r, 0, pf[:n], n == len(pf)))
            budget -= n
        return out

    def _grow_or_preempt(self) -> int:
        """Grows each decoding sequence's reservation to cover the position it writes
        this step, oldest first; preempts the newest running requests while the pool
        is short.  Returns the number preempted."""
        n = 0
        for r in list(self.running):
            if r not in self.running or not r.prompt_done:
                continue
            need = r.position + 1
            if need <= r.kv_len:
                continue
            while not self.kv.reserve(r.slot, need):
                victim = self.running[-1]
                self._preempt(victim)
                n += 1
                if victim is r:
                    break
            else:
                r.kv_len = need
        return n

    def _preempt(self, r: Request) -> None:
        self.running.remove(r)
        self.kv.release(r.slot)
        self.slots.release(r.slot)
        r.slot = -1
        r.ctx = r.prompt + r.output
        r.folded = len(r.output)
        r.n_prefilled = 0
        r.kv_len = 0
        r.preemptions += 1
        self.n_preempted += 1
        self.waiting.appendleft(r)

    def commit(self, chunks: list[ScheduledChunk], next_ids: list[int]) -> list[tuple[Request, int | None]]:
        """Applies a step's results; returns (request, new token or None) per chunk."""
        events = []
        it = iter(next_ids)
        now = time.perf_counter()
        for c in chunks:
            r = c.req
            if not r.prompt_done:
                r.n_prefilled += len(c.tokens)
            tok = next(it) if c.sample else None
            if tok is not None:
                r.output.append(int(tok))
                if r.t_first_token is None:
                    r.t_first_token = now
                if len(r.output) >= r.max_new_tokens:
                    self._finish(r, "length")
                elif not r.ignore_eos and (tok == r.eos_id or tok in r.stop_ids):
                    self._finish(r, "stop")
            events.append((r, tok))
        return events

    def _finish(self, r: Request, reason: str) -> None:
        r.finished = True
        r.finish_reason = reason
        r.t_done = time.perf_counter()
        if r in self.running:
            self.running.remove(r)
        if r.slot >= 0:
            if self.kv is not None:
                self.kv.release(r.slot)
            self.slots.release(r.slot)
            r.slot = -1

    @property
    def idle(self) -> bool:
        return not self.running and not self.waiting
