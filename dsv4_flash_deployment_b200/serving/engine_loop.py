"""The engine thread behind the HTTP server.

One thread owns the :class:`..engine.engine.Engine` (its CUDA stream, graphs
and scheduler) and runs continuous-batching steps while any request is live.
HTTP handlers talk to it through a thread-safe inbox (add / cancel) and read
tokens from a per-request :class:`TokenStream` that the engine thread fills
with ``loop.call_soon_threadsafe``.  Many requests share each step, which is
what the reference's one-request-at-a-time server
(``tpu-v7x/deepseek_v41/server.py:44-150``, a lock around
``spmd_generate_greedy``) does not do; vLLM's async engine plays this role
for the vLLM-served recipes.

Watchdog: a step that raises, or runs longer than ``step_deadline_s``, fails
every live request with a server error and marks the engine unhealthy
(``/health`` answers 503) instead of hanging the clients.
"""

from __future__ import annotations

import asyncio
import queue
import threading
import time
from collections import deque
from dataclasses import dataclass, field


@dataclass
class GenParams:
    max_tokens: int
    ignore_eos: bool = False
    stop_ids: tuple[int, ...] = ()
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    logprobs: int | None = None     # alternatives per token (None: no log-probabilities)
    seed: int | None = None


@dataclass
class TokenStream:
    loop: asyncio.AbstractEventLoop
    q: asyncio.Queue = field(default_factory=asyncio.Queue)
    req: object = None
    t_submit: float = field(default_factory=time.perf_counter)

    def put(self, item) -> None:
        self.loop.call_soon_threadsafe(self.q.put_nowait, item)


def _deliver(items) -> None:
    for q, item in items:
        q.put_nowait(item)


class _Outbox:
    """A step's stream items, handed to each event loop in one call: one wake-up of
    the HTTP thread per step instead of one per generated token (each
    ``call_soon_threadsafe`` writes to the loop's wake-up pipe and takes the lock
    of its ready queue)."""

    def __init__(self):
        self.by_loop: dict = {}

    def put(self, s: TokenStream, item) -> None:
        self.by_loop.setdefault(s.loop, []).append((s.q, item))

    def flush(self) -> None:
        for loop, items in self.by_loop.items():
            loop.call_soon_threadsafe(_deliver, items)
        self.by_loop = {}


class EngineLoop:
    def __init__(self, engine, step_deadline_s: float = 600.0, idle_wait_s: float = 0.002):
        self.engine = engine
        self.inbox: queue.SimpleQueue = queue.SimpleQueue()
        self.step_deadline_s = step_deadline_s
        self.idle_wait_s = idle_wait_s
        self.healthy = True
        self.draining = False         # set by drain(): new requests are refused, live ones finish
        self.error: str | None = None
        self._stop = threading.Event()
        self._wake = threading.Event()
        self._live: dict[int, TokenStream] = {}
        self.stats = {"requests": 0, "finished": 0, "failed": 0, "generated_tokens": 0, "prompt_tokens": 0,
                      "steps": 0, "step_time_s": 0.0, "last_step_ms": 0.0, "last_batch_tokens": 0}
        self.step_ms_window: deque = deque(maxlen=1024)
        self.ttft_window: deque = deque(maxlen=1024)
        self.thread = threading.Thread(target=self._run, name="engine-loop", daemon=True)

    # ------------------------------------------------------------ client API
    def start(self) -> "EngineLoop":
        self.thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        self._wake.set()
        self.thread.join(timeout=30)

    def drain(self, timeout_s: float = 30.0) -> bool:
        """Graceful shutdown: refuse new requests and wait (up to ``timeout_s``) for
        the live ones to finish.  Returns True when none is left."""
        self.draining = True
        deadline = time.perf_counter() + timeout_s
        while time.perf_counter() < deadline:
            if not self._live and self.inbox.empty():
                return True
            time.sleep(0.01)
        return not self._live

    def submit(self, prompt: list[int], params: GenParams) -> TokenStream:
        s = TokenStream(asyncio.get_running_loop())
        self.inbox.put(("add", prompt, params, s))
        self._wake.set()
        return s

    def cancel(self, s: TokenStream) -> None:
        self.inbox.put(("cancel", s))
        self._wake.set()

    @property
    def n_live(self) -> int:
        return len(self._live)

    # ----------------------------------------------------------- engine side
    def _drain(self) -> None:
        eng = self.engine
        while True:
            try:
                msg = self.inbox.get_nowait()
            except queue.Empty:
                return
            if msg[0] == "add":
                _, prompt, p, s = msg
                if not self.healthy:
                    s.put(("error", f"engine unhealthy: {self.error}"))
                    continue
                if self.draining:
                    s.put(("error", "the server is shutting down"))
                    continue
                try:
                    # the filtering / log-probability options only when asked for, so an
                    # engine front that does not take them still serves the rest
                    kw = {}
                    if p.top_k or p.top_p < 1.0 or p.logprobs is not None or p.seed is not None:
                        kw = {"top_k": p.top_k, "top_p": p.top_p, "logprobs": p.logprobs, "seed": p.seed}
                    req = eng.add_request(prompt, p.max_tokens, ignore_eos=p.ignore_eos, stop_ids=p.stop_ids,
                                          temperature=p.temperature, **kw)
                except (ValueError, TypeError) as e:
                    s.put(("error", str(e)))
                    continue
                s.req = req
                self._live[req.req_id] = s
                self.stats["requests"] += 1
                self.stats["prompt_tokens"] += len(prompt)
            elif msg[0] == "cancel":
                s = msg[1]
                if s.req is not None and not s.req.finished:
                    eng.sched.cancel(s.req)

    def _fail_all(self, why: str) -> None:
        for s in self._live.values():
            s.put(("error", why))
        self.stats["failed"] += len(self._live)
        self._live.clear()

    def _run(self) -> None:
        eng = self.engine
        beat = getattr(eng, "heartbeat", None)
        last_beat = time.perf_counter()
        while not self._stop.is_set():
            self._drain()
            if eng.sched.idle or not self.healthy:
                self._wake.wait(timeout=0.05)
                self._wake.clear()
                # keep the other ranks' control collectives inside their timeout
                if beat is not None and self.healthy and time.perf_counter() - last_beat > 1.0:
                    try:
                        beat()
                    except Exception as e:  # noqa: BLE001
                        self.healthy = False
                        self.error = f"control plane: {type(e).__name__}: {e}"
                    last_beat = time.perf_counter()
                continue
            t0 = time.perf_counter()
            try:
                events = eng.step()
            except Exception as e:  # noqa: BLE001
                self.healthy = False
                self.error = f"{type(e).__name__}: {e}"
                self._fail_all(self.error)
                continue
            dt = time.perf_counter() - t0
            self.stats["steps"] += 1
            self.stats["step_time_s"] += dt
            self.stats["last_step_ms"] = dt * 1e3
            self.step_ms_window.append(dt * 1e3)
            self.stats["last_batch_tokens"] = eng.stats.get("last_T", 0)
            if dt > self.step_deadline_s:
                self.healthy = False
                self.error = f"step took {dt:.1f} s (deadline {self.step_deadline_s} s)"
            out = _Outbox()
            for req, tok in events:
                s = self._live.get(req.req_id)
                if s is None:
                    continue
                if tok is not None:
                    self.stats["generated_tokens"] += 1
                    if len(req.output) == 1:
                        self.ttft_window.append(time.perf_counter() - s.t_submit)
                    lps = getattr(req, "logprobs", None)
                    lp = lps[len(req.output) - 1] if lps and len(lps) >= len(req.output) else None
                    out.put(s, ("token", (tok, lp)))
            # finished (length / stop / cancelled) requests
            for rid in [rid for rid, s in self._live.items() if s.req.finished]:
                s = self._live.pop(rid)
                self.stats["finished"] += 1
                out.put(s, ("done", s.req.finish_reason))
            out.flush()
            if not self.healthy:
                self._fail_all(self.error)
