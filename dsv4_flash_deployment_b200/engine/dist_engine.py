"""Multi-rank serving control plane (one process per GPU, rank 0 fronts the API).

Attention is data-parallel: every request lives on one rank (its cache slot,
its scheduler), while the MoE exchanges tokens between all ranks inside each
model step, so all ranks step in lockstep.  Per step:

  rank 0   broadcast  {adds for each rank, cancels, any_work}     (CPU group)
  all      apply the adds/cancels to the local scheduler; if any rank has
           work, run a real step (or a 1-token dummy step on a reserved slot
           when this rank has none, to join the step's collectives)
  all      gather     [(request id, token, finished, reason, logprob)] -> rank 0

The messages travel on a control channel (engine/control.py): by default a
shared-memory file for the ranks of one node (tens of microseconds per round
trip), or the CPU process group (gloo; milliseconds, across nodes).

Rank 0 assigns new requests to the rank with the fewest live requests.  In the
replicated mode (tensor-parallel layout) every request goes to every rank: the
local schedulers see the same adds and cancels in the same order, so they
build the same step, the tensor-parallel kernels exchange their partials, and
only rank 0 reports tokens (all ranks hold the same ones).  The
control messages travel on a gloo group so they never queue behind NCCL
kernels.  A rank that dies or stalls makes the next control collective fail
after the group's timeout; rank 0 raises, and the HTTP layer fails the live
requests and reports unhealthy.

Reference: the coordinator/worker lockstep of ``tpu-v7x/deepseek_v41/
engine.py:602-632`` (``broadcast_one_to_all`` of a header + padded ids) and
``server.py:1-5``; Ray + vLLM multihost for the vLLM recipes.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

from ..models.model import SeqChunk, StepMeta
from .control import GlooControl


@dataclass
class GlobalRequest:
    req_id: int
    rank: int
    prompt: list[int]
    max_new_tokens: int
    output: list[int] = field(default_factory=list)
    finished: bool = False
    finish_reason: str | None = None
    cancelled: bool = False
    t_arrival: float = field(default_factory=time.perf_counter)
    t_first_token: float | None = None
    t_done: float | None = None
    logprobs: list = field(default_factory=list)   # per token when the request asked for them


class _SchedView:
    """What the engine loop and /metrics read from a scheduler, over all ranks."""

    def __init__(self, de: "DistributedEngine"):
        self.de = de

    @property
    def idle(self) -> bool:
        return not self.de.live and not self.de.pending_adds

    def cancel(self, req: GlobalRequest) -> None:
        req.cancelled = True
        self.de.pending_cancels.append(req.req_id)

    @property
    def running(self):
        return list(self.de.live.values())

    @property
    def waiting(self):
        return list(self.de.pending_adds)

    @property
    def max_seqs(self) -> int:
        return (1 if self.de.replicated else self.de.world) * self.de.local.sched.max_seqs

    @property
    def slots(self):
        de = self.de

        class _S:
            n_free = max(0, (1 if de.replicated else de.world) * de.local.sched.max_seqs - len(de.live))
        return _S()


def _local_step(engine, msg: dict, rank: int, id_map: dict, pad_slot: int, replicated: bool = False) -> list[tuple]:
    """Applies a control message to this rank's engine and runs its part of the step."""
    for gid, r, prompt, mt, ignore_eos, stop_ids, temperature, extra in msg["adds"]:
        if r == rank or r == -1:
            req = engine.add_request(prompt, mt, ignore_eos=ignore_eos, stop_ids=stop_ids, temperature=temperature,
                                     **extra)
            id_map[req.req_id] = gid
            id_map[("g", gid)] = req
    for gid in msg["cancels"]:
        req = id_map.get(("g", gid))
        if req is not None:
            engine.sched.cancel(req)
    if not msg["any_work"]:
        return []
    before = engine.stats["steps"]
    events = engine.step() if not engine.sched.idle else []
    if engine.stats["steps"] == before and not replicated:
        # no local forward ran: join the step's collectives with a 1-token step on the reserved slot
        engine.run_meta(StepMeta(engine.cfg, [SeqChunk(pad_slot, 0, [0], True)]))
        engine.stats["dummy_steps"] = engine.stats.get("dummy_steps", 0) + 1
    out = []
    for req, tok in events:
        gid = id_map.get(req.req_id)
        lp = req.logprobs[len(req.output) - 1] if tok is not None and req.logprobs else None
        out.append((gid, tok, req.finished, req.finish_reason, lp))
    # requests finished without an event this step (cancelled before scheduling)
    for key in [k for k in id_map if isinstance(k, tuple)]:
        req = id_map[key]
        if req.finished:
            if not any(e[0] == key[1] for e in out):
                out.append((key[1], None, True, req.finish_reason, None))
            del id_map[key]
            id_map.pop(req.req_id, None)
    if replicated and rank != 0:
        return []   # every rank produced the same tokens; rank 0 reports them
    return out


class DistributedEngine:
    """Rank-0 front with the :class:`.engine.Engine` API over all ranks."""

    def __init__(self, local_engine, cpu_group=None, pad_slot: int | None = None, replicated: bool = False,
                 control=None):
        self.local = local_engine
        self.replicated = replicated
        self.cfg = local_engine.cfg
        self.group = cpu_group
        self.ctl = control if control is not None else GlooControl(cpu_group)
        self.rank = self.ctl.rank
        self.world = self.ctl.world
        self.pad_slot = local_engine.sched.max_seqs if pad_slot is None else pad_slot
        self.live: dict[int, GlobalRequest] = {}
        self.pending_adds: list[GlobalRequest] = []
        self.pending_cancels: list[int] = []
        self.load = [0] * self.world
        self.next_id = 0
        self.id_map: dict = {}
        self.sched = _SchedView(self)
        self.stats = {"steps": 0, "dummy_steps": 0, "graph_captures": 0}
        self.eos_id = local_engine.eos_id

    def add_request(self, prompt: list[int], max_new_tokens: int, ignore_eos: bool = False,
                    stop_ids=(), temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                    logprobs: int | None = None, seed: int | None = None) -> GlobalRequest:
        if not prompt:
            raise ValueError("empty prompt")
        # checked here, on rank 0, so that no rank is sent a request its engine refuses
        sp = self.local.sampling_params(temperature, top_k, top_p, logprobs, seed)
        if len(prompt) + max_new_tokens > self.local.sched.max_seq_len:
            raise ValueError(f"prompt {len(prompt)} + {max_new_tokens} new tokens exceeds max_seq_len "
                             f"{self.local.sched.max_seq_len}")
        kv = getattr(self.local.sched, "kv", None)
        if kv is not None and not kv.fits(len(prompt) + max_new_tokens):
            raise ValueError(f"prompt {len(prompt)} + {max_new_tokens} new tokens exceeds the paged cache pool")
        r = -1 if self.replicated else min(range(self.world), key=lambda i: self.load[i])
        g = GlobalRequest(self.next_id, r, list(prompt), max_new_tokens)
        extra = {} if not (sp.top_k or sp.top_p < 1.0 or sp.wants_logprobs or sp.seed is not None) else \
            {"top_k": sp.top_k, "top_p": sp.top_p, "logprobs": sp.logprobs, "seed": sp.seed}
        g._opts = (bool(ignore_eos), tuple(stop_ids), sp.temperature, extra)
        self.next_id += 1
        self.load[r] += 1
        self.pending_adds.append(g)
        return g

    def step(self) -> list[tuple[GlobalRequest, int | None]]:
        adds = [(g.req_id, g.rank, g.prompt, g.max_new_tokens, *g._opts) for g in self.pending_adds]
        for g in self.pending_adds:
            self.live[g.req_id] = g
        self.pending_adds = []
        msg = {"adds": adds, "cancels": self.pending_cancels, "any_work": bool(self.live), "stop": False}
        self.pending_cancels = []
        self.ctl.broadcast(msg)
        mine = _local_step(self.local, msg, 0, self.id_map, self.pad_slot, self.replicated)
        gathered = self.ctl.gather(mine)
        now = time.perf_counter()
        events = []
        for evs in gathered:
            for gid, tok, fin, reason, lp in evs or []:
                g = self.live.get(gid)
                if g is None:
                    continue
                if tok is not None:
                    g.output.append(int(tok))
                    if lp is not None:
                        g.logprobs.append(lp)
                    if g.t_first_token is None:
                        g.t_first_token = now
                if fin:
                    g.finished, g.finish_reason, g.t_done = True, reason, now
                    if g.rank >= 0:
                        self.load[g.rank] -= 1
                    del self.live[gid]
                events.append((g, tok))
        self.stats["steps"] += 1
        self.stats["last_T"] = self.local.stats.get("last_T", 0)
        self.stats["graph_captures"] = self.local.stats.get("graph_captures", 0)
        return events

    def heartbeat(self) -> None:
        """An empty control step (no model step when no rank has work)."""
        self.step()

    def shutdown(self) -> None:
        self.ctl.broadcast({"adds": [], "cancels": [], "any_work": False, "stop": True})
        self.ctl.close()

    def generate(self, prompts: list[list[int]], max_new_tokens: int, ignore_eos: bool = False,
                 **sampling) -> list[list[int]]:
        reqs = [self.add_request(p, max_new_tokens, ignore_eos, **sampling) for p in prompts]
        while not all(r.finished for r in reqs):
            self.step()
        return [r.output for r in reqs]


def worker_loop(local_engine, cpu_group=None, pad_slot: int | None = None, replicated: bool = False,
                control=None) -> int:
    """Ranks > 0: follow rank 0's control messages until it sends stop. Returns steps run."""
    ctl = control if control is not None else GlooControl(cpu_group)
    rank = ctl.rank
    pad = local_engine.sched.max_seqs if pad_slot is None else pad_slot
    id_map: dict = {}
    n = 0
    while True:
        msg = ctl.broadcast()
        if msg["stop"]:
            ctl.close()
            return n
        mine = _local_step(local_engine, msg, rank, id_map, pad, replicated)
        ctl.gather(mine)
        n += 1
