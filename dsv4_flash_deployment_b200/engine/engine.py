"""Serving engine: scheduler + model step + CUDA-graph replay.

Public API (what the server, the benchmark and users call):

    eng = Engine.build(cfg, ...)                  # random-init or checkpoint weights
    req = eng.add_request(prompt_ids, max_new_tokens, ignore_eos=True)
    events = eng.step()                           # one continuous-batching step
    outs = eng.generate([prompt, ...], max_new_tokens)

Each step: the scheduler picks decode tokens and prompt chunks, the host
builds :class:`StepMeta`, copies it from pinned memory to the device, the
model step runs (replayed from a CUDA graph captured per batch shape), and the
sampled token ids come back to the host.  The step is the reference engine's
``generate_greedy`` inner loop (deepseek_v41/engine.py:384-475) generalized to
many sequences, and the vLLM scheduler loop for the vLLM-served recipes.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Iterable

import torch

from ..models.model import DSV4Model, SeqChunk, StepMeta
from ..models.sampling import SamplingParams, logprob_entries
from ..ops.gemm import ErrorWord
from .scheduler import Request, Scheduler


class Engine:
    """``bucket``: graph-replayed steps are padded to bucketed token / sampled-row
    counts (``StepMeta.padded``), so a serving run with changing batch
    compositions replays a few dozen graphs instead of capturing one per
    composition.  ``max_graphs`` bounds the graph cache (least recently used
    graph released first).  ``preempt``: with paged caches, admit on the
    prompt's blocks and preempt (recompute) the newest request when the pool
    runs short, instead of reserving every block up front (engine/scheduler.py)."""

    def __init__(self, model: DSV4Model, max_seqs: int, max_batched_tokens: int, max_seq_len: int,
                 chunk_size: int | None = None, use_graphs: bool = True, eos_id: int | None = None,
                 bucket: bool = True, max_graphs: int = 48, preempt: bool = False):
        self.model = model
        self.cfg = model.cfg
        self.sched = Scheduler(max_seqs, max_batched_tokens, max_seq_len, chunk_size,
                               kv=getattr(model, "pager", None), preempt=preempt)
        self.use_graphs = use_graphs and model.dev.type == "cuda"
        self.bucket = bucket
        self.max_graphs = max(1, max_graphs)
        self.graphs: OrderedDict = OrderedDict()
        self.pinned: dict = {}
        self.eos_id = self.cfg.eos_token_id if eos_id is None else eos_id
        self.stream = torch.cuda.Stream(model.dev) if model.dev.type == "cuda" else None
        self.stats = {"steps": 0, "tokens": 0, "graph_captures": 0, "graph_evictions": 0, "padded_tokens": 0}

    # ----------------------------------------------------------------- build
    @classmethod
    def build(cls, cfg, device="cuda", max_seqs: int = 16, max_batched_tokens: int = 512, max_seq_len: int = 2048,
              weights: dict | None = None, seed: int = 0, expert_storage_layers: int | None = None, ep=None,
              use_graphs: bool = True, chunk_size: int | None = None, extra_slots: int = 0, tp=None,
              experts_from=None, kv_block: int = 0, kv_pool_tokens: int = 0, engram_from=None,
              engram_shm: str | None = None, engram_token_map=None, kv_preempt: bool = False) -> "Engine":
        """``extra_slots`` cache slots beyond ``max_seqs`` are kept out of the scheduler
        (the multi-rank control plane runs its 1-token join steps on one).  ``tp``:
        tensor-parallel group (every rank runs the same steps).  ``experts_from``: a
        model whose expert blocks this one shares (same expert ownership per rank).
        ``kv_block`` / ``kv_pool_tokens``: paged compressed caches (admission then
        also waits for free blocks; ``kv_preempt``: optimistic admission with
        recompute preemption instead).  ``engram_token_map``: compressed token map of
        the tokenizer for the Engram hashes (None: ``id % C``)."""
        from .builder import build_model
        model = build_model(cfg, device, max_tokens=max_batched_tokens, n_slots=max_seqs + extra_slots,
                            max_seq_len=max_seq_len, weights=weights, seed=seed,
                            expert_storage_layers=expert_storage_layers, ep=ep, tp=tp, experts_from=experts_from,
                            kv_block=kv_block, kv_pool_tokens=kv_pool_tokens, engram_from=engram_from,
                            engram_shm=engram_shm, engram_token_map=engram_token_map)
        return cls(model, max_seqs, max_batched_tokens, max_seq_len, chunk_size, use_graphs, preempt=kv_preempt)

    # ------------------------------------------------------------------- API
    def add_request(self, prompt: list[int], max_new_tokens: int, ignore_eos: bool = False,
                    stop_ids: Iterable[int] = (), temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                    logprobs: int | None = None, seed: int | None = None) -> Request:
        """``temperature`` 0 decodes greedily; > 0 samples softmax(logits / T),
        restricted to the ``top_k`` most likely tokens (0: all) and to the top-p
        nucleus (``top_p`` 1.0: all).  ``logprobs`` n >= 0: every generated token
        also carries its log-probability and the n most likely alternatives
        (``Request.logprobs``), from the raw logits.  ``seed``: the request's samples
        depend on (seed, position) only, so a seeded request repeats its output
        whatever it is batched with."""
        sp = self.sampling_params(temperature, top_k, top_p, logprobs, seed)
        return self.sched.add(prompt, max_new_tokens, ignore_eos=ignore_eos, eos_id=self.eos_id,
                              stop_ids=tuple(stop_ids), temperature=sp.temperature, top_k=sp.top_k, top_p=sp.top_p,
                              want_logprobs=sp.logprobs, seed=sp.seed)

    def sampling_params(self, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                        logprobs: int | None = None, seed: int | None = None) -> SamplingParams:
        """Checked decoding rule of a request (ValueError when this engine cannot
        apply it: top-k / top-p / log-probabilities need the whole vocabulary's
        logits on one GPU, so the vocab-parallel head refuses them)."""
        sp = SamplingParams(float(temperature), int(top_k or 0), float(1.0 if top_p is None else top_p),
                            None if logprobs is None else int(logprobs), None if seed is None else int(seed))
        if (sp.filters or sp.wants_logprobs) and getattr(self.model, "tp", None) is not None:
            raise ValueError("top_k / top_p / logprobs are not supported with the tensor-parallel (vocab-parallel) head")
        return sp

    def step(self) -> list[tuple[Request, int | None]]:
        chunks = self.sched.schedule()
        if not chunks:
            return []
        meta = StepMeta(self.cfg, [SeqChunk(c.req.slot, c.start_pos, c.tokens, c.sample,
                                            temperature=c.req.temperature, top_k=c.req.top_k, top_p=c.req.top_p,
                                            logprobs=c.req.want_logprobs, seed=c.req.seed) for c in chunks])
        ids = self.run_meta(meta)
        if meta.want_lp:
            it = iter(self.last_logprobs)
            for c in chunks:
                if c.sample:
                    e = next(it)
                    if e is not None:
                        c.req.logprobs.append(e)
        return self.sched.commit(chunks, ids)

    last_logprobs: list = []   # per sampled row of the last step that asked for log-probabilities

    _trace_left: int | None = None

    def run_meta(self, meta: StepMeta) -> list[int]:
        """Uploads ``meta``, runs the model step, returns the sampled ids on the host."""
        m = self.model
        if self.stream is not None:
            with torch.cuda.stream(self.stream):
                out = self._run_device(meta)
                host = out.to("cpu", non_blocking=True) if len(out) else out.cpu()
            self.stream.synchronize()
        else:
            out = self._run_device(meta)
            host = out
        if meta.want_lp:
            n = len(host)
            m = self.model
            self.last_logprobs = logprob_entries(m.lp_chosen[:n].tolist(), m.lp_vals[:n].tolist(),
                                                 m.lp_ids[:n].tolist(), meta.lp_want[:n])
        self.stats["steps"] += 1
        self.stats["tokens"] += meta.T
        self.stats["last_T"] = meta.T
        return [int(x) for x in host.tolist()]

    def _run_device(self, meta: StepMeta) -> torch.Tensor:
        m = self.model
        if self._trace_left is None:
            from ..utils.trace import trace_steps_from_env
            self._trace_left = trace_steps_from_env()
        if self.use_graphs and self.bucket and self._trace_left <= 0:
            # padded to bucketed shapes; the padding's sampled rows are dropped here
            pm = meta.padded(m.max_tokens, m.max_sample, m.n_slots)
            self.stats["padded_tokens"] += pm.T - meta.T
            out = self._run_graph(pm)
            return out[:pm.n_out]
        m.upload(meta, self.pinned)
        if self._trace_left > 0:
            # numeric trace of the first steps (eager): per-layer stream statistics
            from ..utils.trace import format_stats, layer_stats, log
            self._trace_left -= 1
            trace: dict = {}
            out = m.forward(meta, trace=trace)
            for line in format_stats(layer_stats(trace)):
                log.info("step %d T=%d %s", self.stats["steps"], meta.T, line)
            return out
        if not self.use_graphs:
            return m.forward(meta)
        return self._run_graph(meta, uploaded=True)

    def _run_graph(self, meta: StepMeta, uploaded: bool = False) -> torch.Tensor:
        m = self.model
        if not uploaded:
            m.upload(meta, self.pinned)
        key = meta.key()
        g = self.graphs.get(key)
        if g is None:
            # The first step of a shape runs eagerly (it is the real step: it advances
            # the caches once and its output is returned).  Capture then records the
            # same launches without executing them; later steps of this shape replay.
            out = m.forward(meta)
            torch.cuda.current_stream().synchronize()
            ErrorWord.check(m.dev)
            while len(self.graphs) >= self.max_graphs:
                self.graphs.popitem(last=False)       # least recently used
                self.stats["graph_evictions"] += 1
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=torch.cuda.current_stream()):
                gout = m.forward(meta)
            self.graphs[key] = (graph, gout)
            self.stats["graph_captures"] += 1
            return out
        self.graphs.move_to_end(key)
        graph, out = g
        graph.replay()
        return out

    def generate(self, prompts: list[list[int]], max_new_tokens: int, ignore_eos: bool = False,
                 **sampling) -> list[list[int]]:
        """Runs the prompts to completion; ``sampling``: :meth:`add_request`'s decoding
        options (temperature, top_k, top_p, seed, logprobs)."""
        reqs = [self.add_request(p, max_new_tokens, ignore_eos, **sampling) for p in prompts]
        while not all(r.finished for r in reqs):
            self.step()
        return [r.output for r in reqs]

    def check_errors(self) -> None:
        ErrorWord.check(self.model.dev)
