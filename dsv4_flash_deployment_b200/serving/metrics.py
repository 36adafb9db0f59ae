"""Prometheus text exposition of the serving counters (no client library needed)."""

from __future__ import annotations


def _q(xs, q):
    if not xs:
        return 0.0
    s = sorted(xs)
    return s[min(int(q * len(s)), len(s) - 1)]


def render_prometheus(st) -> str:
    lp = st.loop
    s = lp.stats
    eng = lp.engine
    sched = eng.sched
    lines = []

    def metric(name, kind, help_, value, labels=""):
        lines.append(f"# HELP dsv4_{name} {help_}")
        lines.append(f"# TYPE dsv4_{name} {kind}")
        lines.append(f"dsv4_{name}{labels} {value}")

    metric("requests_total", "counter", "Requests accepted by the engine.", s["requests"])
    metric("requests_finished_total", "counter", "Requests finished (length, stop or cancelled).", s["finished"])
    metric("requests_failed_total", "counter", "Requests failed by an engine error.", s["failed"])
    metric("prompt_tokens_total", "counter", "Prompt tokens accepted.", s["prompt_tokens"])
    metric("generation_tokens_total", "counter", "Tokens generated.", s["generated_tokens"])
    metric("engine_steps_total", "counter", "Continuous-batching steps run.", s["steps"])
    metric("engine_step_seconds_total", "counter", "Wall time spent in steps.", f"{s['step_time_s']:.6f}")
    metric("step_ms_p50", "gauge", "Median step time over the last 1024 steps (ms).", f"{_q(lp.step_ms_window, .5):.3f}")
    metric("step_ms_p99", "gauge", "p99 step time over the last 1024 steps (ms).", f"{_q(lp.step_ms_window, .99):.3f}")
    metric("ttft_s_p50", "gauge", "Median time to first token over the last 1024 requests (s).",
           f"{_q(lp.ttft_window, .5):.4f}")
    metric("batch_tokens", "gauge", "Tokens in the last step.", s["last_batch_tokens"])
    metric("running_requests", "gauge", "Requests holding a cache slot.", len(sched.running))
    metric("waiting_requests", "gauge", "Requests queued for a slot.", len(sched.waiting))
    metric("cache_slots_used_ratio", "gauge", "Fraction of KV cache slots in use.",
           f"{1.0 - sched.slots.n_free / max(sched.max_seqs, 1):.4f}")
    kv = getattr(sched, "kv", None)
    if kv is not None and hasattr(kv, "free_blocks"):
        free = kv.free_blocks()
        lines.append("# HELP dsv4_kv_blocks_used_ratio Fraction of the paged compressed-cache blocks in use, per "
                     "compression ratio.")
        lines.append("# TYPE dsv4_kv_blocks_used_ratio gauge")
        for r in sorted(free):
            lines.append(f'dsv4_kv_blocks_used_ratio{{ratio="{r}"}} {1.0 - free[r] / max(kv.n_blocks[r], 1):.4f}')
    metric("preemptions_total", "counter", "Requests preempted for recompute (paged caches, kv_preempt).",
           getattr(sched, "n_preempted", 0))
    metric("graph_captures_total", "counter", "CUDA graphs captured.", eng.stats.get("graph_captures", 0))
    metric("graph_evictions_total", "counter", "CUDA graphs released by the bounded graph cache.",
           eng.stats.get("graph_evictions", 0))
    metric("padded_tokens_total", "counter", "Padding tokens added to reach bucketed step shapes.",
           eng.stats.get("padded_tokens", 0))
    spec = eng.stats.get("spec")
    if spec:
        metric("spec_accepted_tokens_total", "counter", "Draft tokens accepted.", spec.get("accepted", 0))
        metric("spec_draft_tokens_total", "counter", "Draft tokens proposed.", spec.get("drafted", 0))
    metric("healthy", "gauge", "1 when the engine loop is healthy.", 1 if lp.healthy else 0)
    metric("draining", "gauge", "1 while a shutdown drains the live requests.", 1 if getattr(lp, "draining", False) else 0)
    return "\n".join(lines) + "\n"
