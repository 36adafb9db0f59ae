"""Numeric tracing of the residual streams (parity debugging).

The reference's patch series adds per-layer activation statistics behind an
environment switch (``DSV41_TRACE_LAYER_STATS``, vLLM patch 0009): RMS and the
fraction of exact zeros of every layer's hidden state.  The same here:
``DSV4_TRACE_LAYER_STATS=N`` makes the engine run its first N steps eagerly
with ``forward(trace=...)`` and log one line per layer and sublayer output:

    layer 3: rms 1.0213 max|x| 14.25 zero 0.0000 | attn rms 0.0871 ...

The statistics are computed on the device from the traced tensors; only a few
floats per layer cross to the host.
"""

from __future__ import annotations

import logging
import os

import torch

log = logging.getLogger("dsv4.trace")


def trace_steps_from_env() -> int:
    v = os.environ.get("DSV4_TRACE_LAYER_STATS", "0")
    try:
        return max(0, int(v))
    except ValueError:
        return 1 if v.lower() in ("1", "true", "yes") else 0


def tensor_stats(x: torch.Tensor) -> dict:
    """RMS, max |x| and the fraction of exact zeros of a tensor (fp32 math)."""
    f = x.float()
    n = max(1, f.numel())
    return {"rms": float(f.square().mean().sqrt()) if f.numel() else 0.0,
            "max": float(f.abs().max()) if f.numel() else 0.0,
            "zero": float((f == 0).sum()) / n}


def layer_stats(trace: dict) -> dict:
    """{layer id: {"x": stats of the streams entering the layer, "attn": stats of
    the attention sublayer output}} from a ``forward(trace=...)`` dict."""
    out: dict = {}
    for k, v in trace.items():
        if isinstance(k, int):
            out.setdefault(k, {})["x"] = tensor_stats(v)
        elif isinstance(k, str) and k.startswith("attn"):
            out.setdefault(int(k[4:]), {})["attn"] = tensor_stats(v)
    return dict(sorted(out.items()))


def format_stats(stats: dict) -> list[str]:
    lines = []
    for lid, d in stats.items():
        parts = [f"layer {lid}:"]
        for name in ("x", "attn"):
            if name in d:
                s = d[name]
                parts.append(f"{name} rms {s['rms']:.4g} max|x| {s['max']:.4g} zero {s['zero']:.4f}")
        lines.append(" | ".join(parts))
    return lines
