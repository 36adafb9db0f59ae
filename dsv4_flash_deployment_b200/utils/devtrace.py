"""Device timestamp ring: per-op device time inside a replayed CUDA graph.

CUDA events cannot be recorded inside a captured graph, and a profiler
serializes kernels and cannot wrap a multi-rank job.  This trace instead
launches a one-thread kernel (``ts_mark``, ``csrc/misc.cu``) after every op
group of the model step; the kernel waits for the preceding kernel to complete
and stores ``%globaltimer`` into a slot of a device ring.  Captured with the
step, the marks replay with it, so the difference of consecutive slots is what
each op group cost on the stream (its own kernels plus the launch gap before
them), on every rank of a multi-GPU job at the same time.

The marks serialize the op groups (a mark waits for the whole previous grid),
so programmatic-dependent-launch overlap between groups is lost; the step
total under the trace is reported next to the untraced step time.

    tr = DeviceTrace(device, capacity=4096)
    model.dev_trace = tr
    tr.begin()                  # before a step (eager, or before its capture)
    ... model.forward(meta) ...   # op groups call tr.mark(name) at their end
    times = tr.read()           # {name: [ns per occurrence]} of the last run
"""

from __future__ import annotations

import torch


class DeviceTrace:
    def __init__(self, device, capacity: int = 8192):
        self.dev = torch.device(device)
        self.ring = torch.zeros(capacity, dtype=torch.int64, device=self.dev)
        self.names: list[str] = []
        self.cursor = 0
        self._frozen = False
        from ..ops import _ext
        self.ext = _ext.load(required=True)

    def begin(self) -> None:
        """Starts a step: slot 0 is the step's start mark."""
        self.cursor = 0
        self.mark("<start>")

    def freeze(self) -> None:
        """After the first step the name list is fixed; later steps (captures,
        replays) must issue the same marks in the same order."""
        self._frozen = True

    def mark(self, name: str) -> None:
        i = self.cursor
        if i >= self.ring.numel():
            raise RuntimeError(f"device trace ring full ({self.ring.numel()} marks)")
        if self._frozen:
            if i >= len(self.names) or self.names[i] != name:
                raise RuntimeError(f"device trace: mark {i} is {name!r}, expected "
                                   f"{self.names[i] if i < len(self.names) else None!r}")
        elif i == len(self.names):
            self.names.append(name)
        self.ext.ts_mark(self.ring, i)
        self.cursor = i + 1

    def read(self) -> dict[str, list[int]]:
        """Nanoseconds of every op group occurrence of the last run (synchronizes)."""
        n = self.cursor
        ts = self.ring[:n].cpu().tolist()
        out: dict[str, list[int]] = {}
        for i in range(1, n):
            out.setdefault(self.names[i], []).append(ts[i] - ts[i - 1])
        return out

    def total_ns(self) -> int:
        n = self.cursor
        ts = self.ring[:n].cpu().tolist()
        return ts[-1] - ts[0] if n > 1 else 0


def summarize(runs: list[dict[str, list[int]]]) -> dict[str, dict]:
    """Mean per step over runs: total ms and occurrences of each op group."""
    acc: dict[str, list[float]] = {}
    cnt: dict[str, int] = {}
    for r in runs:
        for k, v in r.items():
            acc.setdefault(k, []).append(sum(v) / 1e6)
            cnt[k] = len(v)
    return {k: {"ms": sum(v) / len(v), "n": cnt[k]} for k, v in acc.items()}
