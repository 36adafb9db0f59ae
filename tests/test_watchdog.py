"""Serving watchdog (CPU only): a step that raises, or one that runs past the
per-step deadline, fails every live request with an error and marks the engine
unhealthy; later submissions are refused instead of hanging."""

import asyncio
import time

from dsv4_flash_deployment_b200.engine.scheduler import Scheduler
from dsv4_flash_deployment_b200.serving.engine_loop import EngineLoop, GenParams


class FakeEngine:
    """Scheduler-driven engine whose step sleeps or raises on demand."""

    def __init__(self, mode: str, sleep_s: float = 0.0):
        self.sched = Scheduler(max_seqs=4, max_batched_tokens=64, max_seq_len=256)
        self.stats = {}
        self.mode, self.sleep_s = mode, sleep_s

    def add_request(self, prompt, max_new_tokens, ignore_eos=False, stop_ids=(), temperature=0.0):
        return self.sched.add(prompt, max_new_tokens, ignore_eos=ignore_eos, stop_ids=tuple(stop_ids))

    def step(self):
        chunks = self.sched.schedule()
        if self.mode == "raise":
            raise RuntimeError("device error word set: code=2 kernel=4 detail=16")
        time.sleep(self.sleep_s)
        return self.sched.commit(chunks, [5] * sum(c.sample for c in chunks))


async def _drive(loop: EngineLoop):
    streams = [loop.submit(list(range(10, 20)), GenParams(max_tokens=50, ignore_eos=True)) for _ in range(2)]
    items = []
    for s in streams:
        while True:
            kind, val = await asyncio.wait_for(s.q.get(), timeout=30)
            if kind in ("error", "done"):
                items.append((kind, val))
                break
    late = loop.submit([1, 2, 3], GenParams(max_tokens=2))
    items.append(await asyncio.wait_for(late.q.get(), timeout=30))
    return items


def test_failing_step_fails_requests_and_marks_unhealthy():
    loop = EngineLoop(FakeEngine("raise")).start()
    try:
        items = asyncio.run(_drive(loop))
    finally:
        loop.stop()
    assert [k for k, _ in items] == ["error", "error", "error"]
    assert "code=2" in items[0][1] and "unhealthy" in items[2][1]
    assert not loop.healthy and loop.stats["failed"] == 2


def test_step_past_deadline_fails_requests():
    loop = EngineLoop(FakeEngine("slow", sleep_s=0.3), step_deadline_s=0.1).start()
    try:
        items = asyncio.run(_drive(loop))
    finally:
        loop.stop()
    assert [k for k, _ in items] == ["error", "error", "error"]
    assert "deadline" in items[0][1]
    assert not loop.healthy


def test_drain_refuses_new_requests_and_lets_live_ones_finish():
    async def go(loop):
        live = loop.submit(list(range(10, 20)), GenParams(max_tokens=20, ignore_eos=True))
        while live.req is None:
            await asyncio.sleep(0.005)
        drained = asyncio.get_running_loop().run_in_executor(None, loop.drain, 30.0)
        while not loop.draining:
            await asyncio.sleep(0.001)
        late = loop.submit([1, 2, 3], GenParams(max_tokens=2))
        late_item = await asyncio.wait_for(late.q.get(), timeout=30)
        n = 0
        while True:
            kind, _ = await asyncio.wait_for(live.q.get(), timeout=30)
            if kind == "done":
                break
            n += kind == "token"
        return late_item, n, await drained

    loop = EngineLoop(FakeEngine("slow", sleep_s=0.01)).start()
    try:
        late_item, n, ok = asyncio.run(go(loop))
    finally:
        loop.stop()
    assert late_item[0] == "error" and "shutting down" in late_item[1]
    assert n == 20 and ok and loop.healthy
