"""Streaming capacity of the HTTP front: how many tokens per second the server
process can stream when the engine costs (almost) nothing.

The server (``serving/app.py`` + ``serving/engine_loop.py``) runs over a stand-in
engine whose step sleeps ``--step-ms`` and returns one token for every running
request, so what is measured is the front's own per-token work: the engine
thread's scheduling and hand-off, the event loop's wake-ups, the SSE encoding
and the socket writes.  Clients run in separate processes (so their parsing
does not share the server's interpreter) and open ``--streams`` streaming
completions of ``--tokens`` tokens each.  At 8 GPUs the engine decodes about
22,000 tokens per second, which the front must stream from one process.

    python -m dsv4_flash_deployment_b200.bench.front_bench --streams 512 --tokens 300
"""

from __future__ import annotations

import argparse
import asyncio
import json
import subprocess
import sys
import time


class StandInEngine:
    """Scheduler-driven engine without a model: each step sleeps ``step_s`` and
    samples token 70 + row % 20 for every sampled chunk."""

    def __init__(self, max_seqs: int, step_s: float):
        from ..engine.scheduler import Scheduler

        self.sched = Scheduler(max_seqs=max_seqs, max_batched_tokens=1 << 20, max_seq_len=1 << 16)
        self.stats = {}
        self.eos_id = 1
        self.step_s = step_s

    def add_request(self, prompt, max_new_tokens, ignore_eos=False, stop_ids=(), temperature=0.0, **kw):
        return self.sched.add(prompt, max_new_tokens, ignore_eos=ignore_eos, stop_ids=tuple(stop_ids))

    def step(self):
        chunks = self.sched.schedule()
        time.sleep(self.step_s)
        return self.sched.commit(chunks, [70 + i % 20 for i, c in enumerate(chunks) if c.sample])


async def _client(port: int, n: int, tokens: int) -> tuple[int, float]:
    import aiohttp

    async with aiohttp.ClientSession(connector=aiohttp.TCPConnector(limit=0)) as s:
        async def one():
            r = await s.post(f"http://127.0.0.1:{port}/v1/completions",
                             json={"prompt": [0, 5, 6], "max_tokens": tokens, "ignore_eos": True, "stream": True})
            k = 0
            async for line in r.content:
                if line.startswith(b"data: {"):
                    k += 1
            return k
        t0 = time.perf_counter()
        got = await asyncio.gather(*(one() for _ in range(n)))
        return sum(got), time.perf_counter() - t0


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--streams", type=int, default=512)
    ap.add_argument("--tokens", type=int, default=300)
    ap.add_argument("--step-ms", type=float, default=1.0)
    ap.add_argument("--clients", type=int, default=4, help="client processes")
    ap.add_argument("--port", type=int, default=8765)
    ap.add_argument("--client", type=int, default=None, help=argparse.SUPPRESS)
    a = ap.parse_args(argv)
    if a.client is not None:
        n, dt = asyncio.run(_client(a.port, a.client, a.tokens))
        print(f"{n} {dt:.4f}", flush=True)
        return

    from aiohttp import web

    from ..serving.app import ServerState, build_app
    from ..serving.engine_loop import EngineLoop
    from ..serving.tokenizer import ByteTokenizer

    loop = EngineLoop(StandInEngine(a.streams, a.step_ms / 1e3)).start()
    st = ServerState(loop, ByteTokenizer(1024, 0, 1), "stand-in", 1 << 16)

    async def run():
        runner = web.AppRunner(build_app(st))
        await runner.setup()
        await web.TCPSite(runner, "127.0.0.1", a.port).start()
        per = -(-a.streams // a.clients)
        procs = [await asyncio.create_subprocess_exec(
            sys.executable, "-m", "dsv4_flash_deployment_b200.bench.front_bench", "--client", str(per),
            "--tokens", str(a.tokens), "--port", str(a.port), stdout=subprocess.PIPE) for _ in range(a.clients)]
        total, wall = 0, 0.0
        for p in procs:
            out, _ = await p.communicate()
            n, dt = out.decode().split()
            total, wall = total + int(n), max(wall, float(dt))
        await runner.cleanup()
        return total, wall

    total, wall = asyncio.run(run())
    loop.stop()
    print(json.dumps({"streams": per_streams(a), "tokens_streamed": total, "wall_s": round(wall, 3),
                      "tok_s": round(total / wall, 1), "engine_steps": loop.stats["steps"],
                      "step_ms": a.step_ms}))


def per_streams(a) -> int:
    return -(-a.streams // a.clients) * a.clients


if __name__ == "__main__":
    main()
