"""Run a function on N local ranks (one process each) under torch.distributed.

Used for CPU multi-rank runs (``gloo``) of the host-side parallel logic —
expert-parallel dispatch semantics, the serving control plane, failure
detection — and by the tests.  Every rank is a fresh ``spawn`` process that
joins a process group at 127.0.0.1 with a short timeout; the parent collects
each rank's return value or traceback, and kills exactly the PIDs it started
if a rank hangs past the deadline.
"""

from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import queue
import socket
import traceback
from typing import Any, Callable


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _child(fn, rank, world, port, backend, pg_timeout_s, env, args, q):
    os.environ.update(env)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist

    try:
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=pg_timeout_s))
        out = fn(rank, world, *args)
        q.put((rank, "ok", out))
    except BaseException as e:  # noqa: BLE001  (report every failure to the parent)
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))
    finally:
        try:
            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:
            pass


class RankFailure(RuntimeError):
    def __init__(self, results: dict[int, tuple[str, Any]], msg: str):
        super().__init__(msg)
        self.results = results


def spawn(fn: Callable, world: int, *args, backend: str = "gloo", timeout_s: float = 120.0,
          pg_timeout_s: float = 30.0, env: dict[str, str] | None = None) -> list[Any]:
    """Runs ``fn(rank, world, *args)`` on ``world`` processes; returns the per-rank results.

    Raises :class:`RankFailure` (with every rank's status) if a rank raised,
    exited without a result, or did not finish within ``timeout_s``.
    """
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_child, args=(fn, r, world, port, backend, pg_timeout_s, env or {}, args, q),
                         daemon=True) for r in range(world)]
    for p in procs:
        p.start()
    results: dict[int, tuple[str, Any]] = {}
    deadline = datetime.datetime.now() + datetime.timedelta(seconds=timeout_s)
    while len(results) < world:
        left = (deadline - datetime.datetime.now()).total_seconds()
        if left <= 0:
            break
        try:
            rank, status, val = q.get(timeout=min(left, 0.5))
            results[rank] = (status, val)
        except queue.Empty:
            # a rank that died without reporting (e.g. os._exit) never sends a result
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=5)
        if p.is_alive():
            p.kill()
            p.join(timeout=5)
    for r in range(world):
        if r not in results:
            results[r] = ("missing", f"rank {r} exited (code {procs[r].exitcode}) or timed out without a result")
    bad = {r: v for r, v in results.items() if v[0] != "ok"}
    if bad:
        msg = "; ".join(f"rank {r}: {s}: {str(v).splitlines()[0] if v else ''}" for r, (s, v) in sorted(bad.items()))
        raise RankFailure(results, msg)
    return [results[r][1] for r in range(world)]
