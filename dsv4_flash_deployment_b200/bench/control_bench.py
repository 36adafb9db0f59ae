"""Round trip of the multi-rank serving front's control channel: rank 0
broadcasts an empty step message and gathers one event from every rank, as one
serving step does, over the gloo group and over the shared-memory channel
(``engine/control.py``).  CPU ranks on this machine; median and p90 of 400
round trips after 400 warm-up ones.

    python -m dsv4_flash_deployment_b200.bench.control_bench --worlds 2 4 8
"""

from __future__ import annotations

import argparse
import json
import time


def _round_trips(rank, world, kind, n):
    import torch.distributed as dist

    from ..engine.control import make_control

    ch = make_control(kind, dist.group.WORLD, timeout_s=60)
    msg = {"adds": [], "cancels": [], "any_work": True, "stop": False}
    ts = []
    for i in range(2 * n):
        t0 = time.perf_counter()
        ch.broadcast(msg if rank == 0 else None)
        ch.gather([(1, 5, False, None, None)])
        if i >= n:
            ts.append(time.perf_counter() - t0)
    ch.close()
    ts.sort()
    return {"median_us": round(ts[len(ts) // 2] * 1e6, 1), "p90_us": round(ts[int(0.9 * len(ts))] * 1e6, 1)}


def main(argv=None) -> None:
    from ..utils.launch import spawn

    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--worlds", type=int, nargs="+", default=[2, 4, 8])
    ap.add_argument("--n", type=int, default=400)
    a = ap.parse_args(argv)
    for w in a.worlds:
        for kind in ("gloo", "shm"):
            r = spawn(_round_trips, w, kind, a.n, timeout_s=600)[0]
            print(json.dumps({"world": w, "channel": kind, **r}), flush=True)


if __name__ == "__main__":
    main()
