"""Shared-memory control channel of the multi-rank serving front (CPU ranks).

Round trips of pickled messages of many sizes in lockstep, an oversized message
refused, a rank that exits between steps reported by rank 0's next gather
within seconds, rank 0's exit reported to a waiting rank, and the serving front
(DistributedEngine) over the channel matching the oracle's greedy tokens.  The
ranks rendezvous over a gloo group (the path of the file travels there)."""

import os
import time

import pytest
import torch

from dsv4_flash_deployment_b200.utils.launch import RankFailure, spawn

pytestmark = pytest.mark.skipif(not os.path.isdir("/dev/shm"), reason="no /dev/shm")


def _round_trips(rank, world):
    import torch.distributed as dist

    from dsv4_flash_deployment_b200.engine.control import ControlError, ShmControl

    ch = ShmControl.create(dist.group.WORLD, bcast_bytes=1 << 20, reply_bytes=1 << 16, timeout_s=30)
    seen = []
    for i in range(200):
        payload = {"step": i, "blob": bytes(range(256)) * (i * 17 % 300)}
        got = ch.broadcast(payload if rank == 0 else None)
        seen.append(got["step"] == i and got["blob"] == payload["blob"])
        replies = ch.gather((rank, i, "x" * (rank * i % 500)))
        if rank == 0:
            assert replies == [(r, i, "x" * (r * i % 500)) for r in range(world)]
    out = {"ok": all(seen)}
    if rank == 0:
        try:
            ch.broadcast({"blob": b"\0" * (2 << 20)})
            out["oversize"] = "sent"
        except ControlError as e:
            out["oversize"] = str(e)
        ch.broadcast({"step": -1})
        ch.gather(None)
        t0 = time.perf_counter()
        for _ in range(300):
            ch.broadcast({"adds": [], "cancels": [], "any_work": True, "stop": False})
            ch.gather([])
        out["rt_us"] = (time.perf_counter() - t0) / 300 * 1e6
    else:
        assert ch.broadcast()["step"] == -1
        ch.gather(None)
        for _ in range(300):
            ch.broadcast()
            ch.gather([(1, 5, False, None, None)])
    ch.close()
    return out


def test_round_trips_in_lockstep():
    res = spawn(_round_trips, 3, timeout_s=120)
    assert all(r["ok"] for r in res)
    assert "larger than its area" in res[0]["oversize"]
    assert res[0]["rt_us"] < 5000     # a gloo round trip costs about 1-3 ms on the same machine


def _worker_exits(rank, world):
    import torch.distributed as dist

    from dsv4_flash_deployment_b200.engine.control import ControlError, ShmControl

    ch = ShmControl.create(dist.group.WORLD, timeout_s=60)
    for i in range(3):
        ch.broadcast({"i": i} if rank == 0 else None)
        ch.gather(i)
    if rank == 1:
        os._exit(0)                    # leaves between steps, without a word
    ch.broadcast({"i": 3} if rank == 0 else None)
    t0 = time.time()
    try:
        ch.gather(3)
    except ControlError as e:
        return {"detected": str(e), "after_s": time.time() - t0}
    return {"detected": None}


def test_a_rank_that_exits_is_reported_quickly():
    with pytest.raises(RankFailure) as ei:
        spawn(_worker_exits, 2, timeout_s=120, pg_timeout_s=5)
    r0 = ei.value.results[0]
    assert r0[0] == "ok", r0
    assert "rank 1" in r0[1]["detected"] and "gone" in r0[1]["detected"] and r0[1]["after_s"] < 5, r0


def _rank0_exits(rank, world):
    import torch.distributed as dist

    from dsv4_flash_deployment_b200.engine.control import ControlError, ShmControl

    ch = ShmControl.create(dist.group.WORLD, timeout_s=60)
    ch.broadcast({"i": 0} if rank == 0 else None)
    ch.gather(0)
    if rank == 0:
        os._exit(0)
    t0 = time.time()
    try:
        ch.broadcast()
    except ControlError as e:
        return {"detected": str(e), "after_s": time.time() - t0}
    return {"detected": None}


def test_rank0_exit_is_reported_to_waiting_ranks():
    with pytest.raises(RankFailure) as ei:
        spawn(_rank0_exits, 2, timeout_s=120, pg_timeout_s=5)
    r1 = ei.value.results[1]
    assert r1[0] == "ok", r1
    assert "rank 0" in r1[1]["detected"] and r1[1]["after_s"] < 5, r1


PROMPTS = [[0] + [40 + (i * 11 + j) % 170 for j in range(12 + 5 * i)] for i in range(3)]


def _serve_over_shm(rank, world):
    import torch.distributed as dist

    from dsv4_flash_deployment_b200.engine.config import EngineConfig
    from dsv4_flash_deployment_b200.engine.control import make_control
    from dsv4_flash_deployment_b200.engine.dist_engine import DistributedEngine, worker_loop
    from dsv4_flash_deployment_b200.serving.launch import build_local_engine

    eng = build_local_engine(EngineConfig(device="cpu", model="toy-v4", max_seqs=2, max_batched_tokens=32,
                                          chunk_size=16, max_model_len=96), extra_slots=1)
    ctl = make_control("shm", dist.group.WORLD, timeout_s=60)
    if rank != 0:
        return {"steps": worker_loop(eng, dist.group.WORLD, control=ctl)}
    de = DistributedEngine(eng, dist.group.WORLD, control=ctl)
    reqs = [de.add_request(p, 4, ignore_eos=True) for p in PROMPTS]
    while not all(r.finished for r in reqs):
        de.step()
    de.shutdown()
    return {"outs": [r.output for r in reqs], "ranks": [r.rank for r in reqs]}


def test_serving_front_over_shared_memory_matches_oracle():
    from dsv4_flash_deployment_b200.config import toy_v4_config
    from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
    from dsv4_flash_deployment_b200.ref.model import RefModel

    res = spawn(_serve_over_shm, 2, timeout_s=300)
    cfg = toy_v4_config()
    ref = RefModel(cfg, make_random_weights(cfg, seed=0, include_mtp=False), max_seq_len=96)
    for p, got in zip(PROMPTS, res[0]["outs"]):
        want, _ = ref.generate(torch.tensor([p]), 4)
        assert got == want[0].tolist()
    assert sorted(set(res[0]["ranks"])) == [0, 1] and res[1]["steps"] > 0


def test_stale_control_files_are_removed(tmp_path):
    import subprocess
    import sys

    from dsv4_flash_deployment_b200.engine.control import ShmControl

    p = subprocess.run([sys.executable, "-c", "import os; print(os.getpid())"], capture_output=True, text=True)
    dead = int(p.stdout)
    stale = tmp_path / f"dsv4_ctl_{dead}_abcd1234"
    live = tmp_path / f"dsv4_ctl_{os.getpid()}_beef0000"
    other = tmp_path / "dsv4_ctl_notapid_x"
    for f in (stale, live, other):
        f.write_bytes(b"x")
    assert ShmControl.remove_stale(str(tmp_path)) == [str(stale)]
    assert live.exists() and other.exists() and not stale.exists()
