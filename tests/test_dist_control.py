"""Multi-rank control plane over gloo (CPU oracle engines, data-parallel).

Rank 0 fronts the engine API and assigns requests to ranks; ranks step in
lockstep and report tokens back.  Failure detection: a rank that exits
between steps makes rank 0's next control collective fail within the group
timeout (host-side fault injection, no device involved).
"""

import os
import time

import pytest
import torch

from dsv4_flash_deployment_b200.utils.launch import RankFailure, spawn

PROMPTS = [[0] + [40 + (i * 11 + j) % 170 for j in range(12 + 5 * i)] for i in range(3)]
N_NEW = 4


def _engine():
    from dsv4_flash_deployment_b200.engine.config import EngineConfig
    from dsv4_flash_deployment_b200.serving.launch import build_local_engine

    ec = EngineConfig(device="cpu", model="toy-v4", max_seqs=2, max_batched_tokens=32, chunk_size=16,
                      max_model_len=96)
    return build_local_engine(ec, extra_slots=1)


def _rank_generate(rank, world):
    import torch.distributed as dist

    from dsv4_flash_deployment_b200.engine.dist_engine import DistributedEngine, worker_loop

    eng = _engine()
    if rank != 0:
        n = worker_loop(eng, dist.group.WORLD)
        return {"steps": n, "served": eng.stats["steps"], "dummy": eng.stats.get("dummy_steps", 0)}
    de = DistributedEngine(eng, dist.group.WORLD)
    reqs = [de.add_request(p, N_NEW, ignore_eos=True) for p in PROMPTS]
    while not all(r.finished for r in reqs):
        de.step()
    de.shutdown()
    return {"outs": [r.output for r in reqs], "ranks": [r.rank for r in reqs]}


def test_two_ranks_serve_and_match_oracle():
    from dsv4_flash_deployment_b200.config import toy_v4_config
    from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
    from dsv4_flash_deployment_b200.ref.model import RefModel

    res = spawn(_rank_generate, 2, timeout_s=300)
    cfg = toy_v4_config()
    ref = RefModel(cfg, make_random_weights(cfg, seed=0, include_mtp=False), max_seq_len=96)
    for p, got in zip(PROMPTS, res[0]["outs"]):
        want, _ = ref.generate(torch.tensor([p]), N_NEW)
        assert got == want[0].tolist()
    assert sorted(set(res[0]["ranks"])) == [0, 1]   # both ranks served requests
    assert res[1]["steps"] > 0 and res[1]["served"] > 0


def _rank_generate_replicated(rank, world):
    import torch.distributed as dist

    from dsv4_flash_deployment_b200.engine.dist_engine import DistributedEngine, worker_loop

    eng = _engine()
    if rank != 0:
        n = worker_loop(eng, dist.group.WORLD, replicated=True)
        return {"steps": n, "served": eng.stats["steps"], "dummy": eng.stats.get("dummy_steps", 0),
                "tokens": eng.stats["tokens"]}
    de = DistributedEngine(eng, dist.group.WORLD, replicated=True)
    reqs = [de.add_request(p, N_NEW, ignore_eos=True) for p in PROMPTS]
    while not all(r.finished for r in reqs):
        de.step()
    de.shutdown()
    return {"outs": [r.output for r in reqs], "ranks": [r.rank for r in reqs], "tokens": eng.stats["tokens"],
            "max_seqs": de.sched.max_seqs}


def test_replicated_mode_runs_the_same_steps_on_every_rank():
    """Tensor-parallel serving: every rank schedules every request and runs the
    same steps (same token count, no dummy steps); rank 0 alone reports tokens."""
    from dsv4_flash_deployment_b200.config import toy_v4_config
    from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
    from dsv4_flash_deployment_b200.ref.model import RefModel

    res = spawn(_rank_generate_replicated, 2, timeout_s=300)
    cfg = toy_v4_config()
    ref = RefModel(cfg, make_random_weights(cfg, seed=0, include_mtp=False), max_seq_len=96)
    for p, got in zip(PROMPTS, res[0]["outs"]):
        want, _ = ref.generate(torch.tensor([p]), N_NEW)
        assert got == want[0].tolist()
    assert set(res[0]["ranks"]) == {-1}
    assert res[0]["max_seqs"] == 2
    assert res[1]["dummy"] == 0 and res[1]["tokens"] == res[0]["tokens"]


def _rank_dies(rank, world):
    import torch.distributed as dist

    from dsv4_flash_deployment_b200.engine.dist_engine import DistributedEngine, worker_loop

    eng = _engine()
    if rank == 1:
        # follow two control steps, then leave between steps without a word
        from dsv4_flash_deployment_b200.engine import dist_engine as de_mod
        n = 0
        orig = de_mod._local_step

        def counting(*a, **kw):
            nonlocal n
            n += 1
            if n > 2:
                os._exit(0)
            return orig(*a, **kw)
        de_mod._local_step = counting
        worker_loop(eng, dist.group.WORLD)
        return "unreachable"
    de = DistributedEngine(eng, dist.group.WORLD)
    reqs = [de.add_request(p, 16, ignore_eos=True) for p in PROMPTS]
    t0 = time.time()
    try:
        while not all(r.finished for r in reqs):
            de.step()
    except Exception as e:  # noqa: BLE001
        return {"detected": True, "after_s": time.time() - t0, "error": type(e).__name__}
    return {"detected": False}


def test_dead_rank_is_detected_not_hung():
    with pytest.raises(RankFailure) as ei:
        spawn(_rank_dies, 2, timeout_s=120, pg_timeout_s=5)
    r0 = ei.value.results[0]
    assert r0[0] == "ok", r0
    assert r0[1]["detected"] and r0[1]["after_s"] < 60, r0
    assert ei.value.results[1][0] == "missing"


def _rank_generate_sampling_options(rank, world):
    import torch.distributed as dist

    from dsv4_flash_deployment_b200.engine.dist_engine import DistributedEngine, worker_loop

    eng = _engine()
    if rank != 0:
        worker_loop(eng, dist.group.WORLD)
        return {}
    de = DistributedEngine(eng, dist.group.WORLD)
    greedy_lp = [de.add_request(p, N_NEW, ignore_eos=True, logprobs=2) for p in PROMPTS]
    seeded = [de.add_request(PROMPTS[0], N_NEW, ignore_eos=True, temperature=3.0, seed=5, top_k=50)
              for _ in range(2)]
    while not all(r.finished for r in greedy_lp + seeded):
        de.step()
    de.shutdown()
    return {"outs": [r.output for r in greedy_lp], "lps": [r.logprobs for r in greedy_lp],
            "seeded": [r.output for r in seeded], "seeded_ranks": [r.rank for r in seeded]}


def test_sampling_options_cross_the_control_plane():
    """Log-probabilities come back from the rank that served the request, and a
    seeded request gives the same samples on either rank."""
    from dsv4_flash_deployment_b200.config import toy_v4_config
    from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
    from dsv4_flash_deployment_b200.ref.model import RefModel

    res = spawn(_rank_generate_sampling_options, 2, timeout_s=300)[0]
    cfg = toy_v4_config()
    ref = RefModel(cfg, make_random_weights(cfg, seed=0, include_mtp=False), max_seq_len=96)
    for p, got, lps in zip(PROMPTS, res["outs"], res["lps"]):
        want, _ = ref.generate(torch.tensor([p]), N_NEW)
        assert got == want[0].tolist()
        assert len(lps) == N_NEW and all(e["top"][0][0] == t and len(e["top"]) == 2 for e, t in zip(lps, got))
    assert res["seeded"][0] == res["seeded"][1] and sorted(res["seeded_ranks"]) == [0, 1]
