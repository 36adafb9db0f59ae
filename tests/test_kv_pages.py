"""Paged compressed caches, host side: the native block allocator, the per-ratio
block tables and reservation-based admission in the scheduler (CPU only)."""

import numpy as np
import pytest

from dsv4_flash_deployment_b200.config import v4_flash_config
from dsv4_flash_deployment_b200.engine.scheduler import Scheduler
from dsv4_flash_deployment_b200.models.kv_pages import KvPager
from dsv4_flash_deployment_b200.ops.host import KvBlockAllocator


def test_block_allocator_reserve_grow_release():
    a = KvBlockAllocator(n_blocks=6, n_slots=3, max_per_slot=4)
    assert a.free_blocks == 6
    assert a.reserve(0, 3)
    assert list(a.row(0)) == [0, 1, 2, -1]
    assert a.reserve(0, 4)                     # grow keeps the mapped prefix
    assert list(a.row(0)[:3]) == [0, 1, 2] and a.slot_blocks(0) == 4
    assert not a.reserve(1, 3)                 # only 2 left: refused, nothing changed
    assert a.free_blocks == 2 and a.slot_blocks(1) == 0
    assert not a.reserve(2, 5)                 # beyond the table row
    a.release(0)
    assert a.free_blocks == 6 and list(a.row(0)) == [-1] * 4
    assert a.reserve(1, 4)
    assert sorted(a.row(1)) == [0, 1, 2, 3]    # released blocks are handed out again
    with pytest.raises(ValueError):
        KvBlockAllocator(0, 1, 1)


def _pager(pool_tokens, max_seq=1024, block=16, slots=2):
    cfg = v4_flash_config()                    # ratios 4 and 128
    return cfg, KvPager(cfg, "cpu", slots + 1, max_seq, block, pool_tokens)


def test_pager_geometry_and_tables():
    cfg, pg = _pager(pool_tokens=1024)
    assert pg.ratios == [4, 128]
    assert pg.max_c == {4: 256, 128: 8}
    assert pg.n_blocks == {4: 16, 128: 1}
    assert pg.rows(4) == 17 * 16               # + the scratch block
    # descriptor: table address, ld, shift, logical capacity
    d4 = pg.desc[4].tolist()
    assert d4[0] == pg.table[4].data_ptr() and d4[1:] == [16, 4, 256]
    # unmapped entries point at the scratch block
    assert (pg.host[4] == 16).all() and (pg.host[128] == 1).all()
    assert pg.reserve(1, 700)                  # 176 entries of ratio 4 -> 11 blocks; 6 of ratio 128 -> 1
    assert (pg.host[4][1, :11] == np.arange(11)).all() and (pg.host[4][1, 11:] == 16).all()
    assert pg.host[128][1, 0] == 0
    pg.sync()
    assert (pg.table[4].numpy() == pg.host[4]).all()
    assert not pg.reserve(0, 500)              # ratio 128 has no block left: all or nothing
    assert pg.free_blocks() == {4: 5, 128: 0}
    pg.release(1)
    pg.sync()
    assert pg.free_blocks() == {4: 16, 128: 1} and (pg.table[4].numpy() == 16).all()
    with pytest.raises(ValueError):
        KvPager(cfg, "cpu", 3, 1024, 12)       # block size must be a power of two


def _finish_prompt_and_decode(s, steps):
    out = []
    for _ in range(steps):
        chunks = s.schedule()
        out.append([(c.req.req_id, len(c.tokens)) for c in chunks])
        s.commit(chunks, [7] * sum(c.sample for c in chunks))
    return out


def test_scheduler_admission_waits_for_blocks():
    _, pg = _pager(pool_tokens=1024)
    s = Scheduler(max_seqs=2, max_batched_tokens=1024, max_seq_len=1024, kv=pg)
    a = s.add(list(range(600)), 3, ignore_eos=True)
    b = s.add(list(range(400)), 3, ignore_eos=True)
    first = s.schedule()
    # b has a free slot but not enough blocks: it waits at the head of the queue
    assert [c.req for c in first] == [a] and b.slot < 0 and s.slots.n_free == 1
    s.commit(first, [7])
    while not a.finished:
        s.commit(s.schedule(), [7])
    assert pg.free_blocks() == {4: 16, 128: 1}
    nxt = s.schedule()
    assert [c.req for c in nxt] == [b] and b.slot >= 0
    assert pg.alloc[4].slot_blocks(b.slot) == -(-(403 // 4 + 1) // 16)


def test_scheduler_rejects_requests_larger_than_the_pool():
    _, pg = _pager(pool_tokens=512)
    s = Scheduler(max_seqs=2, max_batched_tokens=256, max_seq_len=1024, kv=pg)
    with pytest.raises(ValueError, match="paged cache pool"):
        s.add(list(range(900)), 10)
    s.add(list(range(300)), 10)                # fits


def test_memory_estimate_counts_the_paged_pool():
    from dsv4_flash_deployment_b200.engine.memory import non_expert_bytes

    cfg = v4_flash_config()
    full = non_expert_bytes(cfg, 512, 512, 16384)
    paged_same = non_expert_bytes(cfg, 512, 512, 16384, kv_block=64)
    paged_small = non_expert_bytes(cfg, 512, 512, 16384, kv_block=64, kv_pool_tokens=512 * 2048)
    # same capacity: the pools only add the scratch blocks (and drop the padding slot)
    assert abs(paged_same - full) < 0.01 * full
    assert paged_small < full - 10 * 2 ** 30   # 2k instead of 16k tokens per sequence


def test_cancel_releases_blocks_and_unblocks_the_queue():
    _, pg = _pager(pool_tokens=1024)
    s = Scheduler(max_seqs=2, max_batched_tokens=1024, max_seq_len=1024, kv=pg)
    a = s.add(list(range(900)), 8, ignore_eos=True)
    b = s.add(list(range(300)), 8, ignore_eos=True)
    first = s.schedule()
    assert [c.req for c in first] == [a] and b.slot < 0      # b waits for blocks
    s.commit(first, [7])
    s.cancel(a)
    nxt = s.schedule()                                       # a's blocks return, b is admitted
    assert a.finished and a.finish_reason == "cancelled"
    assert [c.req for c in nxt] == [b]
    assert pg.alloc[4].slot_blocks(b.slot) == -(-(308 // 4 + 1) // 16)
    assert pg.free_blocks()[4] == 16 - pg.alloc[4].slot_blocks(b.slot)


def test_pager_for_ratio_one_and_two_caches():
    from dsv4_flash_deployment_b200.config import v41_flash_config

    cfg = v41_flash_config()
    pg = KvPager(cfg, "cpu", 5, 4096, 64, pool_tokens=3 * 4096)
    assert set(pg.ratios) <= {1, 2} and pg.ratios
    for r in pg.ratios:
        assert pg.max_c[r] == 4096 // r
        assert pg.n_blocks[r] == -(-(3 * 4096 // r) // 64)
        assert pg.desc[r][1].item() * 64 >= pg.max_c[r]          # ld blocks cover a whole sequence
    assert pg.fits(4096) and pg.reserve(0, 4096) and pg.reserve(1, 4096) and pg.reserve(2, 4096)
    assert not pg.reserve(3, 100)                                 # pool holds three full sequences
    pg.release(1)
    assert pg.reserve(3, 4096)


class _Seq:
    """Deterministic stand-in for a model: the next token is a function of the
    whole context (so a recompute after a preemption must rebuild it exactly)."""

    @staticmethod
    def next_token(ctx):
        return (sum((i + 1) * t for i, t in enumerate(ctx)) * 31 + len(ctx)) % 1000


def _drive(sched, reqs, max_steps=2000):
    """Runs the scheduler with _Seq as the model: every sampled chunk's token is
    _Seq.next_token of its request's full context (prefill + generated)."""
    steps = 0
    while not all(r.finished for r in reqs):
        chunks = sched.schedule()
        toks = []
        for c in chunks:
            if c.sample:
                r = c.req
                ctx = r.prefill[:c.start_pos + len(c.tokens)] if not r.prompt_done else \
                    r.prefill + r.output[r.folded:]
                toks.append(_Seq.next_token(ctx))
        sched.commit(chunks, toks)
        steps += 1
        assert steps < max_steps
    return steps


def _want(prompt, n):
    ctx, out = list(prompt), []
    for _ in range(n):
        t = _Seq.next_token(ctx)
        out.append(t)
        ctx.append(t)
    return out


def test_preemption_recomputes_and_keeps_every_token():
    from dsv4_flash_deployment_b200.config import toy_v4_config

    cfg = toy_v4_config()                                # ratio 4 only
    pg = KvPager(cfg, "cpu", 4 + 1, 1024, 16, 640)      # ratio 4: 160 entries = 10 blocks of 16
    sched = Scheduler(max_seqs=4, max_batched_tokens=96, max_seq_len=1024, chunk_size=64, kv=pg, preempt=True)
    prompts = [[(7 * i + j) % 1000 for j in range(n)] for i, n in enumerate((100, 90, 120, 70))]
    reqs = [sched.add(p, 200, ignore_eos=True) for p in prompts]
    _drive(sched, reqs)
    assert sched.n_preempted > 0 and any(r.preemptions for r in reqs)
    for p, r in zip(prompts, reqs):
        assert r.output == _want(p, 200), r.req_id
    assert pg.free_blocks() == {4: 10}
    # reservation mode on the same pool: no preemption, same tokens, fewer requests at once
    pg2 = KvPager(cfg, "cpu", 4 + 1, 1024, 16, 640)
    s2 = Scheduler(max_seqs=4, max_batched_tokens=96, max_seq_len=1024, chunk_size=64, kv=pg2)
    reqs2 = [s2.add(p, 200, ignore_eos=True) for p in prompts]
    _drive(s2, reqs2)
    assert s2.n_preempted == 0 and [r.output for r in reqs2] == [r.output for r in reqs]


def test_preempted_request_positions_continue_after_recompute():
    from dsv4_flash_deployment_b200.engine.scheduler import Request

    r = Request(0, [1, 2, 3], 10)
    r.n_prefilled = 3
    r.output = [9, 8]
    assert r.position == 4                       # token 8 goes to position 4
    r.ctx, r.folded, r.n_prefilled = r.prompt + r.output, 2, 0
    assert not r.prompt_done and r.prefill == [1, 2, 3, 9, 8]
    r.n_prefilled = 5
    r.output.append(7)                           # sampled at the end of the recompute
    assert r.prompt_done and r.position == 5


def test_engine_with_preemption_matches_greedy_on_the_oracle():
    import torch

    from dsv4_flash_deployment_b200.config import toy_v4_config
    from dsv4_flash_deployment_b200.engine.engine import Engine
    from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
    from dsv4_flash_deployment_b200.models.oracle_step import OracleStepModel
    from dsv4_flash_deployment_b200.ref.model import RefModel

    cfg = toy_v4_config()
    w = make_random_weights(cfg, seed=3, include_mtp=False)
    model = OracleStepModel(cfg, w, n_slots=3, max_seq_len=128)
    model.pager = KvPager(cfg, "cpu", 3 + 1, 128, 4, 96)   # 24 entries of ratio 4: 6 blocks of 4
    eng = Engine(model, 3, 48, 128, 16, use_graphs=False, preempt=True)
    prompts = [[(5 * i + 3 * j) % 900 + 20 for j in range(n)] for i, n in enumerate((22, 15, 30))]
    reqs = [eng.add_request(p, 26, ignore_eos=True, logprobs=1) for p in prompts]
    while not all(r.finished for r in reqs):
        eng.step()
    assert eng.sched.n_preempted > 0
    ref = RefModel(cfg, w, max_seq_len=128)
    for p, r in zip(prompts, reqs):
        out, _ = ref.generate(torch.tensor([p]), 26)
        assert r.output == out[0].tolist()
        assert len(r.logprobs) == 26 and all(e["top"][0][0] == t for e, t in zip(r.logprobs, r.output))


def test_metrics_report_paged_block_use():
    import types

    from dsv4_flash_deployment_b200.config import toy_v4_config
    from dsv4_flash_deployment_b200.serving.metrics import render_prometheus

    pg = KvPager(toy_v4_config(), "cpu", 3, 1024, 16, 640)
    sched = Scheduler(max_seqs=2, max_batched_tokens=64, max_seq_len=1024, kv=pg)
    sched.add(list(range(300)), 10)
    sched.schedule()                                   # admits: 78 entries of ratio 4 -> 5 of 10 blocks
    loop = types.SimpleNamespace(stats={"requests": 1, "finished": 0, "failed": 0, "prompt_tokens": 300,
                                        "generated_tokens": 0, "steps": 0, "step_time_s": 0.0,
                                        "last_batch_tokens": 0},
                                 step_ms_window=[], ttft_window=[], healthy=True,
                                 engine=types.SimpleNamespace(sched=sched, stats={}))
    text = render_prometheus(types.SimpleNamespace(loop=loop))
    assert 'dsv4_kv_blocks_used_ratio{ratio="4"} 0.5000' in text


def test_pool_size_from_memory_utilization():
    """The pool fills what the utilization leaves after weights and buffers: its
    bytes plus everything else come to the budget (within one block of the largest
    ratio), more memory gives a larger pool, and a budget without room for one
    request is refused."""
    from dsv4_flash_deployment_b200.engine.memory import (expert_block_bytes, kv_pool_tokens_for,
                                                           non_expert_bytes)

    cfg = v4_flash_config()
    GiB = 2 ** 30
    args = dict(max_tokens=1024, n_slots=513, max_seq=2048, kv_block=64, ep_world=8)
    pool = kv_pool_tokens_for(cfg, 178 * GiB, 0.85, **args)
    used = non_expert_bytes(cfg, 1024, 513, 2048, 64, pool) + cfg.n_layers * expert_block_bytes(cfg, 8)
    step = 128 * 64
    per_tok = (non_expert_bytes(cfg, 1024, 513, 2048, 64, pool + step) - non_expert_bytes(cfg, 1024, 513, 2048, 64,
                                                                                          pool)) / step
    assert used <= 0.85 * 178 * GiB < used + (step + 1) * per_tok
    assert pool % step == 0 and pool > 513 * 2048       # more context than the per-slot caches would hold
    assert kv_pool_tokens_for(cfg, 178 * GiB, 0.95, **args) > pool
    with pytest.raises(ValueError, match="not one"):
        kv_pool_tokens_for(cfg, 20 * GiB, 0.85, **args)
    with pytest.raises(ValueError):
        kv_pool_tokens_for(cfg, 178 * GiB, 1.5, **args)
