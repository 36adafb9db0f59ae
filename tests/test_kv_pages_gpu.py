"""Paged compressed caches on the GPU: an engine whose compressed KV / indexer-key
caches are block pools (small blocks, slots recycled so reused blocks hold a
previous request's entries) gives the same logits, step for step, as the engine
with contiguous per-slot caches.  Both run the same kernels on the same data;
only the cache row addresses differ."""

import pytest
import torch

from dsv4_flash_deployment_b200.engine.engine import Engine

from test_model_gpu import small_v4, small_v41

pytestmark = pytest.mark.gpu


def _lockstep(cfg, block, use_graphs):
    max_len = 128
    kw = dict(max_seqs=2, max_batched_tokens=64, max_seq_len=max_len, seed=5, use_graphs=use_graphs)
    ref = Engine.build(cfg, "cuda", **kw)
    pag = Engine.build(cfg, "cuda", kv_block=block, **kw)
    assert pag.model.pager is not None and ref.model.pager is None
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (70, 23, 41, 9)]
    new = [12, 30, 8, 20]
    reqs = []
    for eng in (ref, pag):
        reqs.append([eng.add_request(p, n, ignore_eos=True) for p, n in zip(prompts, new)])
    worst = 1.0
    steps = 0
    while not all(r.finished for r in reqs[0]):
        ev_r, ev_p = ref.step(), pag.step()
        assert [(r.req_id, t) for r, t in ev_r] == [(r.req_id, t) for r, t in ev_p]
        n = ref.stats["last_T"]
        rows = len([t for _, t in ev_r if t is not None])
        lr = ref.model.logits[:rows, : cfg.vocab_size].float()
        lp = pag.model.logits[:rows, : cfg.vocab_size].float()
        if rows:
            worst = min(worst, float(torch.nn.functional.cosine_similarity(lr, lp, dim=-1).min()))
        steps += 1
        assert n > 0
    assert all(r.finished for r in reqs[1])
    assert [r.output for r in reqs[0]] == [r.output for r in reqs[1]]
    assert worst > 0.9999, worst
    # every block went back to the pool
    pg = pag.model.pager
    assert pg.free_blocks() == pg.n_blocks
    pag.check_errors()
    ref.check_errors()
    return steps


@pytest.mark.parametrize("use_graphs", [False, True])
def test_paged_v4_matches_contiguous(use_graphs):
    assert _lockstep(small_v4(), block=4, use_graphs=use_graphs) > 10


def test_paged_v41_reference_index_mode_matches_contiguous():
    # ratios 2 and 1, the alternate (ratio-1) key cache for non-closing decode tokens
    assert _lockstep(small_v41(), block=8, use_graphs=True) > 10
