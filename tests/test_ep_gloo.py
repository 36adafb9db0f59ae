"""Config-1 plumbing: data-parallel attention + expert parallelism over gloo.

Tiny V4-style decoder (2 layers, hidden 256, 4 heads x 64, vocab 1024, 8
experts top-2 sigmoid + 1 shared, ratio-4 compressed attention with an
indexer keeping 4 blocks of 16), weights N(0, 0.02), seed 0; batch 2 of 64
random prompt tokens, 16 greedy tokens.  World 2: each rank steps one
sequence and owns 4 experts; routed pairs travel by all_to_all.  The tokens
must equal the single-rank dense oracle's.
"""

import torch

from dsv4_flash_deployment_b200.config import toy_v4_config
from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
from dsv4_flash_deployment_b200.ref.model import RefModel
from dsv4_flash_deployment_b200.utils.launch import spawn

N_NEW = 16


def _prompts():
    g = torch.Generator().manual_seed(0)
    return torch.randint(0, 1024, (2, 64), generator=g)


def _ep_rank(rank, world):
    from dsv4_flash_deployment_b200.parallel.ep_host import ep_ref_model

    cfg = toy_v4_config()
    w = make_random_weights(cfg, seed=0, init_std=0.02)
    m = ep_ref_model(cfg, w, max_seq_len=128)
    n_exp = sum(1 for k in m.w if k.endswith(".w1.weight") and ".experts." in k)
    prompts = _prompts()[rank:rank + 1]
    out, _ = m.generate(prompts, N_NEW)
    return {"tokens": out[0].tolist(), "local_expert_tensors": n_exp, "stats": m.ep.stats}


def test_config1_ep2_matches_dense():
    cfg = toy_v4_config()
    w = make_random_weights(cfg, seed=0, init_std=0.02)
    dense, _ = RefModel(cfg, w, max_seq_len=128).generate(_prompts(), N_NEW)
    res = spawn(_ep_rank, 2, timeout_s=300)
    for r in range(2):
        assert res[r]["tokens"] == dense[r].tolist(), (r, res[r]["tokens"], dense[r].tolist())
        # each rank holds only its 4 experts x 2 layers
        assert res[r]["local_expert_tensors"] == 4 * cfg.n_layers
        assert res[r]["stats"]["calls"] == (64 + N_NEW) * cfg.n_layers
    # some pairs crossed ranks in both directions
    assert res[0]["stats"]["recv_rows"] > 0 and res[1]["stats"]["recv_rows"] > 0
