"""Engram tables in shared files on the GPU: a random-init V4.1 model whose
tables live in shared files under /dev/shm (filled by the first model, mapped
by the next)
gives the logits of the same model with private tables (cosine >= 0.99999 at
every position: the same tables and weights, the same kernels; a wrong table
row moves the logits far more).  All three page-lock
their host pages (the second and third over two mappings of the same file)
and gather rows from them with the zero-copy kernel."""

import glob
import os
import uuid

import pytest
import torch

from dsv4_flash_deployment_b200.engine.builder import build_model

from test_model_gpu import _steps, small_v41

pytestmark = pytest.mark.gpu


@pytest.fixture
def shm_prefix():
    if not os.path.isdir("/dev/shm"):
        pytest.skip("no /dev/shm")
    prefix = f"/dev/shm/dsv4_engram_test_{uuid.uuid4().hex[:12]}"
    yield prefix
    for f in glob.glob(prefix + ".*"):
        os.remove(f)


def test_shared_engram_tables_match_private_tables(shm_prefix):
    cfg = small_v41(engram_layer_ids=(1, 3), engram_max_ngram_size=4, engram_n_heads=8, engram_head_dim=64,
                    engram_vocab_size=2048, engram_num_embeddings=(51342, 54000), index_k_mode="intended")
    prefix = shm_prefix
    kw = dict(max_tokens=64, n_slots=3, max_seq_len=64, seed=4)
    private = build_model(cfg, "cuda", **kw)
    filled = build_model(cfg, "cuda", engram_shm=prefix, **kw)
    for lid in (1, 3):
        for part in ("q", "sf"):
            assert os.path.exists(f"{prefix}.l{lid}.{part}.ready")
    mapped = build_model(cfg, "cuda", engram_shm=prefix, **kw)
    g = torch.Generator().manual_seed(3)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (30, 22)]
    want = _steps(private, cfg, seqs, 12)
    for m in (filled, mapped):
        got = _steps(m, cfg, seqs, 12)
        assert got.keys() == want.keys()
        cos = [float(torch.nn.functional.cosine_similarity(got[k], want[k], dim=-1)) for k in want]
        assert min(cos) >= 0.99999, min(cos)
