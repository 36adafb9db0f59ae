"""Negative controls on the device model: perturbing one component must move the
logits (the reference's megakernel verification perturbs five components and
requires max |diff| > 1e-2, ``MK/scripts/verify_reference_engine.py:253-334``).
A component whose kernel silently contributed nothing would pass the parity
tests' cosine bars on random weights but fail here.  The unperturbed model,
rebuilt from the same weights, must reproduce the logits (the kernels are
deterministic)."""

import pytest
import torch

from dsv4_flash_deployment_b200.engine.builder import build_model
from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
from dsv4_flash_deployment_b200.models.model import SeqChunk, StepMeta
from dsv4_flash_deployment_b200.ops.gemm import ErrorWord

from test_model_gpu import small_v41

pytestmark = pytest.mark.gpu

N_DEC = 3


def _cfg():
    # V4.1 structure with Engram layers; prompts longer than 2 x index_topk so the
    # indexer really selects
    return small_v41(engram_layer_ids=(1, 3), engram_max_ngram_size=4, engram_n_heads=8, engram_head_dim=64,
                     engram_vocab_size=2048, engram_num_embeddings=(51342, 54000), index_k_mode="intended")


def _logits(cfg, w, seqs, perturb=None) -> torch.Tensor:
    model = build_model(cfg, "cuda", max_tokens=128, n_slots=4, max_seq_len=128, weights=w)
    if perturb is not None:
        perturb(model)
    out = []
    n = len(seqs)
    steps = [StepMeta(cfg, [SeqChunk(i, 0, s[:-N_DEC], True) for i, s in enumerate(seqs)])]
    for k in range(N_DEC):
        steps.append(StepMeta(cfg, [SeqChunk(i, len(s) - N_DEC + k, [s[len(s) - N_DEC + k]], True)
                                    for i, s in enumerate(seqs)]))
    for meta in steps:
        model.upload(meta)
        model.forward(meta)
        torch.cuda.synchronize()
        ErrorWord.check("cuda")
        out.append(model.logits[:n, : cfg.vocab_size].float().cpu())
    return torch.cat(out)


def _zero_compressor(m):
    for L in m.layers:
        if L.comp_norm is not None:
            L.comp_norm.zero_()


def _negate_indexer_heads(m):
    for L in m.layers:
        if L.idx_wproj is not None:
            L.idx_wproj.neg_()


def _negate_router(m):
    for L in m.layers:
        L.gate_w.neg_()


def _zero_engram_gate(m):
    for wgt in m.engram.wgt:
        wgt.zero_()


def _drop_sinks(m):
    for L in m.layers:
        L.sink.fill_(-30.0)


PERTURB = {"compressor": _zero_compressor, "indexer": _negate_indexer_heads, "router": _negate_router,
           "engram": _zero_engram_gate, "attention_sink": _drop_sinks}


@pytest.fixture(scope="module")
def base():
    torch.manual_seed(4)
    cfg = _cfg()
    w = make_random_weights(cfg, seed=9)
    seqs = [torch.randint(0, cfg.vocab_size, (n,)).tolist() for n in (44, 37)]
    return cfg, w, seqs, _logits(cfg, w, seqs)


def test_rebuilt_model_reproduces_logits(base):
    cfg, w, seqs, ref = base
    again = _logits(cfg, w, seqs)
    assert (again - ref).abs().max().item() < 1e-3


@pytest.mark.parametrize("name", sorted(PERTURB))
def test_perturbing_a_component_moves_the_logits(base, name):
    cfg, w, seqs, ref = base
    got = _logits(cfg, w, seqs, PERTURB[name])
    assert (got - ref).abs().max().item() > 1e-2, name
