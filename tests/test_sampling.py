"""Temperature sampling rule of the device head (``DSV4Model._gumbel``), run on
CPU tensors: rows at temperature 0 keep their logits exactly (greedy), and the
argmax of logits + T * Gumbel noise follows softmax(logits / T)."""

import types

import torch

import pytest

from dsv4_flash_deployment_b200.models.model import DSV4Model, SeqChunk, StepMeta
from dsv4_flash_deployment_b200.models.sampling import (SamplingParams, chosen_logprob, gumbel_, logprob_top,
                                                        top_k_top_p_mask_)
from dsv4_flash_deployment_b200.config import toy_v4_config


def _head(logits, temps):
    h = types.SimpleNamespace(logits=logits.clone(), m_temp=temps.clone(), _gnoise=None)
    DSV4Model._gumbel(h, logits.shape[0])
    return h.logits


def test_zero_temperature_rows_are_untouched():
    torch.manual_seed(0)
    lg = torch.randn(3, 50)
    out = _head(lg, torch.tensor([0.0, 1.0, 0.0]))
    assert torch.equal(out[0], lg[0]) and torch.equal(out[2], lg[2])
    assert not torch.equal(out[1], lg[1])


def test_gumbel_max_follows_softmax():
    torch.manual_seed(1)
    V, T, n = 6, 0.7, 40000
    base = torch.tensor([1.0, 0.5, 0.0, -0.5, 2.0, 0.2])
    lg = base.repeat(n, 1)
    picks = _head(lg, torch.full((n,), T)).argmax(1)
    freq = torch.bincount(picks, minlength=V).float() / n
    want = torch.softmax(base / T, 0)
    assert (freq - want).abs().max().item() < 0.01, (freq, want)


def test_step_meta_carries_per_row_temperatures():
    cfg = toy_v4_config()
    m = StepMeta(cfg, [SeqChunk(0, 0, [5, 6, 7], True, temperature=0.8), SeqChunk(1, 0, [9], False),
                       SeqChunk(2, 4, [3], True)])
    assert m.sampling and len(m.sample_rows) == 2
    assert abs(m.temps[0] - 0.8) < 1e-6 and m.temps[1] == 0.0
    g = StepMeta(cfg, [SeqChunk(0, 0, [5], True)])
    assert not g.sampling and g.key() != m.key()


def _kept(row):
    return set(torch.nonzero(torch.isfinite(row)).flatten().tolist())


def test_top_k_keeps_the_k_largest():
    torch.manual_seed(2)
    lg = torch.randn(4, 40)
    out = lg.clone()
    top_k_top_p_mask_(out, torch.tensor([1.0, 1.0, 0.5, 1.0]), torch.tensor([3, 1, 7, 0], dtype=torch.int32),
                      torch.ones(4))
    for i, k in enumerate([3, 1, 7, 40]):
        assert _kept(out[i]) == set(torch.topk(lg[i], k).indices.tolist())
        fin = torch.isfinite(out[i])
        assert torch.equal(out[i][fin], lg[i][fin])


def test_top_p_is_the_smallest_nucleus_at_temperature():
    torch.manual_seed(3)
    V = 30
    lg = torch.randn(6, V) * 2
    temps = torch.tensor([1.0, 0.5, 2.0, 1.0, 0.7, 1.0])
    ps = torch.tensor([0.5, 0.9, 0.3, 0.999, 0.05, 1.0])
    ks = torch.tensor([0, 0, 0, 0, 0, 5], dtype=torch.int32)
    out = lg.clone()
    top_k_top_p_mask_(out, temps, ks, ps)
    for i in range(6):
        order = torch.argsort(lg[i], descending=True)
        kk = V if ks[i] == 0 else int(ks[i])
        pr = torch.softmax(lg[i][order[:kk]] / temps[i], 0)
        want = []
        mass = 0.0
        for j in range(kk):
            if ps[i] < 1.0 and mass >= ps[i]:
                break
            want.append(int(order[j]))
            mass += float(pr[j])
        assert _kept(out[i]) == set(want), (i, sorted(_kept(out[i])), sorted(want))


def test_top_k_then_top_p_sampling_frequencies():
    torch.manual_seed(4)
    base = torch.tensor([2.0, 1.5, 1.0, 0.5, 0.0, -1.0])
    n, T = 30000, 1.0
    lg = base.repeat(n, 1)
    top_k_top_p_mask_(lg, torch.full((n,), T), torch.full((n,), 4, dtype=torch.int32), torch.full((n,), 0.8))
    gumbel_(lg, torch.full((n,), T), torch.empty_like(lg))
    picks = lg.argmax(1)
    freq = torch.bincount(picks, minlength=6).float() / n
    p4 = torch.softmax(base[:4] / T, 0)          # top-4, then the smallest prefix with mass >= 0.8
    keep = 1
    while p4[:keep].sum() < 0.8:
        keep += 1
    want = torch.zeros(6)
    want[:keep] = torch.softmax(base[:keep] / T, 0)
    assert (freq - want).abs().max().item() < 0.012, (freq, want)


def test_logprob_rule_matches_log_softmax():
    torch.manual_seed(5)
    lg = torch.randn(3, 50) * 3
    lse, vals, ids = logprob_top(lg, 5)
    lsm = torch.log_softmax(lg, -1)
    assert torch.allclose(vals, torch.topk(lsm, 5).values, atol=1e-5)
    assert torch.equal(ids, torch.topk(lg, 5).indices)
    pick = torch.tensor([7, 0, 49], dtype=torch.int32)
    assert torch.allclose(chosen_logprob(lg, pick, lse), lsm[torch.arange(3), pick.long()], atol=1e-5)


def test_step_meta_filtering_and_logprob_rows():
    cfg = toy_v4_config()
    m = StepMeta(cfg, [SeqChunk(0, 0, [5, 6], True, temperature=0.8, top_k=4, logprobs=2),
                       SeqChunk(1, 0, [9], True), SeqChunk(2, 3, [1], True, temperature=0.0, top_p=0.5)])
    assert m.filtering and m.want_lp and m.lp_want == [2, None, None]
    assert m.topk.tolist() == [4, 0, 0] and abs(m.topp[2] - 0.5) < 1e-6
    # top-p on a greedy row changes nothing: no filtering pass
    g = StepMeta(cfg, [SeqChunk(0, 0, [5], True, top_p=0.5)])
    assert not g.filtering and not g.want_lp
    assert g.key() == StepMeta(cfg, [SeqChunk(0, 0, [5], True)]).key() != m.key()
    assert StepMeta(cfg, [SeqChunk(0, 0, [5], True, logprobs=0)]).key() != g.key()
    p = m.padded(64, 8, 7)
    assert len(p.topk) == len(p.sample_rows) == len(p.lp_want) == len(p.temps) and p.n_out == 3
    assert p.filtering and p.want_lp


def test_sampling_params_validation():
    assert SamplingParams(0.5, 3, 0.9, 2).filters
    assert not SamplingParams(0.0, 3, 0.9).filters
    for bad in (dict(temperature=-1), dict(top_k=-2), dict(top_p=0.0), dict(top_p=1.2), dict(logprobs=21)):
        with pytest.raises(ValueError):
            SamplingParams(**bad)
