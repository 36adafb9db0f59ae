"""Temperature sampling rule of the device head (``DSV4Model._gumbel``), run on
CPU tensors: rows at temperature 0 keep their logits exactly (greedy), and the
argmax of logits + T * Gumbel noise follows softmax(logits / T)."""

import math
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


def test_seeded_noise_is_splitmix64_and_split_invariant():
    from dsv4_flash_deployment_b200.models import sampling as S

    keys = torch.tensor([S.seed_key(123, 5), S.seed_key(-7, 0), S.seed_key(2 ** 40 + 3, 99)])
    g = S.seeded_gumbel(keys, 12)
    m = (1 << 64) - 1
    for i, k in enumerate(keys.tolist()):
        for v in range(12):
            # entry (s, v) is SplitMix64 at state key + (v - 1) * gamma, top 24 bits as a uniform
            z = S.splitmix64(((k & m) + (v - 1) * 0x9E3779B97F4A7C15) & m)
            u = ((z >> 40) + 0.5) / 2 ** 24
            assert abs(-math.log(-math.log(u)) - g[i, v].item()) < 1e-5
    # a vocabulary shard starting at v0 draws the same columns
    assert torch.equal(S.seeded_gumbel(keys, 5, 7), g[:, 7:12])
    # Gumbel-max over seeded noise still samples softmax(logits / T)
    base = torch.tensor([1.0, 0.5, 0.0, -0.5, 2.0, 0.2])
    n, T = 30000, 0.8
    ks = torch.tensor([S.seed_key(s, 11) for s in range(n)])
    picks = (base / T + S.seeded_gumbel(ks, 6)).argmax(1)
    freq = torch.bincount(picks, minlength=6).float() / n
    assert (freq - torch.softmax(base / T, 0)).abs().max().item() < 0.012


def test_seeded_rows_in_the_head_rule():
    from dsv4_flash_deployment_b200.models import sampling as S

    lg = torch.zeros(3, 40)
    keys = torch.tensor([S.seed_key(5, 3), 0, S.seed_key(5, 3)])
    has = torch.tensor([True, False, True])
    a, b = lg.clone(), lg.clone()
    gumbel_(a, torch.ones(3), torch.empty_like(a), (keys, has))
    gumbel_(b, torch.ones(3), torch.empty_like(b), (keys, has))
    assert torch.equal(a[0], b[0]) and torch.equal(a[0], a[2])      # same (seed, position): same noise
    assert not torch.equal(a[1], b[1])                               # unseeded row: the generator's


def test_step_meta_seed_keys_follow_positions():
    from dsv4_flash_deployment_b200.models.sampling import seed_key

    cfg = toy_v4_config()
    m = StepMeta(cfg, [SeqChunk(0, 4, [5, 6, 7], True, temperature=1.0, seed=9), SeqChunk(1, 2, [1], True)])
    assert m.seeded and m.has_seed.tolist() == [True, False]
    assert m.seedkey[0] == seed_key(9, 6)
    greedy_seeded = StepMeta(cfg, [SeqChunk(0, 4, [5], True, seed=9)])
    assert not greedy_seeded.seeded
    p = m.padded(64, 8, 7)
    assert len(p.seedkey) == len(p.has_seed) == len(p.sample_rows)


def test_seeded_request_repeats_whatever_its_batch():
    from dsv4_flash_deployment_b200.engine.config import EngineConfig
    from dsv4_flash_deployment_b200.serving.launch import build_local_engine

    eng = build_local_engine(EngineConfig(device="cpu", model="toy-v4", max_seqs=3, max_batched_tokens=48,
                                          chunk_size=16, max_model_len=96))
    p = [3 + (7 * i) % 200 for i in range(20)]
    alone = eng.add_request(p, 8, ignore_eos=True, temperature=3.0, seed=42)
    while not alone.finished:
        eng.step()
    others = [eng.add_request([9, 8, 7, 6] * k, 10, ignore_eos=True, temperature=3.0) for k in (2, 3)]
    again = eng.add_request(p, 8, ignore_eos=True, temperature=3.0, seed=42)
    other_seed = eng.add_request(p, 8, ignore_eos=True, temperature=3.0, seed=43)
    while not all(r.finished for r in others + [again, other_seed]):
        eng.step()
    assert again.output == alone.output
    assert other_seed.output != alone.output
