"""Temperature sampling rule of the device head (``DSV4Model._gumbel``), run on
CPU tensors: rows at temperature 0 keep their logits exactly (greedy), and the
argmax of logits + T * Gumbel noise follows softmax(logits / T)."""

import types

import torch

from dsv4_flash_deployment_b200.models.model import DSV4Model, SeqChunk, StepMeta
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
