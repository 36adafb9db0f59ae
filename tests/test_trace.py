"""Layer-statistics trace (CPU): statistics of traced tensors and the env switch."""

import torch

from dsv4_flash_deployment_b200.utils import trace as tr


def test_layer_stats_and_format(monkeypatch):
    x = torch.zeros(4, 4, 8, dtype=torch.bfloat16)
    x[0, 0, 0] = 3.0
    x[1, 2, 3] = -4.0
    a = torch.full((4, 8), 0.5, dtype=torch.bfloat16)
    st = tr.layer_stats({2: x, "attn2": a, 0: torch.ones(2, 3)})
    assert list(st) == [0, 2]
    assert abs(st[2]["x"]["rms"] - (25.0 / 128) ** 0.5) < 1e-6
    assert st[2]["x"]["max"] == 4.0
    assert abs(st[2]["x"]["zero"] - 126 / 128) < 1e-9
    assert st[2]["attn"]["rms"] == 0.5 and st[2]["attn"]["zero"] == 0.0
    lines = tr.format_stats(st)
    assert lines[1].startswith("layer 2:") and "attn rms 0.5" in lines[1]
    monkeypatch.setenv("DSV4_TRACE_LAYER_STATS", "3")
    assert tr.trace_steps_from_env() == 3
    monkeypatch.setenv("DSV4_TRACE_LAYER_STATS", "yes")
    assert tr.trace_steps_from_env() == 1
    monkeypatch.delenv("DSV4_TRACE_LAYER_STATS")
    assert tr.trace_steps_from_env() == 0


import pytest  # noqa: E402


@pytest.mark.gpu
def test_engine_traces_first_steps(monkeypatch, caplog):
    """DSV4_TRACE_LAYER_STATS=2: the first two engine steps run eagerly with the
    trace and log one line per layer; later steps go back to graph replay."""
    import logging

    from dsv4_flash_deployment_b200.config import v4_flash_config
    from dsv4_flash_deployment_b200.engine.engine import Engine

    monkeypatch.setenv("DSV4_TRACE_LAYER_STATS", "2")
    # kernel dimensions of V4 (64 x 512 heads, 128-wide indexer heads), small elsewhere
    cfg = v4_flash_config(n_layers=3, dim=512, vocab_size=1024, padded_vocab_size=1024, q_lora_rank=256,
                          o_lora_rank=128, n_routed_experts=16, moe_inter_dim=256, index_n_heads=8, index_topk=8)
    eng = Engine.build(cfg, "cuda", max_seqs=2, max_batched_tokens=32, max_seq_len=128)
    with caplog.at_level(logging.INFO, logger="dsv4.trace"):
        out = eng.generate([list(range(10, 30))], 4, ignore_eos=True)
    assert len(out[0]) == 4
    lines = [r.getMessage() for r in caplog.records if r.name == "dsv4.trace"]
    assert len(lines) == 2 * cfg.n_layers
    assert all("rms" in ln for ln in lines)
    eng.check_errors()
