"""Typed engine configuration: precedence (defaults < file < flags), ModelConfig
overrides, typed flags, unknown-field errors (CPU only)."""

import json

import pytest

from dsv4_flash_deployment_b200.engine.config import EngineConfig


def test_defaults_file_flags_precedence(tmp_path):
    f = tmp_path / "ec.json"
    f.write_text(json.dumps({"max_seqs": 64, "max_model_len": 4096, "parallel": "tp",
                             "overrides": {"n_layers": 4}}))
    ec = EngineConfig.from_args(["--config-file", str(f), "--max-seqs", "8", "--kv-block", "64",
                                 "--override", "vocab_size=2048", "--no-use-cuda-graphs"])
    assert ec.max_seqs == 8                      # flag beats file
    assert ec.max_model_len == 4096              # file beats default
    assert ec.parallel == "tp"
    assert ec.kv_block == 64 and isinstance(ec.kv_block, int)
    assert ec.kv_pool_tokens == 0
    assert ec.use_cuda_graphs is False
    assert ec.overrides == {"n_layers": 4, "vocab_size": 2048}
    assert EngineConfig().max_batched_tokens == ec.max_batched_tokens   # untouched default
    d = ec.to_dict()
    assert d["kv_block"] == 64 and d["overrides"]["vocab_size"] == 2048


def test_yaml_file_and_unknown_fields(tmp_path):
    y = tmp_path / "ec.yaml"
    y.write_text("max_seqs: 3\nchunk_size: 256\n")
    ec = EngineConfig.from_args(["--config-file", str(y)])
    assert ec.max_seqs == 3 and ec.chunk_size == 256
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps({"max_sequences": 3}))
    with pytest.raises(ValueError, match="unknown EngineConfig fields"):
        EngineConfig.from_args(["--config-file", str(bad)])


def test_model_config_resolution():
    ec = EngineConfig(model="v4.1-flash", overrides={"n_layers": 2})
    cfg = ec.model_config()
    assert cfg.n_layers == 2 and cfg.family == "v4.1"
