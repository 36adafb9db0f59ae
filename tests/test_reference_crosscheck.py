"""Cross-checks against the reference's own code where it runs on a CPU without
its TPU stack: its configuration tables and its Engram hasher and token map
(pure numpy / sympy / tokenizers; the model oracle itself needs JAX, which this
image does not have).

The reference is looked up at ``DSV4_REFERENCE_ROOT`` (a checkout: the directory
that holds ``models/``), else at the repository's ``baseline/_ref`` (the
git-ignored place the reference is installed into); without either, every test
here is skipped.  Checked:

* the V4.1-Flash hyperparameters and the reference's ``tiny_config`` against
  ``config.py`` field by field;
* Engram row ids of random token sequences (full V4.1 layout and the tiny one)
  against the reference's ``compute_engram_hash_ids``, bit for bit;
* the tokenizer-normalized compressed token map against the reference's
  ``build_compressed_token_map`` on a tokenizer fixture;
* the checkpoint contract: every tensor name, dtype and shape against the
  reference's ``expected_checkpoint_specs`` (full V4.1 and tiny, MTP stages
  included), a checkpoint written by the reference's
  ``write_synthetic_checkpoint`` loaded by this library's validated reader bit
  for bit, and one written by this library read by the reference's
  ``SafetensorsCheckpoint`` bit for bit.
"""

import dataclasses
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = os.environ.get("DSV4_REFERENCE_ROOT") or str(Path(__file__).resolve().parent.parent / "baseline" / "_ref")
PKG = Path(ROOT) / "models" / "DeepSeekV4.1-Flash-v6e16" / "tpu-v7x" if ROOT else None

pytestmark = pytest.mark.skipif(PKG is None or not (PKG / "deepseek_v41" / "config.py").exists(),
                                reason="no reference checkout (DSV4_REFERENCE_ROOT or baseline/_ref)")


@pytest.fixture(scope="module")
def ref():
    pytest.importorskip("sympy")
    sys.path.insert(0, str(PKG))
    try:
        from deepseek_v41 import config as rc
        from deepseek_v41 import engram_hash as rh
    finally:
        sys.path.remove(str(PKG))
    return rc, rh


@pytest.fixture(scope="module")
def ref_ckpt():
    pytest.importorskip("ml_dtypes")
    sys.path.insert(0, str(PKG))
    try:
        from deepseek_v41 import checkpoint as rk
        from deepseek_v41 import config as rc
    finally:
        sys.path.remove(str(PKG))
    return rc, rk


def _same(ours, theirs, skip=()):
    diffs = {}
    for f in dataclasses.fields(theirs):
        if f.name in skip or not hasattr(ours, f.name):
            continue
        a, b = getattr(ours, f.name), getattr(theirs, f.name)
        if isinstance(b, (list, tuple)):
            a, b = tuple(a), tuple(b)
        if a != b:
            diffs[f.name] = (a, b)
    return diffs


def test_v41_config_tables_match(ref):
    from dsv4_flash_deployment_b200.config import v41_flash_config, v41_tiny_config

    rc, _ = ref
    assert _same(v41_flash_config(), rc.DSV41Config()) == {}
    assert _same(v41_tiny_config(), rc.tiny_config()) == {}
    # every reference field has a counterpart here
    missing = [f.name for f in dataclasses.fields(rc.DSV41Config) if not hasattr(v41_flash_config(), f.name)]
    assert missing == []


@pytest.mark.parametrize("which", ["tiny", "full"])
def test_engram_row_ids_match_bit_for_bit(ref, which):
    from dsv4_flash_deployment_b200.config import v41_flash_config, v41_tiny_config
    from dsv4_flash_deployment_b200.ref.engram import EngramHasher

    rc, rh = ref
    ours_cfg, theirs_cfg = ((v41_tiny_config(), rc.tiny_config()) if which == "tiny"
                            else (v41_flash_config(), rc.DSV41Config()))
    rng = np.random.default_rng(7)
    ids = rng.integers(0, ours_cfg.vocab_size, size=(3, 41), dtype=np.int64)
    ids[1, 5:9] = ours_cfg.engram_pad_id           # pad tokens inside a sequence
    want = rh.compute_engram_hash_ids(ids, theirs_cfg)          # [B, L, layers, cols]
    h = EngramHasher(ours_cfg)
    for b in range(ids.shape[0]):
        got = h.hash(h.compress(ids[b]), np.arange(ids.shape[1]))
        assert np.array_equal(got, want[b]), which


def test_compressed_token_map_matches(ref, tmp_path):
    tokenizers = pytest.importorskip("tokenizers")
    from dsv4_flash_deployment_b200.ref.engram import compressed_token_map

    _, rh = ref
    vocab = ["<unk>", "Hello", "hello", "HÉLLO", " ", "\t\t", "ﬁne", "fine", "Straße", "x\ny", "x y", "café",
             "cafe", "  Word　", "Ⅻ", "İ", " ", "á"]
    tok = tokenizers.Tokenizer(tokenizers.models.WordLevel({t: i for i, t in enumerate(vocab)}, unk_token="<unk>"))
    p = tmp_path / "tokenizer.json"
    tok.save(str(p))
    want, wc = rh.build_compressed_token_map(str(p))
    got, gc = compressed_token_map(str(p))
    assert gc == wc and got.tolist() == want.tolist()
    # no tokenizer: id % C on both sides
    w2, c2 = rh.build_compressed_token_map(None, vocab_size=129280)
    g2, d2 = compressed_token_map(None, 129280)
    assert d2 == c2 and np.array_equal(g2, w2)


@pytest.mark.parametrize("which", ["tiny", "full"])
def test_checkpoint_specs_match(ref_ckpt, which):
    from dsv4_flash_deployment_b200.config import v41_flash_config, v41_tiny_config
    from dsv4_flash_deployment_b200.io.checkpoint_spec import checkpoint_specs

    rc, rk = ref_ckpt
    ours_cfg, theirs_cfg = ((v41_tiny_config(), rc.tiny_config()) if which == "tiny"
                            else (v41_flash_config(), rc.DSV41Config()))
    want = {k: (t, tuple(s)) for k, (t, s) in rk.expected_checkpoint_specs(theirs_cfg, include_mtp=True).items()}
    got = {k: (t, tuple(s)) for k, (t, s) in checkpoint_specs(ours_cfg, include_mtp=True).items()}
    assert sorted(set(want) - set(got)) == [] and sorted(set(got) - set(want)) == []
    diff = {k: (got[k], want[k]) for k in want if got[k] != want[k]}
    assert diff == {}


def _bytes(x):
    import numpy as np
    import torch

    if isinstance(x, torch.Tensor):
        return x.contiguous().view(torch.uint8).numpy().tobytes()
    return np.ascontiguousarray(x).view(np.uint8).tobytes()


def test_reference_checkpoint_loads_here_and_ours_loads_there(ref_ckpt, tmp_path):
    from dsv4_flash_deployment_b200.config import v41_tiny_config
    from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
    from dsv4_flash_deployment_b200.io.safetensors import load_checkpoint, save_checkpoint

    from dsv4_flash_deployment_b200.config import ModelConfig

    rc, rk = ref_ckpt
    theirs = rk.write_synthetic_checkpoint(rc.tiny_config(), tmp_path / "theirs", seed=5, num_shards=3)
    # the checkpoint's config.json, read by this library's loader, is the same model
    cfg_here = ModelConfig.from_json(tmp_path / "theirs" / "config.json")
    assert _same(cfg_here, rc.tiny_config()) == {}
    got = load_checkpoint(tmp_path / "theirs", cfg_here, include_mtp=True)
    assert set(got) == set(theirs)
    bad = [k for k in theirs if _bytes(got[k]) != _bytes(theirs[k])]
    assert bad == []

    ours = make_random_weights(v41_tiny_config(), seed=6, include_mtp=True)
    save_checkpoint(tmp_path / "ours", ours, v41_tiny_config(), shard_bytes=1 << 20)
    reader = rk.SafetensorsCheckpoint(tmp_path / "ours")
    assert sorted(reader.keys()) == sorted(ours)
    bad = [k for k in ours if _bytes(reader.read_tensor(k)) != _bytes(ours[k])]
    assert bad == []
