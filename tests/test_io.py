"""Checkpoint IO: safetensors reader/writer, validated loader, pre-shard blobs,
integrity manifests (corrupt-shard detection), native threaded reader."""

import json

import pytest
import torch

from dsv4_flash_deployment_b200.config import toy_v4_config
from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
from dsv4_flash_deployment_b200.io.integrity import IntegrityError, verify_manifest, write_manifest
from dsv4_flash_deployment_b200.io.preshard import load_shard, preshard
from dsv4_flash_deployment_b200.io.safetensors import (CheckpointError, load_checkpoint, read_tensors,
                                                       save_checkpoint, write_safetensors)


def _eq(a, b):
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def test_format_interop_with_reference_library(tmp_path):
    st = pytest.importorskip("safetensors.torch")
    t = {"a": torch.randn(3, 5).to(torch.bfloat16), "b": torch.arange(7, dtype=torch.int8),
         "c": torch.randn(4, 4), "d": (torch.randn(8, 16) * 3).to(torch.float8_e4m3fn)}
    write_safetensors(tmp_path / "ours.safetensors", t)
    back = st.load_file(str(tmp_path / "ours.safetensors"))
    assert all(_eq(back[k], t[k]) for k in t)
    st.save_file(t, str(tmp_path / "theirs.safetensors"))
    mine = read_tensors(tmp_path / "theirs.safetensors")
    assert all(_eq(mine[k], t[k]) for k in t)


def test_checkpoint_roundtrip_validation_and_shards(tmp_path):
    cfg = toy_v4_config()
    w = make_random_weights(cfg, seed=5, include_mtp=False)
    files = save_checkpoint(tmp_path / "ck", w, cfg, shard_bytes=2 << 20)
    assert len(files) > 1
    back = load_checkpoint(tmp_path / "ck", cfg)
    assert set(back) == set(w) and all(_eq(back[k], w[k]) for k in w)
    # a missing and a mis-shaped tensor are reported, not loaded
    bad = dict(w)
    del bad["layers.0.attn.wq_a.weight"]
    bad["layers.1.ffn.gate.bias"] = torch.zeros(3)
    save_checkpoint(tmp_path / "bad", bad, cfg)
    with pytest.raises(CheckpointError, match="1 missing.*1 mismatched"):
        load_checkpoint(tmp_path / "bad", cfg)


def test_preshard_ranks_and_integrity(tmp_path):
    cfg = toy_v4_config()
    w = make_random_weights(cfg, seed=6, include_mtp=False)
    save_checkpoint(tmp_path / "ck", w, cfg)
    preshard(tmp_path / "ck", tmp_path / "ps", cfg, world=2)
    for r in range(2):
        sh = load_shard(tmp_path / "ps", r, 2, verify=True)
        exp = {k for k in sh if ".experts." in k}
        ids = {int(k.split(".experts.")[1].split(".")[0]) for k in exp}
        assert ids == set(range(4 * r, 4 * r + 4))
        assert all(_eq(sh[k], w[k]) for k in sh)
        assert sum(1 for k in w if ".experts." not in k) == len(sh) - len(exp)
        meta = json.loads((tmp_path / "ps" / f"rank{r}-of-2.json").read_text())
        assert all(e["offset"] % 4096 == 0 for e in meta["tensors"].values())
    # manifest + a flipped byte is caught
    write_manifest(tmp_path / "ck")
    assert verify_manifest(tmp_path / "ck")["files"] >= 1
    f = sorted((tmp_path / "ck").glob("*.safetensors"))[0]
    b = bytearray(f.read_bytes())
    b[-100] ^= 0x40
    f.write_bytes(bytes(b))
    with pytest.raises(IntegrityError):
        verify_manifest(tmp_path / "ck")
    blob = tmp_path / "ps" / "rank1-of-2.bin"
    b = bytearray(blob.read_bytes())
    b[4096] ^= 1
    blob.write_bytes(bytes(b))
    with pytest.raises(ValueError, match="sha256"):
        load_shard(tmp_path / "ps", 1, 2, verify=True)


def test_engine_loads_checkpoint(tmp_path):
    from dsv4_flash_deployment_b200.engine.config import EngineConfig
    from dsv4_flash_deployment_b200.serving.launch import build_local_engine

    cfg = toy_v4_config()
    w = make_random_weights(cfg, seed=0, include_mtp=False)
    save_checkpoint(tmp_path / "ck", w, cfg)
    ec = EngineConfig(device="cpu", model="toy-v4", checkpoint=str(tmp_path / "ck"), max_seqs=2,
                      max_batched_tokens=32, max_model_len=64)
    a = build_local_engine(ec).generate([[0, 5, 9, 33, 70]], 3, ignore_eos=True)
    ec2 = EngineConfig(device="cpu", model="toy-v4", max_seqs=2, max_batched_tokens=32, max_model_len=64)
    b = build_local_engine(ec2).generate([[0, 5, 9, 33, 70]], 3, ignore_eos=True)
    assert a == b


def test_checkpoint_command_line_tools(tmp_path, capsys):
    """synth -> inspect -> verify -> preshard through the CLI; a checkpoint of
    another model is reported tensor by tensor and a corrupted file fails verify."""
    import json

    from dsv4_flash_deployment_b200.io.__main__ import main

    ck, sh = tmp_path / "ck", tmp_path / "sh"

    def run(*args):
        rc = main(list(args))
        return rc, json.loads(capsys.readouterr().out.strip().splitlines()[-1])

    rc, out = run("synth", "--model", "toy-v4", "--out", str(ck), "--shard-gib", "0.001")
    assert rc == 0 and out["tensors"] == 175 and out["files"] > 1
    rc, out = run("inspect", "--model", "toy-v4", "--ckpt", str(ck))
    assert rc == 0 and out["ok"] and out["missing"] == out["mismatched"] == out["unexpected"] == 0
    rc, out = run("inspect", "--model", "v4-check", "--ckpt", str(ck))
    assert rc == 1 and out["missing"] > 0 and out["first_missing"]
    rc, out = run("verify", "--ckpt", str(ck))
    assert rc == 0 and out["files"] == len(list(ck.glob("*.safetensors")))
    rc, out = run("preshard", "--model", "toy-v4", "--ckpt", str(ck), "--out", str(sh), "--world", "2")
    assert rc == 0 and len(out["files"]) == 2
    f = sorted(ck.glob("*.safetensors"))[0]
    raw = bytearray(f.read_bytes())
    raw[-1] ^= 0xFF
    f.write_bytes(bytes(raw))
    rc, out = run("verify", "--ckpt", str(ck))
    assert rc == 1 and "sha256 mismatch" in out["error"]
