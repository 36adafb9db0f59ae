"""Deployment files (CPU): the container entrypoint is valid bash, and the
Kubernetes manifest's server arguments parse with the engine's own CLI, so the
manifest cannot drift from the flags the server accepts."""

import subprocess
from pathlib import Path

import yaml

from dsv4_flash_deployment_b200.engine.config import EngineConfig

ROOT = Path(__file__).resolve().parent.parent


def test_entrypoint_is_valid_bash():
    r = subprocess.run(["bash", "-n", str(ROOT / "deploy" / "entrypoint.sh")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_manifest_args_parse_with_the_server_cli():
    docs = list(yaml.safe_load_all((ROOT / "deploy" / "k8s" / "dsv4-b200-server.yaml").read_text()))
    dep = next(d for d in docs if d["kind"] == "Deployment")
    c = dep["spec"]["template"]["spec"]["containers"][0]
    ec = EngineConfig.from_args(c["args"])
    assert ec.parallel == "ep" and ec.ep_transport == "fused"
    assert c["resources"]["limits"]["nvidia.com/gpu"] == 8
    assert any(e["name"] == "NGPU" for e in c["env"])


def test_dockerfile_builds_the_extension_and_uses_the_entrypoint():
    txt = (ROOT / "deploy" / "Dockerfile").read_text()
    assert "g.build()" in txt and "deploy/entrypoint.sh" in txt
