"""Verification runner on the GPU: parity against the CPU oracle, the Sinkhorn
negative control and a decode timing stage on the kernel-shaped V4 check model,
and the DSpark stage (speculative vs greedy tokens) on the V4.1 check model."""

import json

import pytest

from dsv4_flash_deployment_b200.verify import runner as vr

pytestmark = pytest.mark.gpu


def test_runner_stages_on_the_gpu(tmp_path):
    out = tmp_path / "v4"
    rc = vr.main(["--out", str(out), "--model", "v4-check", "--stages",
                  "cold_startup,parity_ref,parity_neg_control,perf_b2", "--perf-steps", "5", "--ctx", "64"])
    recs = {s: json.loads((out / f"{s}.json").read_text())
            for s in ("cold_startup", "parity_ref", "parity_neg_control", "perf_b2")}
    assert rc == 0, {s: (r.get("passed"), r.get("error")) for s, r in recs.items()}
    assert recs["parity_ref"]["cos_mean"] >= 0.995 and recs["parity_neg_control"]["cos_mean"] < 0.99
    assert recs["perf_b2"]["graph_captures"] > 0 and recs["cold_startup"]["device_allocated_gib"] > 0
    out2 = tmp_path / "v41"
    rc = vr.main(["--out", str(out2), "--model", "v4.1-check", "--stages", "dspark_verify"])
    d = json.loads((out2 / "dspark_verify.json").read_text())
    assert rc == 0, d.get("error")
    assert d["identical_fraction"] >= 0.9 and d["acceptance"]
