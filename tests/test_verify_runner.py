"""Verification runner (CPU plumbing): stage records with their pass rules, the
negative control, skipped stages with a reason, resume (passed stages kept,
failed ones rerun, ``--force``), and a failing stage recorded without stopping
the run."""

import json

from dsv4_flash_deployment_b200.verify import runner as vr

ARGS = ["--model", "toy-v4", "--device", "cpu", "--perf-steps", "3", "--ctx", "20", "--n-seqs", "2",
        "--seq-len", "30"]


def _rec(out, st):
    return json.loads((out / f"{st}.json").read_text())


def test_stages_records_and_resume(tmp_path, monkeypatch):
    out = tmp_path / "v"
    rc = vr.main(["--out", str(out), "--stages", "cold_startup,parity_ref,parity_neg_control,perf_b2,dspark_verify",
                  *ARGS])
    assert rc == 0
    p = _rec(out, "parity_ref")
    assert p["passed"] and p["cos_min"] > 0.9999 and p["top1"] == 1.0 and p["positions"] > 10
    assert p["hardware"]["torch"] and p["model"] == "toy-v4" and "rule" in p
    n = _rec(out, "parity_neg_control")
    assert n["passed"] and n["cos_mean"] < 0.99
    perf = _rec(out, "perf_b2")
    assert perf["passed"] and perf["batch"] == 2 and perf["tpot_ms_median"] > 0
    d = _rec(out, "dspark_verify")
    assert d["skipped"] and not d["passed"] and "MTP" in d["reason"]
    summ = _rec(out, "summary")
    assert summ["stages"]["parity_ref"] == "passed" and summ["stages"]["gsm8k"] == "not run"
    md = (out / "summary.md").read_text()
    assert "| parity_ref | passed |" in md and "| gsm8k | not run |" in md and "cos_mean" in md

    # resume: passed stages are kept as they are; a failing stage is recorded, the run goes on
    t_before = _rec(out, "parity_ref")["time"]

    def boom(self, st):
        raise RuntimeError("injected failure")
    monkeypatch.setattr(vr.Runner, "stage_perf_b1", boom)
    rc = vr.main(["--out", str(out), "--stages", "parity_ref,perf_b1,cold_startup", *ARGS])
    assert rc == 1
    assert _rec(out, "parity_ref")["time"] == t_before
    f = _rec(out, "perf_b1")
    assert not f["passed"] and "injected failure" in f["error"]
    assert _rec(out, "summary")["stages"]["perf_b1"] == "failed"
    monkeypatch.undo()
    # the failed stage runs again; --force reruns a passed one
    assert vr.main(["--out", str(out), "--stages", "perf_b1", *ARGS]) == 0
    assert _rec(out, "perf_b1")["passed"]
    assert vr.main(["--out", str(out), "--stages", "cold_startup", "--force", *ARGS]) == 0


def test_unknown_stage_is_refused(tmp_path):
    import pytest

    with pytest.raises(SystemExit):
        vr.main(["--out", str(tmp_path), "--stages", "parity_ref,bogus", *ARGS])


def test_golden_files_round_trip_and_catch_a_changed_token(tmp_path):
    from dsv4_flash_deployment_b200.verify import golden as G

    path = tmp_path / "g.json"
    assert G.main(["make", "--model", "toy-v4", "--prompts", "2", "--steps", "5", "--prompt-len", "9",
                   "--out", str(path)]) == 0
    gold = json.loads(path.read_text())
    assert gold["model"] == "toy-v4" and len(gold["sequences"]) == 2
    s0 = gold["sequences"][0]
    assert len(s0["tokens"]) == 5 and all(lp <= 0 for lp in s0["logprobs"]) and all(g >= 0 for g in s0["top2_gap"])
    assert G.main(["check", str(path), "--device", "cpu"]) == 0
    # a golden token that is not the model's argmax (and not a near tie) is caught
    s0["tokens"][2] = (s0["tokens"][2] + 1) % 1000
    s0["top2_gap"][2] = 1.0
    path.write_text(json.dumps(gold))
    assert G.main(["check", str(path), "--device", "cpu", "--min-tie-aware", "1.0"]) == 1
    # the runner's golden stage reads a file for its own model
    out = tmp_path / "v"
    assert vr.main(["--out", str(out), "--stages", "golden", "--golden", str(path), *ARGS, "--min-tie-aware", "0.5"]) == 0
    rec = _rec(out, "golden")
    assert rec["passed"] and rec["strict_top1"] < 1.0 and rec["positions"] == 10
    assert G.bf16_ulp(1.0) == 2 ** -7 and G.bf16_ulp(-3.0) == 2 ** -6
