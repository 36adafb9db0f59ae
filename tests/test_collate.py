"""Bench-line collation: scaling efficiency, clock flags, reference lines skipped (CPU only)."""

import json

from dsv4_flash_deployment_b200.bench.collate import collate, format_table, load_lines, main


def _line(n, v, reasons=(), mhz=1965.0):
    return {"metric": "output tok/s", "value": v, "unit": "tok/s", "n_gpus": n, "steps": 8, "warmup": 4,
            "ms_per_step": 24.5, "scaling": "weak", "vs_baseline": round(v / 8463.7, 3),
            "e2e": {"value": v * 0.99}, "c1_tpot_ms": {"value": 10.2},
            "clocks": {"sm_mhz": mhz, "sm_max_mhz": 1965.0, "reasons": list(reasons)}}


def test_collate_scaling_and_flags(tmp_path, capsys):
    f = tmp_path / "scale.json"
    lines = [_line(1, 5000.0), _line(2, 9000.0, ["sw_power_cap"]), _line(8, 20000.0, ["hw_thermal_slowdown"]),
             _line(4, 1.0, mhz=900.0), {"impl": "reference", "unavailable": "tpu only"}]
    f.write_text("noise\n" + "\n".join(json.dumps(x) for x in lines) + "\n")
    rows = collate(load_lines([str(f)]))
    assert [r["n_gpus"] for r in rows] == [1, 2, 4, 8]
    assert rows[1]["scaling_efficiency"] == 0.9 and rows[1]["power_capped"] and not rows[1]["clock_flags"]
    assert rows[2]["clock_flags"] == ["clock_low_no_reason"]
    assert rows[3]["clock_flags"] == ["hw_thermal_slowdown"] and rows[3]["scaling_efficiency"] == 0.5
    table = format_table(rows)
    assert table.count("\n") == len(rows) + 1 and "hw_thermal_slowdown" in table
    main([str(f), "--json"])
    assert json.loads(capsys.readouterr().out)[0]["per_gpu"] == 5000.0
