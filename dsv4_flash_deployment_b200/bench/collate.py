"""Collates ``bench.py`` JSON lines (one file per run, or many lines in one file)
into a scaling table: aggregate and per-GPU throughput, scaling efficiency
against the smallest GPU count, end-to-end value, C=1 TPOT and the clock
record of each run.  Runs whose clock record shows a thermal or hardware
slowdown, or SM clocks far below the maximum with no reason, are flagged (the
timing rules reject them); ``sw_power_cap`` is kept and noted.

The reference assembles its headline report the same way from per-run result
files (``megakernel/scripts/benchmark_megakernel_v6e16.py``,
``recipes/publish_to_ubench.py``).

    python -m dsv4_flash_deployment_b200.bench.collate BENCH_*.json SCALE_*.json [--json]
"""

from __future__ import annotations

import argparse
import json

REJECT_REASONS = {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"}


def load_lines(paths: list[str]) -> list[dict]:
    out = []
    for p in paths:
        with open(p) as f:
            for line in f:
                line = line.strip()
                if line.startswith("{"):
                    try:
                        d = json.loads(line)
                    except json.JSONDecodeError:
                        continue
                    if "value" in d and "n_gpus" in d and d.get("impl", "ours") != "reference":
                        out.append(d)
    return out


def clock_flags(d: dict) -> list[str]:
    c = d.get("clocks") or {}
    flags = sorted(set(c.get("reasons", [])) & REJECT_REASONS)
    mhz, mx = c.get("sm_mhz"), c.get("sm_max_mhz")
    if mhz and mx and mhz < 0.8 * mx and not c.get("reasons"):
        flags.append("clock_low_no_reason")
    return flags


def collate(lines: list[dict]) -> list[dict]:
    """One row per GPU count (the last line wins), sorted by GPU count."""
    by_n: dict[int, dict] = {}
    for d in lines:
        by_n[int(d["n_gpus"])] = d
    if not by_n:
        return []
    n0 = min(by_n)
    base = by_n[n0]["value"] / n0
    rows = []
    for n in sorted(by_n):
        d = by_n[n]
        per = d["value"] / n
        c1 = d.get("c1_tpot_ms")
        rows.append({
            "n_gpus": n, "metric": d.get("metric"), "value": d["value"], "unit": d.get("unit"),
            "per_gpu": round(per, 1),
            "scaling_efficiency": round(per / base, 3) if d.get("scaling", "weak") == "weak"
            else round(d["value"] / (by_n[n0]["value"] * n / n0), 3),
            "vs_baseline": d.get("vs_baseline"), "ms_per_step": d.get("ms_per_step"),
            "e2e": (d.get("e2e") or {}).get("value"),
            "c1_tpot_ms": c1.get("value") if isinstance(c1, dict) else c1,
            "sm_mhz": (d.get("clocks") or {}).get("sm_mhz"),
            "clock_flags": clock_flags(d),
            "power_capped": "sw_power_cap" in (d.get("clocks") or {}).get("reasons", []),
        })
    return rows


def format_table(rows: list[dict]) -> str:
    hdr = ["GPUs", "value", "per GPU", "efficiency", "vs baseline", "ms/step", "e2e", "C=1 ms", "SM MHz", "flags"]
    lines = ["| " + " | ".join(hdr) + " |", "|" + "---|" * len(hdr)]
    for r in rows:
        flags = ", ".join(r["clock_flags"] + (["sw_power_cap"] if r["power_capped"] else [])) or "-"
        vals = [r["n_gpus"], r["value"], r["per_gpu"], r["scaling_efficiency"], r["vs_baseline"], r["ms_per_step"],
                r["e2e"], r["c1_tpot_ms"], r["sm_mhz"], flags]
        lines.append("| " + " | ".join("-" if v is None else str(v) for v in vals) + " |")
    return "\n".join(lines)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("files", nargs="+")
    ap.add_argument("--json", action="store_true", help="print the rows as JSON instead of a table")
    a = ap.parse_args(argv)
    rows = collate(load_lines(a.files))
    print(json.dumps(rows) if a.json else format_table(rows))


if __name__ == "__main__":
    main()
