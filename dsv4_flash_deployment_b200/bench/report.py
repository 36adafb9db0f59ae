"""Markdown report of served concurrency sweeps.

Reads the row files ``bench/sweep.py`` writes (a list of rows, or an object
with ``rows`` plus a description / hardware record, as in ``results/raw/``),
one or more per workload shape, and renders:

* a summary table: peak output tok/s and the concurrency it came at, requests
  per second, mean TTFT and TPOT at the highest concurrency measured;
* one table per shape with every concurrency's row (throughput, per-GPU
  throughput, requests/s, TTFT mean / p50 / p90, TPOT, completed / failed);
* the published reference numbers beside this build's (the reference's TPU
  v6e-16 sweep rows for the same shapes), with the ratio.

A concurrency that a file does not contain, or whose requests failed, is shown
with that reason, never left blank or interpolated.  The reference renders its
sweep report the same way from its sweep files
(``DeepSeekV4-Flash-v6e16/scripts/report.py``; output
``results/benchmark_sweep_report.md``), with PNG charts that this renderer
leaves out (no plotting library in the image).

    python -m dsv4_flash_deployment_b200.bench.report results/raw/1k1k_b200x1.json [more.json ...] \
        --title "DeepSeek-V4-Flash on 1 x B200" --out report.md
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

SHAPE_LABELS = {"1k1k": "1k/1k (balanced)", "8k1k": "8k/1k (prefill-heavy)", "1k8k": "1k/8k (reasoning)"}

# The reference's published peak rows (TPU v6e-16, vLLM + tpu-inference):
# DeepSeekV4-Flash-v6e16/results/raw/{1k1k,8k1k,1k8k}.json, C = 512 rows
# (tok/s at :236, TPOT at :242).
REFERENCE_V4 = {
    "name": "DeepSeek-V4-Flash, vLLM + tpu-inference on TPU v6e-16",
    "1k1k": {"peak": 8463.70, "conc": 512, "tpot_ms": 50.19, "ttft_s": 10.03},
    "8k1k": {"peak": 1758.53, "conc": 512, "tpot_ms": 52.56, "ttft_s": 132.31},
    "1k8k": {"peak": 8067.90, "conc": 512, "tpot_ms": 40.32, "ttft_s": 10.42},
}


def load_rows(paths: list[str]) -> tuple[dict[str, list[dict]], list[dict]]:
    """Rows grouped by shape (a later file's row replaces an earlier one at the same
    concurrency) and the descriptions the files carry."""
    by_shape: dict[str, dict[int, dict]] = {}
    meta = []
    for p in paths:
        d = json.loads(Path(p).read_text())
        rows = d.get("rows", []) if isinstance(d, dict) else d
        if isinstance(d, dict):
            meta.append({"file": Path(p).name, **{k: d[k] for k in ("description", "hardware") if k in d}})
        for r in rows:
            by_shape.setdefault(r.get("shape", "?"), {})[int(r["concurrency"])] = r
    return {s: [v[c] for c in sorted(v)] for s, v in by_shape.items()}, meta


def _f(x, fmt: str = "{:,.1f}", missing: str = "n/a") -> str:
    return missing if x is None else fmt.format(x)


def _ok(r: dict) -> bool:
    return r.get("completed", 0) > 0 and r.get("output_throughput_tok_s") is not None


def summary_row(shape: str, rows: list[dict]) -> dict:
    good = [r for r in rows if _ok(r)]
    if not good:
        return {"shape": shape, "peak": None, "reason": "no completed point"}
    peak = max(good, key=lambda r: r["output_throughput_tok_s"])
    top = max(good, key=lambda r: r["concurrency"])
    return {"shape": shape, "peak": peak["output_throughput_tok_s"], "peak_conc": peak["concurrency"],
            "req_s": peak.get("requests_per_s"), "top_conc": top["concurrency"],
            "ttft_s": None if top.get("ttft_mean_ms") is None else top["ttft_mean_ms"] / 1e3,
            "tpot_ms": top.get("tpot_mean_ms")}


def render(by_shape: dict[str, list[dict]], meta: list[dict], title: str, concurrencies: list[int] | None = None,
           reference: dict | None = REFERENCE_V4) -> str:
    order = [s for s in SHAPE_LABELS if s in by_shape] + sorted(s for s in by_shape if s not in SHAPE_LABELS)
    out = [f"# {title}", ""]
    for m in meta:
        if m.get("description"):
            out += [f"- `{m['file']}`: {m['description']}"]
        hw = m.get("hardware")
        if isinstance(hw, dict):
            out += ["  - hardware: " + ", ".join(f"{k} {v}" for k, v in hw.items())]
    if meta:
        out.append("")
    out += ["## Summary", "", "| Pattern | Peak output tok/s | @ conc | Req/s | TTFT mean @ top conc | TPOT @ top conc |",
            "|---|---:|---:|---:|---:|---:|"]
    sums = {}
    for s in order:
        sr = summary_row(s, by_shape[s])
        sums[s] = sr
        label = SHAPE_LABELS.get(s, s)
        if sr["peak"] is None:
            out.append(f"| `{label}` | {sr['reason']} | | | | |")
            continue
        out.append(f"| `{label}` | **{_f(sr['peak'], '{:,.2f}')}** | {sr['peak_conc']} | {_f(sr['req_s'], '{:.2f}')} | "
                   f"{_f(sr['ttft_s'], '{:.2f} s')} (C={sr['top_conc']}) | {_f(sr['tpot_ms'], '{:.2f} ms')} |")
    if reference:
        out += ["", f"## Beside the published reference ({reference['name']})", "",
                "| Pattern | This build, peak tok/s | Reference, peak tok/s | Ratio | This build, TPOT @ top conc | "
                "Reference, TPOT @ 512 |", "|---|---:|---:|---:|---:|---:|"]
        for s in order:
            ref = reference.get(s)
            sr = sums[s]
            if ref is None:
                continue
            if sr["peak"] is None:
                out.append(f"| `{s}` | {sr['reason']} | {ref['peak']:,.2f} | n/a | n/a | {ref['tpot_ms']:.2f} ms |")
                continue
            out.append(f"| `{s}` | {sr['peak']:,.2f} | {ref['peak']:,.2f} | {sr['peak'] / ref['peak']:.2f}x | "
                       f"{_f(sr['tpot_ms'], '{:.2f} ms')} | {ref['tpot_ms']:.2f} ms |")
    for s in order:
        rows = {r["concurrency"]: r for r in by_shape[s]}
        cs = sorted(set(concurrencies or []) | set(rows))
        out += ["", f"## {SHAPE_LABELS.get(s, s)}", "",
                "| Conc | Output tok/s | tok/s per GPU | Req/s | TTFT mean | TTFT p50 | TTFT p90 | TPOT mean | OK / failed |",
                "|---:|---:|---:|---:|---:|---:|---:|---:|---:|"]
        for c in cs:
            r = rows.get(c)
            if r is None:
                out.append(f"| {c} | not measured | | | | | | | |")
                continue
            if not _ok(r):
                why = r.get("first_error") or "no request completed"
                out.append(f"| {c} | failed: {why} | | | | | | | {r.get('completed', 0)} / {r.get('failed', 0)} |")
                continue
            ms = lambda k: _f(r.get(k), "{:,.0f} ms")  # noqa: E731
            out.append(f"| {c} | {_f(r['output_throughput_tok_s'], '{:,.2f}')} | "
                       f"{_f(r.get('output_tok_s_per_chip'), '{:,.2f}')} | {_f(r.get('requests_per_s'), '{:.3f}')} | "
                       f"{ms('ttft_mean_ms')} | {ms('ttft_p50_ms')} | {ms('ttft_p90_ms')} | "
                       f"{_f(r.get('tpot_mean_ms'), '{:.2f} ms')} | {r.get('completed', 0)} / {r.get('failed', 0)} |")
    out.append("")
    return "\n".join(out)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("files", nargs="+", help="sweep row files (bench/sweep.py --out)")
    ap.add_argument("--title", default="DeepSeek-V4-Flash on B200: served concurrency sweep")
    ap.add_argument("--concurrency", type=int, nargs="*", default=None,
                    help="concurrencies every table lists (missing ones are marked, not interpolated)")
    ap.add_argument("--no-reference", action="store_true")
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    by_shape, meta = load_rows(a.files)
    md = render(by_shape, meta, a.title, a.concurrency, None if a.no_reference else REFERENCE_V4)
    if a.out:
        Path(a.out).write_text(md)
    else:
        print(md)


if __name__ == "__main__":
    main()
