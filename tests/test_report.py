"""Sweep report renderer: summary (peak and the concurrency it came at), the
reference comparison, per-concurrency tables, and missing / failed points shown
with their reason rather than blank or interpolated."""

import json

from dsv4_flash_deployment_b200.bench import report


def _row(c, tok_s, shape="1k1k", completed=None, failed=0, err=None):
    return {"concurrency": c, "shape": shape, "output_throughput_tok_s": tok_s, "output_tok_s_per_chip": tok_s / 8,
            "requests_per_s": c / 100, "ttft_mean_ms": 100.0 * c, "ttft_p50_ms": 90.0 * c, "ttft_p90_ms": 150.0 * c,
            "tpot_mean_ms": 10 + c / 10, "completed": c if completed is None else completed, "failed": failed,
            "first_error": err}


def test_render_summary_reference_and_gaps(tmp_path):
    a = tmp_path / "a.json"
    b = tmp_path / "b.json"
    a.write_text(json.dumps({"description": "run a", "hardware": {"gpu": "B200"},
                             "rows": [_row(1, 90.0), _row(64, 3000.0), _row(512, 9000.0)]}))
    b.write_text(json.dumps([_row(512, 9100.0), _row(128, 0.0, completed=0, failed=128, err="TimeoutError: x"),
                             _row(512, 1200.0, shape="8k1k")]))
    by_shape, meta = report.load_rows([str(a), str(b)])
    assert [r["concurrency"] for r in by_shape["1k1k"]] == [1, 64, 128, 512]
    assert by_shape["1k1k"][-1]["output_throughput_tok_s"] == 9100.0          # the later file wins
    md = report.render(by_shape, meta, "T", concurrencies=[1, 16, 64, 128, 512])
    assert "| `1k/1k (balanced)` | **9,100.00** | 512 |" in md
    assert "| 16 | not measured |" in md
    assert "| 128 | failed: TimeoutError: x |" in md
    assert "| `1k1k` | 9,100.00 | 8,463.70 | 1.08x |" in md
    assert "| `8k1k` | 1,200.00 | 1,758.53 | 0.68x |" in md
    assert "run a" in md and "gpu B200" in md
    out = tmp_path / "r.md"
    report.main([str(a), "--out", str(out), "--no-reference"])
    assert "Beside the published reference" not in out.read_text()
