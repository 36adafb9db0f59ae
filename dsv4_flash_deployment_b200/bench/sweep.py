"""Concurrency sweep client against a running OpenAI-compatible server.

Produces one row per concurrency with the reference sweep's schema
(``kernel-optimizations-recipe/scripts/benchmark_sweep.py:135-165`` and
``results/raw/1k1k.json``): output tok/s = sum of streamed tokens / wall,
TTFT = time to the first non-empty streamed chunk, TPOT = mean over requests
of (e2e - TTFT) / (n - 1), plus the request rate, success rate and first
error.  Rows are written as soon as each point completes.

Prompts: ``ids`` (default) sends ISL uniform-random token ids per request
(the benchmark definition: "1024 uniform-random prompt tokens"); ``words``
builds deterministic word prompts and calibrates their length through
``/tokenize`` so the longest prompt fits the ISL, as the reference client
does for real tokenizers.

    python -m dsv4_flash_deployment_b200.bench.sweep --shape 1k1k --out 1k1k.json \
        --concurrency 1 4 16 64 128 256 512 --n-gpus 8
"""

from __future__ import annotations

import argparse
import asyncio
import json
import random
import statistics
import time

import aiohttp

SHAPES = {
    "1k1k": {"isl": 1024, "osl": 1024, "min_reqs": 4, "label": "1k/1k (balanced)"},
    "8k1k": {"isl": 8192, "osl": 1024, "min_reqs": 4, "label": "8k/1k (prefill-heavy)"},
    "1k8k": {"isl": 1024, "osl": 8192, "min_reqs": 1, "label": "1k/8k (reasoning)"},
}
DEFAULT_CONCURRENCIES = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512]
_WORDS = "amber birch cedar dune ember fjord grove heath iris juniper kestrel lagoon maple nectar orchid pine".split()


def word_prompt(seed: int, n_words: int) -> str:
    rng = random.Random(seed)
    return " ".join(rng.choice(_WORDS) for _ in range(n_words))


def id_prompt(seed: int, isl: int, vocab: int) -> list[int]:
    rng = random.Random(1_000_003 * seed + 17)
    return [rng.randrange(16, vocab) for _ in range(isl)]


async def _count(s, base, model, prompt) -> int:
    async with s.post(f"{base}/tokenize", json={"model": model, "prompt": prompt}) as r:
        r.raise_for_status()
        return (await r.json())["count"]


async def calibrate_words(s, base, model, n_prompts: int, isl: int) -> tuple[int, int, int]:
    lo, hi = 1, isl
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if await _count(s, base, model, word_prompt(0, mid)) <= isl:
            lo = mid
        else:
            hi = mid - 1
    n = lo
    while True:
        counts = await asyncio.gather(*(_count(s, base, model, word_prompt(i, n)) for i in range(n_prompts)))
        if max(counts) <= isl or n <= 1:
            return n, min(counts), max(counts)
        n -= 1


async def one_request(s, base, model, prompt, max_tokens: int) -> dict:
    t0 = time.perf_counter()
    ttft, ntok, usage_tok = None, 0, None
    # the usage chunk counts tokens even where a tokenizer holds a piece back (a
    # character split over tokens), as the reference's client does (recipes/benchmark.py:50,104)
    body = {"model": model, "prompt": prompt, "max_tokens": max_tokens, "temperature": 0.0, "stream": True,
            "ignore_eos": True, "stream_options": {"include_usage": True}}
    async with s.post(f"{base}/v1/completions", json=body) as r:
        if r.status != 200:
            raise RuntimeError(f"HTTP {r.status}: {(await r.text())[:300]}")
        async for raw in r.content:
            line = raw.decode().strip()
            if not line.startswith("data: "):
                continue
            data = line[6:]
            if data == "[DONE]":
                break
            ev = json.loads(data)
            if "error" in ev:
                raise RuntimeError(f"stream error: {ev['error']}")
            if ev.get("usage"):
                usage_tok = ev["usage"].get("completion_tokens", usage_tok)
            if ev["choices"] and ev["choices"][0].get("text"):
                if ttft is None:
                    ttft = time.perf_counter() - t0
                ntok += 1
    return {"ttft_s": ttft, "total_s": time.perf_counter() - t0, "ntok": usage_tok if usage_tok is not None else ntok}


async def run_point(base, model, prompts, concurrency: int, max_tokens: int, timeout_s: float):
    sem = asyncio.Semaphore(concurrency)
    conn = aiohttp.TCPConnector(limit=concurrency + 8)

    async with aiohttp.ClientSession(connector=conn, timeout=aiohttp.ClientTimeout(total=timeout_s)) as s:
        async def guarded(p):
            async with sem:
                return await one_request(s, base, model, p, max_tokens)
        t0 = time.perf_counter()
        res = await asyncio.gather(*(guarded(p) for p in prompts), return_exceptions=True)
        return res, time.perf_counter() - t0


def summarize(res, wall: float, concurrency: int, n_gpus: int) -> dict:
    ok = [r for r in res if isinstance(r, dict)]
    err = [r for r in res if not isinstance(r, dict)]
    ntok = sum(r["ntok"] for r in ok)
    ttft = sorted(r["ttft_s"] * 1e3 for r in ok if r["ttft_s"] is not None)
    tpot = [(r["total_s"] - (r["ttft_s"] or 0.0)) / max(r["ntok"] - 1, 1) * 1e3 for r in ok if r["ntok"] > 1]

    def pct(xs, q):
        return xs[min(int(q * len(xs)), len(xs) - 1)] if xs else None

    return {"concurrency": concurrency, "num_prompts": len(res), "completed": len(ok), "failed": len(err),
            "success_rate_pct": 100.0 * len(ok) / len(res) if res else 0.0,
            "first_error": f"{type(err[0]).__name__}: {err[0]}" if err else None,
            "wall_time_s": wall, "output_tokens": ntok, "output_throughput_tok_s": ntok / wall,
            "output_tok_s_per_chip": ntok / wall / n_gpus, "requests_per_s": len(ok) / wall,
            "ttft_mean_ms": statistics.mean(ttft) if ttft else None, "ttft_p50_ms": pct(ttft, 0.5),
            "ttft_p90_ms": pct(ttft, 0.9), "tpot_mean_ms": statistics.mean(tpot) if tpot else None}


async def sweep(base: str, model: str, shape: dict, shape_key: str, concurrencies: list[int], out_path: str | None,
                n_gpus: int, prompt_mode: str = "ids", vocab: int = 129280, max_model_len: int | None = None,
                timeout_s: float = 14400.0) -> list[dict]:
    isl, osl, min_reqs = shape["isl"], shape["osl"], shape["min_reqs"]
    n_prompts = max(max(concurrencies), min_reqs)
    if prompt_mode == "words":
        async with aiohttp.ClientSession() as s:
            n_words, isl_min, isl_max = await calibrate_words(s, base, model, n_prompts, isl)
        prompts = [word_prompt(i, n_words) for i in range(n_prompts)]
    else:
        n_words, isl_min, isl_max = 0, isl, isl
        prompts = [id_prompt(i, isl, vocab) for i in range(n_prompts)]
    if max_model_len is not None and isl_max + osl > max_model_len:
        raise SystemExit(f"shape does not fit: isl {isl_max} + osl {osl} > {max_model_len}")
    rows = []
    for c in concurrencies:
        n = max(c, min_reqs)
        t_start = time.time()
        res, wall = await run_point(base, model, prompts[:n], c, osl, timeout_s)
        row = summarize(res, wall, c, n_gpus)
        row.update(shape=shape_key, label=shape["label"], isl_min=isl_min, isl_max=isl_max, osl=osl,
                   n_words=n_words, requests_issued=n, started_at=t_start, prompt_mode=prompt_mode)
        rows.append(row)
        tp = row["tpot_mean_ms"]
        print(f"C={c:4d} n={n:4d} {row['output_throughput_tok_s']:10.1f} tok/s  {row['completed']}/{n} ok  "
              f"ttft {row['ttft_mean_ms'] or 0:.0f} ms  tpot {tp if tp is not None else float('nan'):.2f} ms "
              f"[{wall:.1f}s]", flush=True)
        if out_path:
            with open(out_path, "w") as f:
                json.dump(rows, f, indent=1)
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--base", default="http://127.0.0.1:8000")
    ap.add_argument("--model", default="deepseek-v4-flash")
    ap.add_argument("--shape", default="1k1k", choices=sorted(SHAPES))
    ap.add_argument("--isl", type=int, default=None)
    ap.add_argument("--osl", type=int, default=None)
    ap.add_argument("--out", default=None)
    ap.add_argument("--concurrency", type=int, nargs="*", default=None)
    ap.add_argument("--n-gpus", type=int, default=8)
    ap.add_argument("--prompt-mode", choices=["ids", "words"], default="ids")
    ap.add_argument("--vocab", type=int, default=129280)
    ap.add_argument("--max-model-len", type=int, default=None)
    a = ap.parse_args(argv)
    shape = dict(SHAPES[a.shape])
    if a.isl:
        shape["isl"] = a.isl
    if a.osl:
        shape["osl"] = a.osl
    asyncio.run(sweep(a.base, a.model, shape, a.shape, a.concurrency or DEFAULT_CONCURRENCIES, a.out, a.n_gpus,
                      a.prompt_mode, a.vocab, a.max_model_len))


if __name__ == "__main__":
    main()
