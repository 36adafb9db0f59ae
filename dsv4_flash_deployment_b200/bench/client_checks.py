"""Client-side serving checks against a live server (the reference's
``kernel-optimizations-recipe/scripts/smoke.py`` and ``greedy_determinism.py``).

  smoke        /health, /v1/models, one completion and one chat completion
  determinism  N prompts at temperature 0, sent twice concurrently; every
               output must be identical (continuous batching must not change
               a request's greedy tokens)

    python -m dsv4_flash_deployment_b200.bench.client_checks smoke --base http://127.0.0.1:8000
    python -m dsv4_flash_deployment_b200.bench.client_checks determinism --n 200 --max-tokens 32
"""

from __future__ import annotations

import argparse
import asyncio
import json

import aiohttp

from .sweep import word_prompt


async def smoke(base: str, model: str) -> dict:
    async with aiohttp.ClientSession() as s:
        h = await (await s.get(f"{base}/health")).json()
        m = await (await s.get(f"{base}/v1/models")).json()
        c = await (await s.post(f"{base}/v1/completions", json={
            "model": model, "prompt": "The capital of France is", "max_tokens": 8, "temperature": 0})).json()
        ch = await (await s.post(f"{base}/v1/chat/completions", json={
            "model": model, "messages": [{"role": "user", "content": "Say hi."}], "max_tokens": 8})).json()
    ok = (h.get("status") == "ok" and m["data"] and c["choices"][0]["finish_reason"] in ("length", "stop")
          and ch["choices"][0]["message"]["role"] == "assistant")
    return {"ok": bool(ok), "health": h.get("status"), "model": m["data"][0]["id"],
            "completion": c["choices"][0]["text"], "chat": ch["choices"][0]["message"]["content"]}


async def determinism(base: str, model: str, n: int, max_tokens: int, concurrency: int,
                      max_words: int = 48) -> dict:
    prompts = [word_prompt(1000 + i, 4 + (i * 7) % max_words) for i in range(n)]
    sem = asyncio.Semaphore(concurrency)

    async def one(s, p):
        async with sem:
            async with s.post(f"{base}/v1/completions", json={"model": model, "prompt": p, "max_tokens": max_tokens,
                                                              "temperature": 0, "ignore_eos": True}) as r:
                body = await r.json()
                if r.status != 200:
                    raise RuntimeError(f"HTTP {r.status}: {body}")
                return body["choices"][0]["text"]

    async with aiohttp.ClientSession() as s:
        a = await asyncio.gather(*(one(s, p) for p in prompts))
        b = await asyncio.gather(*(one(s, p) for p in reversed(prompts)))
    b = list(reversed(b))
    diff = [i for i in range(n) if a[i] != b[i]]
    return {"ok": not diff, "n": n, "mismatches": len(diff), "first_mismatch": diff[0] if diff else None}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("check", choices=["smoke", "determinism"])
    ap.add_argument("--base", default="http://127.0.0.1:8000")
    ap.add_argument("--model", default="deepseek-v4-flash")
    ap.add_argument("--n", type=int, default=200)
    ap.add_argument("--max-tokens", type=int, default=32)
    ap.add_argument("--concurrency", type=int, default=64)
    ap.add_argument("--max-words", type=int, default=48)
    a = ap.parse_args(argv)
    if a.check == "smoke":
        r = asyncio.run(smoke(a.base, a.model))
    else:
        r = asyncio.run(determinism(a.base, a.model, a.n, a.max_tokens, a.concurrency, a.max_words))
    print(json.dumps(r))
    raise SystemExit(0 if r["ok"] else 1)


if __name__ == "__main__":
    main()
