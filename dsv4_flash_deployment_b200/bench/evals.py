"""Accuracy evaluation clients against a live server.

Plays the role of the reference's evaluation clients: GPQA-Diamond through the
simple-evals multiple-choice template (``kernel-optimizations-recipe/scripts/
gpqa_diamond.py``; ``deepseek_v41/runner.py`` ``run_gpqa_diamond_stage`` with
its partial-file resume) and GSM8K (``run_gsm8k_stage``).  There is no network
on the serving hosts, so datasets are local JSONL files:

  mc    {"question": str, "choices": [str, ...], "answer": "B" | 1}
        (answer = letter or 0-based index of the correct choice; choices are
        shuffled per question with a seeded RNG, as simple-evals does)
  math  {"question": str, "answer": "42" | "... #### 42"}

Every item is one chat completion.  The reply's final answer is extracted
(the last "Answer: X" letter for mc, the last number for math) and scored.
Each finished item is appended to the partial file at once, so an interrupted
run resumes where it stopped; the summary has pass@1 and a verdict block.

    python -m dsv4_flash_deployment_b200.bench.evals mc --data gpqa_diamond.jsonl --partial gpqa.partial.jsonl
    python -m dsv4_flash_deployment_b200.bench.evals math --data gsm8k_test.jsonl --max-tokens 1024
"""

from __future__ import annotations

import argparse
import asyncio
import json
import os
import random
import re
import time

import aiohttp

LETTERS = "ABCDEFGHIJ"
MC_TEMPLATE = ("Answer the following multiple choice question. The last line of your response should be of "
               "the following format: 'Answer: $LETTER' (without quotes) where LETTER is one of {letters}. "
               "Think step by step before answering.\n\n{question}\n\n{options}")
MATH_TEMPLATE = ("Solve the following math problem step by step. The last line of your response should be "
                 "the final numeric answer.\n\n{question}")
_ANSWER_RE = re.compile(r"(?i)answer\s*[:：]\s*\**\s*\(?([A-J])\)?")
_NUM_RE = re.compile(r"-?\d[\d,]*(?:\.\d+)?")


def load_items(path: str) -> list[dict]:
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


def mc_prompt(item: dict, idx: int, seed: int, template: str = MC_TEMPLATE) -> tuple[str, str]:
    """(prompt, correct letter) with the choices shuffled by (seed, idx)."""
    choices = list(item["choices"])
    ans = item["answer"]
    correct = choices[LETTERS.index(ans.strip().upper()) if isinstance(ans, str) else int(ans)]
    order = list(range(len(choices)))
    random.Random(seed * 1_000_003 + idx).shuffle(order)
    shuffled = [choices[i] for i in order]
    letters = LETTERS[:len(shuffled)]
    options = "\n".join(f"{letters[i]}) {c}" for i, c in enumerate(shuffled))
    prompt = template.format(letters=", ".join(letters), question=item["question"], options=options)
    return prompt, letters[shuffled.index(correct)]


def extract_letter(text: str) -> str | None:
    m = _ANSWER_RE.findall(text or "")
    return m[-1].upper() if m else None


def _number(s: str) -> float | None:
    m = _NUM_RE.findall(s or "")
    if not m:
        return None
    try:
        return float(m[-1].replace(",", ""))
    except ValueError:
        return None


def math_target(item: dict) -> float | None:
    a = str(item["answer"])
    return _number(a.split("####")[-1])


def read_partial(path: str | None) -> dict[int, dict]:
    done: dict[int, dict] = {}
    if path and os.path.exists(path):
        with open(path) as f:
            for line in f:
                if line.strip():
                    r = json.loads(line)
                    done[int(r["idx"])] = r
    return done


async def run_eval(kind: str, base: str, model: str, items: list[dict], max_tokens: int, temperature: float,
                   concurrency: int, partial: str | None = None, seed: int = 0, limit: int | None = None,
                   template: str | None = None) -> dict:
    """Scores ``items`` (``kind`` "mc" or "math"); resumes from ``partial``.  ``template``
    replaces the prompt template (fields {letters}/{question}/{options}, or {question})."""
    if kind not in ("mc", "math"):
        raise ValueError(kind)
    items = items[:limit] if limit else items
    done = read_partial(partial)
    todo = [i for i in range(len(items)) if i not in done]
    sem = asyncio.Semaphore(max(1, concurrency))
    pf = open(partial, "a") if partial else None
    t0 = time.perf_counter()

    async def one(s, i):
        if kind == "mc":
            prompt, target = mc_prompt(items[i], i, seed, template or MC_TEMPLATE)
        else:
            prompt, target = (template or MATH_TEMPLATE).format(question=items[i]["question"]), math_target(items[i])
        async with sem:
            r = await s.post(f"{base}/v1/chat/completions", json={
                "model": model, "messages": [{"role": "user", "content": prompt}],
                "max_tokens": max_tokens, "temperature": temperature})
            body = await r.json()
        if r.status != 200:
            rec = {"idx": i, "error": body.get("error", {}).get("message", str(body)), "correct": False}
        else:
            text = body["choices"][0]["message"]["content"]
            got = extract_letter(text) if kind == "mc" else _number(text)
            ok = got is not None and target is not None and (
                got == target if kind == "mc" else abs(got - target) < 1e-6)
            rec = {"idx": i, "target": target, "extracted": got, "correct": bool(ok),
                   "finish_reason": body["choices"][0].get("finish_reason"),
                   "completion_tokens": body.get("usage", {}).get("completion_tokens")}
        if pf is not None:
            pf.write(json.dumps(rec) + "\n")
            pf.flush()
        done[i] = rec
        return rec

    try:
        async with aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=None)) as s:
            await asyncio.gather(*(one(s, i) for i in todo))
    finally:
        if pf is not None:
            pf.close()
    recs = [done[i] for i in sorted(done) if i < len(items)]
    n = len(recs)
    correct = sum(r["correct"] for r in recs)
    errors = sum(1 for r in recs if "error" in r)
    unparsed = sum(1 for r in recs if "error" not in r and r.get("extracted") is None)
    acc = correct / n if n else 0.0
    return {"kind": kind, "n": n, "correct": correct, "pass@1": round(acc, 4), "errors": errors,
            "unparsed": unparsed, "resumed": len(items) - len(todo), "wall_time_s": round(time.perf_counter() - t0, 2),
            "verdict": {"complete": n == len(items), "ok": errors == 0 and n == len(items),
                        "max_tokens": max_tokens, "temperature": temperature, "seed": seed}}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("kind", choices=["mc", "math"])
    ap.add_argument("--data", required=True, help="local JSONL file")
    ap.add_argument("--base", default="http://127.0.0.1:8000")
    ap.add_argument("--model", default="deepseek-v4-flash")
    ap.add_argument("--max-tokens", type=int, default=14336)
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--concurrency", type=int, default=64)
    ap.add_argument("--partial", default=None, help="append-only results file; an existing one is resumed")
    ap.add_argument("--seed", type=int, default=0, help="choice shuffling seed (mc)")
    ap.add_argument("--limit", type=int, default=None)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    r = asyncio.run(run_eval(a.kind, a.base, a.model, load_items(a.data), a.max_tokens, a.temperature,
                             a.concurrency, a.partial, a.seed, a.limit))
    line = json.dumps(r)
    print(line)
    if a.out:
        with open(a.out, "w") as f:
            f.write(line + "\n")
    raise SystemExit(0 if r["verdict"]["ok"] else 1)


if __name__ == "__main__":
    main()
