"""Golden token files: greedy continuations from the CPU oracle, saved once and
compared with the model step later, teacher-forced and tie-aware.

``make_golden`` runs the oracle (``ref/model.py``) on each prompt for ``steps``
greedy tokens and records, per generated position, the chosen token, its
log-probability and the gap between the two largest logits.  ``compare`` feeds
each golden sequence (prompt + golden tokens) to the model under test
(:func:`.parity.device_logits`, one prefill chunk then one token per step) and
counts, per position, whether its argmax is the golden token: strict top-1,
and tie-aware top-1 where a position whose golden top-2 gap is within one bf16
ULP of the logit counts as agreeing either way (bf16 activations cannot order
such a pair reliably).  The reference generates its goldens the same way, on
CPU from its upstream model (``tpu-v7x/deepseek_v41/golden/make_golden.py``:
8 prompts x 128 steps), and its checks report strict and tie-aware top-1
(``megakernel-recipe/scripts/verify_reference_engine.py``).

    python -m dsv4_flash_deployment_b200.verify.golden make --model v4-check --out golden_v4.json
    python -m dsv4_flash_deployment_b200.verify.golden check golden_v4.json
"""

from __future__ import annotations

import argparse
import json
import math

import torch

GOLDEN_VERSION = 1


def bf16_ulp(x: float) -> float:
    """Spacing of bf16 values near ``x`` (8 bits of mantissa)."""
    if x == 0 or not math.isfinite(x):
        return 2.0 ** -133
    return 2.0 ** (math.floor(math.log2(abs(x))) - 7)


def make_golden(cfg, weights: dict, prompts: list[list[int]], steps: int, max_len: int, meta: dict | None = None) -> dict:
    from ..ref.model import RefModel

    ref = RefModel(cfg, weights, max_seq_len=max_len)
    seqs = []
    for p in prompts:
        st = ref.new_state(1)
        logits = None
        for t in p:
            logits, _ = ref.step(torch.tensor([t]), st)
        toks, lps, gaps = [], [], []
        for _ in range(steps):
            lg = logits[0, : cfg.vocab_size].float()
            top2 = torch.topk(lg, 2)
            tok = int(top2.indices[0])
            toks.append(tok)
            lps.append(float(torch.log_softmax(lg, -1)[tok]))
            gaps.append(float(top2.values[0] - top2.values[1]))
            logits, _ = ref.step(torch.tensor([tok]), st)
        seqs.append({"prompt": list(p), "tokens": toks, "logprobs": lps, "top2_gap": gaps})
    return {"version": GOLDEN_VERSION, "model": cfg.name, "steps": steps, "max_len": max_len,
            **(meta or {}), "sequences": seqs}


def compare(golden: dict, cfg, weights: dict, device: str) -> dict:
    """Teacher-forced top-1 agreement of the model under test with the golden tokens."""
    from .parity import device_logits

    seqs = [g["prompt"] + g["tokens"] for g in golden["sequences"]]
    plen = [len(g["prompt"]) for g in golden["sequences"]]
    # the prediction of golden token i comes from position len(prompt) - 1 + i
    got = device_logits(cfg, weights, [s[:-1] for s in seqs], plen, golden["max_len"], None, device)
    strict = tie = total = 0
    worst_gap_flip = 0.0
    per_seq = []
    for g, lg, n0 in zip(golden["sequences"], got, plen):
        s_ok = 0
        for i, (tok, gap) in enumerate(zip(g["tokens"], g["top2_gap"])):
            row = lg[n0 - 1 + i]
            pred = int(row.argmax())
            ok = pred == tok
            near_tie = gap <= bf16_ulp(float(row.max()))
            strict += ok
            tie += ok or near_tie
            total += 1
            s_ok += ok
            if not ok:
                worst_gap_flip = max(worst_gap_flip, gap)
        per_seq.append(s_ok / len(g["tokens"]))
    return {"positions": total, "strict_top1": strict / total, "tie_aware_top1": tie / total,
            "largest_golden_gap_flipped": worst_gap_flip, "per_sequence_strict": per_seq}


def main(argv=None) -> int:
    from ..config import get_config
    from ..io.checkpoint_spec import make_random_weights

    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    mk = sub.add_parser("make")
    mk.add_argument("--model", default="v4-check")
    mk.add_argument("--seed", type=int, default=3)
    mk.add_argument("--prompts", type=int, default=8)
    mk.add_argument("--prompt-len", type=int, default=24)
    mk.add_argument("--steps", type=int, default=32)
    mk.add_argument("--out", required=True)
    ck = sub.add_parser("check")
    ck.add_argument("golden")
    ck.add_argument("--device", default=None)
    # random-init logits are nearly flat and upstream near-ties (indexer picks) can flip a
    # pick by more than one bf16 ULP: the default bar is the GPU parity tests' top-1 bar
    ck.add_argument("--min-tie-aware", type=float, default=0.8)
    a = ap.parse_args(argv)
    if a.cmd == "make":
        cfg = get_config(a.model)
        g = torch.Generator().manual_seed(a.seed + 11)
        prompts = [torch.randint(0, cfg.vocab_size, (a.prompt_len,), generator=g).tolist() for _ in range(a.prompts)]
        w = make_random_weights(cfg, seed=a.seed)
        gold = make_golden(cfg, w, prompts, a.steps, a.prompt_len + a.steps + 8,
                           {"seed": a.seed, "weights": "random init (io.checkpoint_spec.make_random_weights)"})
        with open(a.out, "w") as f:
            json.dump(gold, f)
        print(json.dumps({"out": a.out, "sequences": len(prompts), "steps": a.steps}))
        return 0
    with open(a.golden) as f:
        gold = json.load(f)
    cfg = get_config(gold["model"])
    w = make_random_weights(cfg, seed=gold["seed"])
    dev = a.device or ("cuda" if torch.cuda.is_available() else "cpu")
    r = compare(gold, cfg, w, dev)
    r["passed"] = r["tie_aware_top1"] >= a.min_tie_aware
    print(json.dumps(r))
    return 0 if r["passed"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
