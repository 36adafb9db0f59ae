"""Resumable model-level verification runner.

Runs named stages in order and writes one ``<stage>.json`` per stage into the
output directory, stamped with the hardware / software provenance, the stage's
configuration, its measurements, its pass rule and ``passed``.  A stage whose
file already records a pass is skipped on the next run (``--force`` reruns
it), so an interrupted run resumes where it stopped; ``summary.json`` lists
every stage's state.  The reference's stage runner works the same way
(``tpu-v7x/deepseek_v41/runner.py``: ``ALL_STAGES`` ``:43-55``,
``stage_already_passed`` ``:130-156``, ``write_stage_result`` ``:158``, stage
bodies ``:293-694``); its rank 0 decides which stages to run and broadcasts
that to the other hosts, while here multi-GPU checks run as their own
``torchrun`` jobs (the ``tp_parity`` / ``ep_parity`` stages) and the runner
itself is one process.

Stages:

  cold_startup        build the engine (checkpoint, or random init on the device);
                      pass: build time <= --max-startup-s (900 s, the reference's bound)
  parity_ref          teacher-forced logits of the model step against the CPU oracle;
                      pass: mean cosine >= 0.995, worst >= 0.97, top-1 >= 0.8
  parity_neg_control  the same with the mHC Sinkhorn iterations set to 0, which must
                      break parity; pass: mean cosine < 0.99
  golden              teacher-forced greedy tokens against a golden file (--golden; made by
                      verify/golden.py from the oracle, or made here when none is given);
                      pass: tie-aware top-1 >= --min-tie-aware (0.8)
  perf_b{1,2,4,8}     decode TPOT with B sequences at --ctx tokens of context through
                      the serving engine (CUDA-graph replay, H2D + D2H each step)
  dspark_verify       DSpark 1+4 speculative decoding against greedy decoding
                      (configs with MTP stages); pass: >= 90 % of tokens identical
  tp_parity/ep_parity the tensor- / expert-parallel self-checks on --gpus GPUs
                      (parallel/tp_check.py, parallel/ep_check.py under torchrun)
  gsm8k/gpqa_diamond  accuracy through a running server (--server, --gsm8k-data /
                      --gpqa-data), resumable from a partial file in the output dir

Random-init logits are nearly flat, so near-tied positions can flip top-1
between two correct implementations: the parity bar is the one the GPU tests
use (``tests/test_model_gpu.py``); each record also states whether the
reference's synthetic-weights bar (top-1 >= 0.99 and cosine >= 0.995) was met.
With ``--device cpu`` the oracle stands in for the model (plumbing check).

    python -m dsv4_flash_deployment_b200.verify.runner --out results/verify/v4-check
    python -m dsv4_flash_deployment_b200.verify.runner --model v4.1-check --stages dspark_verify
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
import traceback
from pathlib import Path

ALL_STAGES = ("cold_startup", "parity_ref", "parity_neg_control", "golden", "perf_b1", "perf_b2", "perf_b4",
              "perf_b8", "dspark_verify", "tp_parity", "ep_parity", "gsm8k", "gpqa_diamond")


# ------------------------------------------------------------------ result files
# named stage sets for --stages
PRESETS = {"all": ALL_STAGES, "quick": ("cold_startup", "parity_ref", "parity_neg_control", "golden"),
           "perf": ("perf_b1", "perf_b2", "perf_b4", "perf_b8")}


def stage_path(out: Path, stage: str) -> Path:
    return Path(out) / f"{stage}.json"


def read_stage(out: Path, stage: str) -> dict | None:
    p = stage_path(out, stage)
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text())
    except (OSError, json.JSONDecodeError):
        return None


def stage_already_passed(out: Path, stage: str) -> bool:
    rec = read_stage(out, stage)
    return bool(rec and rec.get("passed") and not rec.get("skipped"))


def write_stage_result(out: Path, stage: str, rec: dict) -> None:
    """Writes the record atomically (a reader never sees half a file)."""
    p = stage_path(out, stage)
    p.parent.mkdir(parents=True, exist_ok=True)
    tmp = p.with_suffix(".json.tmp")
    tmp.write_text(json.dumps(rec, indent=1, sort_keys=True) + "\n")
    os.replace(tmp, p)


def render_summary(out: Path, model: str, device: str) -> str:
    """A markdown table of every stage record in ``out``: state, rule and the key
    measurements (the numbers a reader checks first)."""
    keys = ("build_s", "cos_mean", "cos_min", "top1", "strict_top1", "tie_aware_top1", "tpot_ms_median",
            "decode_tok_s", "identical_fraction", "pass@1", "rc", "reason", "error")
    rows = [f"# Verification stages: {model} on {device}", "", "| stage | state | rule | measurements |",
            "|---|---|---|---|"]
    for st in ALL_STAGES:
        r = read_stage(out, st)
        if r is None:
            rows.append(f"| {st} | not run | | |")
            continue
        state = "skipped" if r.get("skipped") else ("passed" if r.get("passed") else "failed")
        meas = ", ".join(f"{k} {r[k]:.4g}" if isinstance(r[k], float) else f"{k} {r[k]}"
                         for k in keys if k in r and r[k] is not None)
        rows.append(f"| {st} | {state} | {r.get('rule', '')} | {meas[:300]} |")
    return "\n".join(rows) + "\n"


def skipped(reason: str) -> dict:
    return {"skipped": True, "passed": False, "reason": reason}


# ------------------------------------------------------------------ the runner
class Runner:
    def __init__(self, a: argparse.Namespace):
        from ..config import get_config

        self.a = a
        self.out = Path(a.out)
        self.cfg = get_config(a.model)
        self.device = a.device
        self._w = None

    def weights(self) -> dict:
        """Checkpoint weights (``--checkpoint``) or random ones drawn on the host from
        ``--seed`` (the oracle needs host tensors of every weight)."""
        if self._w is None:
            if self.a.checkpoint:
                from ..io.safetensors import load_checkpoint

                self._w = load_checkpoint(self.a.checkpoint, self.cfg)
            else:
                from ..io.checkpoint_spec import make_random_weights

                self._w = make_random_weights(self.cfg, seed=self.a.seed)
        return self._w

    def sequences(self, n: int, length: int, seed: int) -> list[list[int]]:
        import torch

        g = torch.Generator().manual_seed(seed)
        return [torch.randint(0, self.cfg.vocab_size, (length - 3 * i,), generator=g).tolist() for i in range(n)]

    def run(self) -> dict:
        from ..utils.provenance import provenance

        stages = (list(PRESETS[self.a.stages]) if self.a.stages in PRESETS
                  else [s.strip() for s in self.a.stages.split(",")])
        unknown = [s for s in stages if s not in ALL_STAGES]
        if unknown:
            raise SystemExit(f"unknown stages {unknown}; known: {list(ALL_STAGES)}")
        hw = provenance()
        summary = {}
        for st in stages:
            if not self.a.force and stage_already_passed(self.out, st):
                summary[st] = "passed (kept)"
                print(f"[verify] {st}: passed earlier, skipped", flush=True)
                continue
            t0 = time.time()
            try:
                rec = getattr(self, "stage_" + st)(st)
            except Exception as e:   # noqa: BLE001  (a failing stage is recorded, the next one runs)
                rec = {"passed": False, "error": f"{type(e).__name__}: {e}", "traceback": traceback.format_exc()[-4000:]}
            rec.update(stage=st, model=self.cfg.name, device=self.device, seed=self.a.seed,
                       wall_s=round(time.time() - t0, 2), hardware=hw, time=time.strftime("%Y-%m-%dT%H:%M:%S"))
            write_stage_result(self.out, st, rec)
            state = "skipped" if rec.get("skipped") else ("passed" if rec.get("passed") else "FAILED")
            summary[st] = state
            print(f"[verify] {st}: {state} ({rec['wall_s']} s)" + (f" {rec.get('error') or rec.get('reason')}"
                                                                     if state != "passed" else ""), flush=True)
            self._release()
        all_stages = {s: (read_stage(self.out, s) or {}) for s in ALL_STAGES}
        full = {s: ("not run" if not r else "skipped" if r.get("skipped") else
                    "passed" if r.get("passed") else "failed") for s, r in all_stages.items()}
        write_stage_result(self.out, "summary", {"this_run": summary, "stages": full, "model": self.cfg.name,
                                                 "device": self.device})
        (self.out / "summary.md").write_text(render_summary(self.out, self.cfg.name, self.device))
        return summary

    def _release(self) -> None:
        import gc

        gc.collect()
        if self.device == "cuda":
            import torch

            torch.cuda.synchronize()
            torch.cuda.empty_cache()

    # ------------------------------------------------------------- stages
    def stage_cold_startup(self, st: str) -> dict:
        import torch

        t0 = time.perf_counter()
        eng = self._engine(max_seqs=4, max_len=self.a.max_len)
        if self.device == "cuda":
            torch.cuda.synchronize()
        build_s = time.perf_counter() - t0
        rec = {"build_s": round(build_s, 3), "source": self.a.checkpoint or "random init",
               "rule": f"build_s <= {self.a.max_startup_s}", "passed": build_s <= self.a.max_startup_s}
        if self.device == "cuda":
            rec.update(device_allocated_gib=round(torch.cuda.memory_allocated() / 2 ** 30, 3),
                       device_reserved_gib=round(torch.cuda.memory_reserved() / 2 ** 30, 3))
        del eng
        return rec

    def _parity(self, sinkhorn_iters: int | None) -> dict:
        from .parity import compare, device_logits, oracle_logits

        seqs = self.sequences(self.a.n_seqs, self.a.seq_len, self.a.seed + 1)
        pre = [max(1, len(s) * 2 // 3 - 5 * i) for i, s in enumerate(seqs)]
        w = self.weights()
        got = device_logits(self.cfg, w, seqs, pre, self.a.max_len, sinkhorn_iters, self.device)
        ref = oracle_logits(self.cfg, w, seqs, self.a.max_len)
        r = compare(got, ref)
        r.update(sequences=len(seqs), seq_len=self.a.seq_len, prefill_lens=pre,
                 reference_bar_met=r["top1"] >= 0.99 and r["cos_mean"] >= 0.995)
        return r

    def stage_parity_ref(self, st: str) -> dict:
        r = self._parity(None)
        r["rule"] = "cos_mean >= 0.995 and cos_min >= 0.97 and top1 >= 0.8"
        r["passed"] = r["cos_mean"] >= 0.995 and r["cos_min"] >= 0.97 and r["top1"] >= 0.8
        return r

    def stage_parity_neg_control(self, st: str) -> dict:
        r = self._parity(0)
        r["rule"] = "sinkhorn_iters = 0 must break parity: cos_mean < 0.99"
        r["passed"] = r["cos_mean"] < 0.99
        r["reference_rule_top1_below_0.5"] = r["top1"] < 0.5
        return r

    def stage_golden(self, st: str) -> dict:
        from .golden import compare, make_golden

        if self.a.golden:
            with open(self.a.golden) as f:
                gold = json.load(f)
            if gold["model"] != self.cfg.name:
                return skipped(f"golden file is for {gold['model']}, the runner's model is {self.cfg.name}")
            src = self.a.golden
        else:
            prompts = self.sequences(4, 20, self.a.seed + 13)
            gold = make_golden(self.cfg, self.weights(), prompts, 16, self.a.max_len)
            src = "made by the oracle in this run"
        r = compare(gold, self.cfg, self.weights(), self.device)
        r.update(golden=src, rule=f"tie_aware_top1 >= {self.a.min_tie_aware}",
                 passed=r["tie_aware_top1"] >= self.a.min_tie_aware)
        return r

    def _perf(self, B: int) -> dict:
        import torch

        # every sequence keeps decoding through the timed steps: the first ones also
        # decode while later ones are still prefilling (at most one step per chunk)
        n_new = self.a.perf_warmup + self.a.perf_steps + 2 + -(-B * self.a.ctx // 64) + B
        eng = self._engine(max_seqs=B, max_len=self.a.ctx + n_new + 16)
        seqs = [[(17 * b + 31 * i) % self.cfg.vocab_size for i in range(self.a.ctx)] for b in range(B)]
        reqs = [eng.add_request(s, n_new, ignore_eos=True) for s in seqs]
        while not all(r.prompt_done and r.output for r in reqs):
            eng.step()
        for _ in range(self.a.perf_warmup):
            eng.step()
        if self.device == "cuda":
            torch.cuda.synchronize()
        times = []
        for _ in range(self.a.perf_steps):
            t0 = time.perf_counter()
            ev = eng.step()            # H2D metadata, replay, D2H of the sampled ids, host sync
            times.append(time.perf_counter() - t0)
            assert sum(t is not None for _, t in ev) == B
        times.sort()
        med = times[len(times) // 2]
        rec = {"batch": B, "context": self.a.ctx, "steps": len(times), "tpot_ms_median": round(med * 1e3, 3),
               "tpot_ms_mean": round(sum(times) / len(times) * 1e3, 3),
               "decode_tok_s": round(B / med, 1), "graph_captures": eng.stats.get("graph_captures", 0),
               "rule": "runs (measurement stage)", "passed": True}
        del eng
        return rec

    def stage_perf_b1(self, st): return self._perf(1)
    def stage_perf_b2(self, st): return self._perf(2)
    def stage_perf_b4(self, st): return self._perf(4)
    def stage_perf_b8(self, st): return self._perf(8)

    def stage_dspark_verify(self, st: str) -> dict:
        if self.cfg.n_mtp_layers < 1:
            return skipped(f"model {self.cfg.name} has no MTP stages (try --model v4.1-check)")
        if self.device != "cuda":
            return skipped("DSpark runs on the GPU only")
        import torch

        from ..engine.builder import build_model
        from ..engine.engine import Engine
        from ..spec.dspark import SpecEngine

        w = self.weights()
        prompts = self.sequences(2, 24, self.a.seed + 7)
        n = self.a.dspark_tokens
        base = Engine(build_model(self.cfg, "cuda", max_tokens=64, n_slots=3, max_seq_len=self.a.max_len,
                                  weights=w), 2, 64, self.a.max_len)
        t0 = time.perf_counter()
        want = base.generate(prompts, n, ignore_eos=True)
        torch.cuda.synchronize()
        t_base = time.perf_counter() - t0
        del base
        spec = SpecEngine(build_model(self.cfg, "cuda", max_tokens=64, n_slots=3, max_seq_len=self.a.max_len,
                                      weights=w), w, max_seqs=2)
        t0 = time.perf_counter()
        got = spec.generate(prompts, n)
        torch.cuda.synchronize()
        t_spec = time.perf_counter() - t0
        same = sum(int(a == b) for g, wv in zip(got, want) for a, b in zip(g, wv))
        total = sum(len(wv) for wv in want)
        stats = spec.stats.as_dict() if hasattr(spec.stats, "as_dict") else {}
        return {"tokens": total, "tokens_identical": got == want, "identical_fraction": round(same / total, 4),
                "acceptance": stats, "greedy_s": round(t_base, 3), "dspark_s": round(t_spec, 3),
                "rule": "identical_fraction >= 0.9 (near-ties of random-init logits may flip between the "
                        "1-token and 5-token paths)", "passed": same / total >= 0.9}

    def _torchrun(self, module: str, extra: list[str]) -> dict:
        if self.a.gpus < 2:
            return skipped("needs --gpus >= 2")
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={self.a.gpus}",
               "--master-addr", "127.0.0.1", f"--master-port={self.a.master_port}", "-m", module, *extra]
        p = subprocess.run(cmd, capture_output=True, text=True, timeout=self.a.torchrun_timeout_s)
        line = next((ln for ln in reversed(p.stdout.splitlines()) if ln.startswith("{")), None)
        rec = {"cmd": " ".join(cmd), "rc": p.returncode, "result": json.loads(line) if line else None,
               "stderr_tail": p.stderr[-2000:], "rule": "exit code 0", "passed": p.returncode == 0}
        return rec

    def stage_tp_parity(self, st: str) -> dict:
        return self._torchrun("dsv4_flash_deployment_b200.parallel.tp_check", [])

    def stage_ep_parity(self, st: str) -> dict:
        return self._torchrun("dsv4_flash_deployment_b200.parallel.ep_check", [])

    def _eval(self, kind: str, data: str | None, name: str) -> dict:
        if not self.a.server or not data:
            return skipped(f"needs --server and --{name}-data")
        import asyncio

        from ..bench.evals import load_items, run_eval

        partial = str(self.out / f"{name}.partial.jsonl")
        r = asyncio.run(run_eval(kind, self.a.server, self.a.served_model, load_items(data), self.a.eval_max_tokens,
                                 self.a.eval_temperature, self.a.eval_concurrency, partial, limit=self.a.eval_limit))
        r["rule"] = f"complete, no errors, pass@1 >= {self.a.min_accuracy}"
        r["passed"] = bool(r["verdict"]["ok"] and r["pass@1"] >= self.a.min_accuracy)
        return r

    def stage_gsm8k(self, st: str) -> dict:
        return self._eval("math", self.a.gsm8k_data, "gsm8k")

    def stage_gpqa_diamond(self, st: str) -> dict:
        return self._eval("mc", self.a.gpqa_data, "gpqa")

    # ------------------------------------------------------------- helpers
    def _engine(self, max_seqs: int, max_len: int):
        from ..engine.engine import Engine

        if self.device == "cpu":
            from ..models.oracle_step import OracleStepModel

            model = OracleStepModel(self.cfg, self.weights(), n_slots=max_seqs, max_seq_len=max_len)
            return Engine(model, max_seqs, 64, max_len, use_graphs=False)
        w = self.weights() if self.a.checkpoint else None      # random init is drawn on the device
        return Engine.build(self.cfg, "cuda", max_seqs=max_seqs, max_batched_tokens=max(64, max_seqs),
                            max_seq_len=max_len, weights=w, seed=self.a.seed)


def parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="resumable model-level verification stages")
    ap.add_argument("--out", required=True, help="directory of the <stage>.json records")
    ap.add_argument("--stages", default="all", help="comma-separated stage names, or a preset: all, quick, perf")
    ap.add_argument("--model", default="v4-check", help="named model config")
    ap.add_argument("--device", default=None, choices=["cuda", "cpu"], help="default: cuda when available")
    ap.add_argument("--checkpoint", default=None, help="safetensors directory (default: random weights)")
    ap.add_argument("--seed", type=int, default=3)
    ap.add_argument("--force", action="store_true", help="rerun stages that passed before")
    ap.add_argument("--max-len", type=int, default=128)
    ap.add_argument("--n-seqs", type=int, default=3)
    ap.add_argument("--seq-len", type=int, default=52)
    ap.add_argument("--max-startup-s", type=float, default=900.0)
    ap.add_argument("--golden", default=None, help="golden token file (verify/golden.py make)")
    ap.add_argument("--min-tie-aware", type=float, default=0.8)
    ap.add_argument("--ctx", type=int, default=256, help="context of the perf stages")
    ap.add_argument("--perf-steps", type=int, default=20)
    ap.add_argument("--perf-warmup", type=int, default=3)
    ap.add_argument("--dspark-tokens", type=int, default=20)
    ap.add_argument("--gpus", type=int, default=1, help="GPUs of the tp_parity / ep_parity stages")
    ap.add_argument("--master-port", type=int, default=29531)
    ap.add_argument("--torchrun-timeout-s", type=float, default=900.0)
    ap.add_argument("--server", default=None, help="base URL of a running server (evaluation stages)")
    ap.add_argument("--served-model", default="deepseek-v4-flash")
    ap.add_argument("--gsm8k-data", default=None)
    ap.add_argument("--gpqa-data", default=None)
    ap.add_argument("--eval-max-tokens", type=int, default=2048)
    ap.add_argument("--eval-temperature", type=float, default=0.0)
    ap.add_argument("--eval-concurrency", type=int, default=16)
    ap.add_argument("--eval-limit", type=int, default=None)
    ap.add_argument("--min-accuracy", type=float, default=0.0)
    return ap


def main(argv=None) -> int:
    a = parser().parse_args(argv)
    if a.device is None:
        import torch

        a.device = "cuda" if torch.cuda.is_available() else "cpu"
    if a.device == "cuda":
        from ..ops import _ext

        _ext.load(required=True)
    summary = Runner(a).run()
    bad = [s for s, v in summary.items() if v == "FAILED"]
    print(json.dumps({"verify": summary, "out": str(a.out)}))
    return 1 if bad else 0


if __name__ == "__main__":
    raise SystemExit(main())
