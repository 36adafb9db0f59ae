"""Teacher-forced logits parity between the model step and the CPU oracle.

Both sides see the same token sequences.  The model under test runs each
sequence as one prefill chunk of ``prefill_lens[i]`` tokens and then one token
per step (all sequences batched into each step, as the serving engine mixes
them), and the logits of every position it samples are compared with the
oracle's logits at that position (``ref/model.py``, stepped one token at a
time).  The reference's runner compares its megakernel with its oracle model
the same way (``tpu-v7x/deepseek_v41/runner.py:625-665``: teacher-forced
logits, top-1 agreement and cosine).

``device`` "cuda" runs the sm_100a model (``engine/builder.py``); "cpu" runs
the oracle itself as the model under test (the runner's plumbing check on a
machine without a GPU: parity is exact unless ``sinkhorn_iters`` differs).
"""

from __future__ import annotations

import torch


def oracle_logits(cfg, weights: dict, seqs: list[list[int]], max_len: int,
                  sinkhorn_iters: int | None = None) -> list[torch.Tensor]:
    """Per sequence: fp32 logits [len, V] of every position, one token per oracle step."""
    from ..ref.model import RefModel

    ref = RefModel(cfg, weights, max_seq_len=max_len, sinkhorn_iters=sinkhorn_iters)
    out = []
    for s in seqs:
        st = ref.new_state(1)
        lg = []
        for tok in s:
            logits, _ = ref.step(torch.tensor([tok]), st)
            lg.append(logits[0, : cfg.vocab_size].float())
        out.append(torch.stack(lg))
    return out


def device_logits(cfg, weights: dict, seqs: list[list[int]], prefill_lens: list[int], max_len: int,
                  sinkhorn_iters: int | None = None, device: str = "cuda") -> list[dict[int, torch.Tensor]]:
    """Per sequence: {position: fp32 logits [V]} of the positions the model sampled
    (the last token of the prefill chunk, then every decoded position)."""
    if device == "cpu":
        full = oracle_logits(cfg, weights, seqs, max_len, sinkhorn_iters)
        return [{p: full[i][p] for p in range(prefill_lens[i] - 1, len(s))} for i, s in enumerate(seqs)]
    from ..engine.builder import build_model
    from ..models.model import SeqChunk, StepMeta
    from ..ops.gemm import ErrorWord

    model = build_model(cfg, device, max_tokens=max(128, sum(prefill_lens)), n_slots=len(seqs) + 1,
                        max_seq_len=max_len, weights=weights)
    if sinkhorn_iters is not None:
        model.sinkhorn_iters = sinkhorn_iters
    got: list[dict[int, torch.Tensor]] = [dict() for _ in seqs]
    pos = [0] * len(seqs)
    while any(p < len(s) for p, s in zip(pos, seqs)):
        chunks = []
        for i, s in enumerate(seqs):
            if pos[i] >= len(s):
                continue
            n = prefill_lens[i] if pos[i] == 0 else 1
            chunks.append((i, SeqChunk(i, pos[i], s[pos[i]:pos[i] + n], True)))
        meta = StepMeta(cfg, [c for _, c in chunks])
        model.upload(meta)
        model.forward(meta)
        torch.cuda.synchronize()
        ErrorWord.check(device)
        lg = model.logits[: len(chunks), : cfg.vocab_size].float().cpu()
        for row, (i, c) in enumerate(chunks):
            last = c.start_pos + len(c.tokens) - 1
            got[i][last] = lg[row]
            pos[i] = last + 1
    del model
    return got


def compare(got: list[dict[int, torch.Tensor]], ref: list[torch.Tensor]) -> dict:
    """Worst / mean cosine and top-1 agreement over every compared position."""
    cs = []
    agree = total = 0
    for i, per in enumerate(got):
        for p, lg in per.items():
            r = ref[i][p]
            cs.append(float(torch.nn.functional.cosine_similarity(lg.float(), r.float(), dim=-1)))
            agree += int(int(lg.argmax()) == int(r.argmax()))
            total += 1
    return {"positions": total, "cos_min": min(cs), "cos_mean": sum(cs) / len(cs), "top1": agree / total}
