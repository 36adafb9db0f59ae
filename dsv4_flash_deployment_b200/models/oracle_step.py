"""CPU step model on the oracle, with the step interface of :class:`.model.DSV4Model`.

The serving engine drives a model through three members: ``cfg``, ``dev`` and
``forward(meta) -> sampled ids`` (plus ``upload``).  This class gives the
engine, the scheduler, the HTTP server and the multi-rank control plane a
model that runs anywhere (tests, a laptop, gloo ranks) with the oracle's
exact numerics: every slot owns a :class:`..ref.model.RefState`; a chunk is
stepped token by token; a sampled chunk returns the greedy argmax of its last
token (or a sample under the chunk's temperature / top-k / top-p, with the
same rules as the device head, models/sampling.py).  It is a test and plumbing
backend, not a serving path.
"""

from __future__ import annotations

import torch

from ..ref.model import RefModel, RefState
from .model import StepMeta
from .sampling import LOGPROB_TOP_N, chosen_logprob, logprob_top, seed_key, seeded_gumbel, top_k_top_p_mask_


class OracleStepModel:
    def __init__(self, cfg, weights: dict[str, torch.Tensor], n_slots: int, max_seq_len: int,
                 ref: RefModel | None = None):
        self.cfg = cfg
        self.dev = torch.device("cpu")
        self.ref = ref or RefModel(cfg, weights, max_seq_len=max_seq_len)
        self.states: list[RefState | None] = [None] * n_slots
        self.last_upload_bytes = 0
        self._gen = torch.Generator().manual_seed(0)

    def upload(self, meta: StepMeta, pinned: dict | None = None) -> None:
        self.last_upload_bytes = 0

    def forward(self, meta: StepMeta) -> torch.Tensor:
        out = []
        lp_rows = []
        for c in meta.chunks:
            st = self.states[c.slot]
            if c.start_pos == 0 or st is None:
                if c.start_pos != 0:
                    raise RuntimeError(f"slot {c.slot}: chunk at {c.start_pos} without a prefix")
                st = self.ref.new_state(1)
                self.states[c.slot] = st
            if st.pos != c.start_pos:
                raise RuntimeError(f"slot {c.slot}: state at {st.pos}, chunk starts at {c.start_pos}")
            logits = None
            for tok in c.tokens:
                logits, _ = self.ref.step(torch.tensor([tok]), st)
            if c.sample:
                lg = logits[0].float()[None, : self.cfg.vocab_size].clone()
                raw = lg.clone()
                temp = torch.tensor([c.temperature])
                if c.temperature > 0 and (c.top_k > 0 or c.top_p < 1.0):
                    top_k_top_p_mask_(lg, temp, torch.tensor([c.top_k], dtype=torch.int32),
                                      torch.tensor([c.top_p]))
                if c.temperature > 0:   # Gumbel-max, as the device model samples
                    if c.seed is not None:
                        key = torch.tensor([seed_key(c.seed, c.start_pos + len(c.tokens) - 1)])
                        g = seeded_gumbel(key, lg.shape[1])
                    else:
                        u = torch.rand(lg.shape, generator=self._gen).clamp_(1e-20, 1.0 - 1e-7)
                        g = -torch.log(-torch.log(u))
                    lg = lg + c.temperature * g
                tok = int(lg.argmax())
                out.append(tok)
                n_top = min(LOGPROB_TOP_N, raw.shape[1])
                lse, vals, ids = logprob_top(raw, n_top)
                lp_rows.append((float(chosen_logprob(raw, torch.tensor([tok]), lse)[0]), vals[0], ids[0]))
        S = len(out)
        self.lp_chosen = torch.tensor([r[0] for r in lp_rows], dtype=torch.float32)
        self.lp_vals = torch.stack([r[1] for r in lp_rows]) if S else torch.zeros(0, LOGPROB_TOP_N)
        self.lp_ids = torch.stack([r[2] for r in lp_rows]).int() if S else torch.zeros(0, LOGPROB_TOP_N, dtype=torch.int32)
        return torch.tensor(out, dtype=torch.int32)
