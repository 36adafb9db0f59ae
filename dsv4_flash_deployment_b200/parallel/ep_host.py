"""Expert-parallel dispatch/combine on host tensors (gloo or any backend).

The same protocol as the GPU path in :mod:`.ep` — contiguous expert ranges
per rank, (token, expert) pairs sorted by expert and therefore by owner rank,
a counts exchange then a payload exchange, the expert FFN on the owner, the
weighted rows sent back and summed per token in ascending expert order — but
on CPU tensors through ``torch.distributed.all_to_all_single``, so the
data-parallel-attention + EP plumbing runs (and is tested) without a GPU.

The expert-ascending summation order is also the order of the single-rank
oracle (:meth:`..ref.model.RefModel._moe`), so EP and dense agree to the
last bit whenever the per-row expert FFN is row-independent.

Reference: the routed-expert ``psum`` of the TP/EP decode
(``models/DeepSeekV4.1-Flash-v6e16/tpu-v7x/deepseek_v41/xla_decode.py:1440-1458``)
and vLLM's ``--enable-expert-parallel`` MoE (``kernel-optimizations-recipe/
dsv41-flash-v6e16-serving.yaml:367``).
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


class HostEP:
    def __init__(self, n_experts: int, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split over {self.world} ranks")
        self.per = n_experts // self.world
        self.stats = {"calls": 0, "sent_rows": 0, "recv_rows": 0}

    def owns(self, e: int) -> bool:
        return e // self.per == self.rank

    def local_experts(self) -> range:
        return range(self.rank * self.per, (self.rank + 1) * self.per)

    def _a2a(self, send: torch.Tensor, send_counts: list[int], recv_counts: list[int]) -> torch.Tensor:
        recv = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype)
        dist.all_to_all_single(recv, send.contiguous(), recv_counts, send_counts, group=self.group)
        return recv

    def moe(self, x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor,
            expert_fn: Callable[[int, torch.Tensor, torch.Tensor], torch.Tensor], out_dim: int) -> torch.Tensor:
        """Routed-expert output for this rank's tokens.

        ``x`` [T, D], ``ids``/``wts`` [T, k]; ``expert_fn(e, rows, w)`` returns the
        gate-weighted FFN output of local expert ``e`` for ``rows`` (fp32).
        Every rank must call this the same number of times (T may be 0).
        """
        T, k = ids.shape
        flat_e = ids.reshape(-1).to(torch.int64)
        flat_t = torch.arange(T).repeat_interleave(k)
        flat_w = wts.reshape(-1).float()
        order = torch.sort(flat_e, stable=True).indices          # expert-ascending, stable in token order
        e_s, t_s, w_s = flat_e[order], flat_t[order], flat_w[order]
        dest = e_s // self.per
        send_counts = torch.bincount(dest, minlength=self.world).tolist()
        # counts exchange (one int per peer), then the payload: rows, expert id, weight
        cnt_send = torch.tensor(send_counts, dtype=torch.int64)
        cnt_recv = torch.empty(self.world, dtype=torch.int64)
        dist.all_to_all_single(cnt_recv, cnt_send, group=self.group)
        recv_counts = cnt_recv.tolist()
        rows = self._a2a(x[t_s].float(), send_counts, recv_counts)
        r_e = self._a2a(e_s, send_counts, recv_counts)
        r_w = self._a2a(w_s, send_counts, recv_counts)
        # owner: run each local expert on its rows (source-rank order kept within an expert)
        y_back = torch.zeros(rows.shape[0], out_dim)
        for e in torch.unique(r_e).tolist():
            if not self.owns(e):
                raise RuntimeError(f"rank {self.rank} received rows for expert {e} it does not own")
            sel = torch.nonzero(r_e == e).squeeze(1)
            y_back[sel] = expert_fn(e, rows[sel].to(x.dtype), r_w[sel][:, None]).float()
        # combine: rows come back in the order they were sent (expert-ascending)
        y_pairs = self._a2a(y_back, recv_counts, send_counts)
        y = torch.zeros(T, out_dim)
        for e in torch.unique(e_s).tolist():
            sel = torch.nonzero(e_s == e).squeeze(1)
            y.index_add_(0, t_s[sel], y_pairs[sel])
        self.stats["calls"] += 1
        self.stats["sent_rows"] += int(sum(send_counts))
        self.stats["recv_rows"] += int(sum(recv_counts))
        return y


def ep_ref_model(cfg, weights: dict[str, torch.Tensor], group=None, **kw):
    """A CPU oracle model whose routed experts are split over the ranks of ``group``.

    Each rank keeps only its own experts' tensors; attention and the shared
    expert are replicated (data-parallel attention: each rank steps its own
    sequences).  All ranks must step in lockstep (same number of calls).
    """
    from ..ref import numerics as N
    from ..ref.model import RefModel

    class EPRefModel(RefModel):
        def __init__(self):
            self.ep = HostEP(cfg.n_routed_experts, group)
            local = {f".ffn.experts.{e}." for e in self.ep.local_experts()}
            w = {k: v for k, v in weights.items()
                 if ".ffn.experts." not in k or any(s in k for s in local)}
            super().__init__(cfg, w, **kw)

        def _moe(self, lid: int, x: torch.Tensor, prefix: str) -> torch.Tensor:
            c = self.cfg
            ids, wts = N.route(x, self.w[f"{prefix}.ffn.gate.weight"], self.w[f"{prefix}.ffn.gate.bias"],
                               c.topk_for(lid), c.route_scale, c.score_func)

            def fn(e, rows, wt):
                ep = f"{prefix}.ffn.experts.{e}"
                return N.expert_ffn(rows, self.w[f"{ep}.w1.weight"], self.w[f"{ep}.w1.scale"],
                                    self.w[f"{ep}.w3.weight"], self.w[f"{ep}.w3.scale"],
                                    self.w[f"{ep}.w2.weight"], self.w[f"{ep}.w2.scale"], c.swiglu_limit, wt)

            y = self.ep.moe(x, ids, wts, fn, c.dim)
            sp = f"{prefix}.ffn.shared_experts"
            shared = N.expert_ffn(x, self.w[f"{sp}.w1.weight"], self.w[f"{sp}.w1.scale"],
                                  self.w[f"{sp}.w3.weight"], self.w[f"{sp}.w3.scale"],
                                  self.w[f"{sp}.w2.weight"], self.w[f"{sp}.w2.scale"], c.swiglu_limit)
            return (y + shared).to(torch.bfloat16)

    return EPRefModel()
