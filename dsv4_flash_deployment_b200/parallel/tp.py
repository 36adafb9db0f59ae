"""Tensor parallelism across the GPUs of one node (low-latency decode layout).

Every rank holds the same tokens (the scheduler's step is replicated) and the
same residual streams; the weight-heavy projections are split so each GPU
streams 1/N of them (reference: ``--tensor-parallel-size``,
``deepseek_v41/xla_decode.py:738-962`` shards heads, ``wo_a`` groups and
``wo_b``; the vocab-parallel head ``:1484-1490``):

  attention  wq_b rows by head (64/N heads per rank), the attention kernel on
             those heads, wo_a by group (o_groups/N per rank), wo_b by input
             column -> an f32 partial [T, D] per rank
  experts    ownership as in expert parallelism (E/N per rank); tokens are
             already everywhere, so there is no dispatch: each rank runs its
             experts on the pairs routed to them
  head       rows of the (padded) vocabulary, local argmax -> (value, index)

and three exchanges over NVLink replace the reduce collectives, each split
between the kernel that produces the data and the kernel that consumes it
(no separate collective launch):

  phase 0  the wo_b GEMM publishes its partial when its last tile is stored;
           the next mHC boundary kernel waits and sums every rank's partial in
           rank order (the same bits on every rank, so the replicated streams
           never drift apart)
  phase 1  the grouped W2 GEMM publishes its expert rows; the mHC boundary
           kernel reads each (token, slot) row from the rank that owns the
           expert (the same rows and summation order as one GPU)
  phase 2  the head's merge kernel publishes (value, index) pairs and keeps
           the best over ranks

Replicated (cheap or latency-critical): embedding, wq_a/wkv, norms, the
compressor and indexer (their caches are shared by all heads), the router and
the shared expert.  Peers only read each other's symmetric buffers with plain
loads; no library kernel is given a peer's memory.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops.gemm import MxWeight
from ..ops.layout import ceil_to

PH_ATTN, PH_MOE, PH_HEAD = 0, 1, 2
N_PHASES = 3


def mx_rows(w: MxWeight, r0: int, r1: int) -> MxWeight:
    """Rows [r0, r1) of a block-scaled weight (128-row aligned)."""
    assert r0 % 128 == 0 and r1 % 128 == 0 and r1 <= w.q.shape[0], (r0, r1)
    return MxWeight(w.q[r0:r1].contiguous(), w.sf[r0 // 128:r1 // 128].contiguous(), r1 - r0, w.k, w.kind)


def mx_cols(w: MxWeight, k0: int, k1: int) -> MxWeight:
    """Input columns [k0, k1) of a block-scaled weight (128-column aligned)."""
    assert k0 % 128 == 0 and k1 % 128 == 0 and k1 <= w.k, (k0, k1)
    f = 2 if w.q.shape[1] * 2 == w.k else 1    # e2m1 packs two values per byte
    q = w.q[:, k0 // f:k1 // f].contiguous()
    return MxWeight(q, w.sf[:, k0 // 128:k1 // 128].contiguous(), w.n, k1 - k0, w.kind)


class TPGroup:
    """``moe``: how the experts are split.  "ep" (default): each rank owns E/N whole
    experts and gathers a pair's row from its owner.  "tp": every rank holds the
    1/N slice of every expert's intermediate dimension (W13 rows, W2 input
    columns), runs every routed pair on its slice, and the mHC boundary sums the
    N f32 partial rows of each pair (an EP x TP layout with TP = N);
    balanced weight streaming for decode batches where few experts are active."""

    def __init__(self, rank: int, world: int, group=None, device=None, moe: str = "ep"):
        if moe not in ("ep", "tp"):
            raise ValueError(f"moe split {moe!r}")
        self.rank, self.world, self.group = rank, world, group
        self.moe = moe
        self.dev = torch.device(device) if device is not None else torch.device("cuda", rank)
        self._b = None

    # ------------------------------------------------------------ sharding
    def heads(self, n_heads: int) -> int:
        if n_heads % self.world:
            raise ValueError(f"{n_heads} heads do not split over {self.world} ranks")
        return n_heads // self.world

    def groups(self, o_groups: int) -> int:
        if o_groups % self.world:
            raise ValueError(f"{o_groups} output groups do not split over {self.world} ranks")
        return o_groups // self.world

    def expert_range(self, n_experts: int) -> tuple[int, int]:
        if self.moe == "tp":
            return 0, n_experts
        per = n_experts // self.world
        return self.rank * per, per

    def experts_per_rank(self, n_experts: int) -> int:
        return n_experts if self.moe == "tp" else n_experts // self.world

    def inter_local(self, inter: int) -> int:
        """Expert intermediate width on this rank."""
        if self.moe != "tp":
            return inter
        if inter % (128 * self.world):
            raise ValueError(f"expert intermediate {inter} does not split into 128-wide slices over {self.world}")
        return inter // self.world

    def shard_experts(self, ex):
        """This rank's intermediate slice of an expert block holding every expert whole
        (checkpoint path): W13 rows [e*2I + r*2I/N, ...) (gate/up interleaved in
        64-row blocks, so a 128-row aligned slice keeps pairs together), W2 input
        columns [r*I/N, ...)."""
        from ..models.weights import ExpertBlock
        il = self.inter_local(ex.inter)
        E, r = ex.n_experts, self.rank
        rows = [torch.arange(e * 2 * ex.inter + r * 2 * il, e * 2 * ex.inter + (r + 1) * 2 * il) for e in range(E)]
        idx = torch.cat(rows).to(ex.w13.q.device)
        q13 = ex.w13.q.index_select(0, idx).contiguous()
        blocks = (idx.view(-1, 128)[:, 0] // 128)
        sf13 = ex.w13.sf.index_select(0, blocks).contiguous()
        w13 = MxWeight(q13, sf13, E * 2 * il, ex.w13.k, ex.w13.kind)
        w2 = mx_cols(ex.w2, r * il, (r + 1) * il)
        return ExpertBlock(w13, w2, E, il)

    def vocab_rows(self, vocab: int) -> tuple[int, int]:
        """(first row, rows) of this rank's head shard; the vocabulary is padded to
        128 * world rows so every shard is a whole number of 128-row tiles."""
        rows = ceil_to(vocab, 128 * self.world) // self.world
        return self.rank * rows, rows

    def shard_layer(self, cfg, L) -> None:
        """Keeps this rank's part of a layer's attention weights (in place)."""
        hl = self.heads(cfg.n_heads)
        h0 = self.rank * hl
        L.wq_b = mx_rows(L.wq_b, h0 * cfg.head_dim, (h0 + hl) * cfg.head_dim)
        L.sink = L.sink[h0:h0 + hl].contiguous()
        gl = self.groups(cfg.o_groups)
        rows = L.wo_a.shape[0] // cfg.o_groups
        L.wo_a = L.wo_a[self.rank * gl * rows:(self.rank + 1) * gl * rows].contiguous()
        k = L.wo_b.k // self.world
        L.wo_b = mx_cols(L.wo_b, self.rank * k, (self.rank + 1) * k)

    def shard_head(self, head: torch.Tensor, vocab: int) -> torch.Tensor:
        r0, rows = self.vocab_rows(vocab)
        out = torch.zeros(rows, head.shape[1], dtype=head.dtype, device=head.device)
        n = max(0, min(head.shape[0], r0 + rows) - r0)
        if n:
            out[:n] = head[r0:r0 + n]
        return out

    # ------------------------------------------------------------ buffers
    def alloc(self, T: int, D: int, cap_rows: int, k: int, max_sample: int) -> None:
        """Symmetric buffers, one allocation per rank mapped into every peer:
        [wo_b partial f32 T x D | expert rows bf16 cap x D | pair rows int32 T x k |
        head values f32 | head indices int32 | signal words], 256-byte aligned."""
        import torch.distributed._symmetric_memory as symm_mem

        W = self.world
        S = max(max_sample, 1)
        # expert rows: bf16 whole-expert rows ("ep" split) or f32 partial rows ("tp" split)
        sizes = [T * D * 4, cap_rows * D * (4 if self.moe == "tp" else 2), T * k * 4, S * 4, S * 4, N_PHASES * W * 4]
        offs, cur = [], 0
        for sz in sizes:
            offs.append(cur)
            cur += ceil_to(sz, 256)
        buf = symm_mem.empty(cur, dtype=torch.uint8, device=self.dev)
        buf.zero_()
        hdl = symm_mem.rendezvous(buf, self.group if self.group is not None else dist.group.WORLD)
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        ptrs = [int(p) for p in hdl.buffer_ptrs]
        table = lambda i: torch.tensor([p + offs[i] for p in ptrs], dtype=torch.int64, device=self.dev)
        view = lambda i: buf[offs[i]:offs[i] + sizes[i]]
        b = dict(symm=buf, handle=hdl, k=k,
                 part=view(0).view(torch.float32).view(T, D),
                 yperm=view(1).view(torch.float32 if self.moe == "tp" else torch.bfloat16).view(cap_rows, D),
                 pos=view(2).view(torch.int32).view(T, k),
                 aval=view(3).view(torch.float32), aidx=view(4).view(torch.int32),
                 sig=view(5).view(torch.int32),
                 peer_part=table(0), peer_yperm=table(1), peer_pos=table(2), peer_aval=table(3),
                 peer_aidx=table(4), peer_sig=table(5),
                 done=torch.zeros(N_PHASES, dtype=torch.int32, device=self.dev),
                 epoch=torch.zeros(N_PHASES, dtype=torch.int32, device=self.dev))
        self._b = b
        self._sync = [self._sync_desc(ph) for ph in range(N_PHASES)]

    def _sync_desc(self, ph: int) -> torch.Tensor:
        b = self._b
        return torch.tensor([b["peer_sig"].data_ptr(), b["sig"].data_ptr(), b["done"].data_ptr() + 4 * ph,
                             b["epoch"].data_ptr() + 4 * ph, ph, self.world, self.rank], dtype=torch.int64)

    def sync(self, ph: int) -> torch.Tensor:
        return self._sync[ph]

    def buf(self, name: str) -> torch.Tensor:
        return self._b[name]

    def attn_desc(self) -> torch.Tensor:
        """hc_post descriptor: sum every rank's wo_b partial (phase 0)."""
        d = self._b.get("attn_desc")
        if d is None:
            d = torch.cat([torch.tensor([1], dtype=torch.int64), self._sync[PH_ATTN],
                           torch.tensor([self._b["peer_part"].data_ptr(), 0, 0, 0, 0], dtype=torch.int64)])
            self._b["attn_desc"] = d
        return d

    def moe_desc(self, ids: torch.Tensor, e_local: int) -> torch.Tensor:
        """hc_post descriptor (phase 1): gather each pair's expert row from its owner
        ("ep" split), or sum every rank's f32 partial row of each pair ("tp" split)."""
        key = ("moe_desc", ids.data_ptr(), e_local)
        d = self._b.get(key)
        if d is None:
            b = self._b
            if self.moe == "tp":
                # f32 partial rows of every rank, each at the row of that rank's own plan
                d = torch.cat([torch.tensor([3], dtype=torch.int64), self._sync[PH_MOE],
                               torch.tensor([b["peer_yperm"].data_ptr(), 0, b["peer_pos"].data_ptr(), 0, 0],
                                            dtype=torch.int64)])
            else:
                d = torch.cat([torch.tensor([2], dtype=torch.int64), self._sync[PH_MOE],
                               torch.tensor([0, b["peer_yperm"].data_ptr(), b["peer_pos"].data_ptr(),
                                             ids.data_ptr(), e_local], dtype=torch.int64)])
            b[key] = d
        return d

    def release(self) -> None:
        if self._b is not None:
            torch.cuda.synchronize(self.dev)
            self._b = None
