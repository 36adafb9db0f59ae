"""Expert parallelism across the GPUs of one node.

Ranks own contiguous expert ranges (EP = world size; 256/8 = 32 experts per
rank for V4-Flash, 384/8 = 48 for V4.1).  Attention is data-parallel, so
every rank routes its own tokens and exchanges (token, expert) pairs:

  pack     routed pairs -> per-destination transport records (ep.cu)
  exchange records to their expert's rank          (dispatch)
  experts  plan + unpack + grouped W13/SwiGLU/W2 on the received rows
  return   expert output rows back to the source   (combine)
  combine  the mHC boundary kernel sums a token's rows by position

Transports: ``nccl`` = ``all_to_all_single`` over fixed-capacity per-peer
regions (the baseline; no host synchronization, graph-capturable); ``p2p`` =
the pack/combine kernels store records straight into the peer's receive
buffer through NVLink (symmetric memory) and a device barrier orders the two
sides.  Capacity per peer is the worst case ``T * k`` pairs (every pair of a rank
to one peer), so no routing can overflow; an overflow would be reported
through the device error word, never dropped silently.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import _ext
from ..ops.layout import ceil_to


class EPGroup:
    def __init__(self, rank: int, world: int, group=None, device=None, transport: str = "nccl"):
        self.rank = rank
        self.world = world
        self.group = group
        self.dev = torch.device(device) if device is not None else torch.device("cuda", rank)
        self.transport = transport
        self._bufs = None

    def expert_range(self, n_experts: int) -> tuple[int, int]:
        per = n_experts // self.world
        return self.rank * per, per

    def experts_per_rank(self, n_experts: int) -> int:
        return n_experts // self.world

    def cap_per_peer(self, T: int, k: int) -> int:
        # worst case: every routed pair of this rank goes to one peer (a token's k
        # experts are distinct, so T*k bounds it).  Random-init routers are skewed
        # enough to exceed 2x the average; the bound costs ~35 MB per rank.
        return ceil_to(T * k, 16)

    def recv_rows(self, T: int, k: int) -> int:
        return self.world * self.cap_per_peer(T, k)

    def _alloc(self, T: int, k: int, D: int):
        cap = self.cap_per_peer(T, k)
        rec = ceil_to(D + D // 32 + 8, 16)
        n = self.world * cap
        e = lambda *s, dt: torch.empty(*s, dtype=dt, device=self.dev)
        self._bufs = dict(
            cap=cap, rec=rec, k=k,
            cnt=torch.zeros(self.world, dtype=torch.int32, device=self.dev),
            pos_back=e(T, k, dt=torch.int32),
            ids=e(n, 1, dt=torch.int32), wts=e(n, 1, dt=torch.float32), pos=e(n, 1, dt=torch.int32),
            rank=e(n, 1, dt=torch.int32),
        )
        if self.transport == "p2p":
            self._alloc_p2p(n, rec, D)
        else:
            self._bufs.update(
                send=e(n * rec, dt=torch.uint8), recv=e(n * rec, dt=torch.uint8),
                rcnt=torch.zeros(self.world, dtype=torch.int32, device=self.dev),
                back_send=e(n, D, dt=torch.bfloat16), back_recv=e(n, D, dt=torch.bfloat16))

    def _alloc_p2p(self, n: int, rec: int, D: int):
        """Receive buffers in symmetric memory, mapped into every peer's address space.

        Layout of the one symmetric allocation per rank: [recv records | expert
        output rows coming back | receive counts | signal words], each region
        256-byte aligned.  Peers write into it with plain stores from the
        packing kernels; no library kernel ever reads a peer's region.
        """
        import torch.distributed._symmetric_memory as symm_mem

        W = self.world
        sizes = [n * rec, n * D * 2, W * 4, 2 * W * 4]
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
        b = self._bufs
        b.update(
            symm=buf, symm_handle=hdl,
            recv=buf[offs[0]:offs[0] + sizes[0]],
            back_recv=buf[offs[1]:offs[1] + sizes[1]].view(torch.bfloat16).view(n, D),
            rcnt=buf[offs[2]:offs[2] + sizes[2]].view(torch.int32),
            sig=buf[offs[3]:offs[3] + sizes[3]].view(torch.int32),
            peer_recv=table(0), peer_back=table(1), peer_cnt=table(2), peer_sig=table(3),
            done=torch.zeros(2, dtype=torch.int32, device=self.dev),
            epoch=torch.zeros(2, dtype=torch.int32, device=self.dev),
            send=torch.empty(16, dtype=torch.uint8, device=self.dev),
            back_send=torch.empty(1, D, dtype=torch.bfloat16, device=self.dev),
        )
        done, ep = b["done"].data_ptr(), b["epoch"].data_ptr()
        b["sync0"] = torch.tensor([b["peer_sig"].data_ptr(), b["peer_cnt"].data_ptr(), done, ep], dtype=torch.int64)
        b["sync1"] = torch.tensor([b["peer_sig"].data_ptr(), 0, done + 4, ep + 4], dtype=torch.int64)

    def moe(self, model, L, T: int, k: int):
        """Runs the expert-parallel MoE block; returns (rows, positions, topk) for the combine."""
        cfg, ext = model.cfg, model.ext
        D, I = cfg.dim, cfg.moe_inter_dim
        E = cfg.n_experts_for(L.layer_id)
        e_begin, e_local = self.expert_range(E)
        if self._bufs is None:
            self._alloc(model.max_tokens, k, D)
        b = self._bufs
        cap, rec = b["cap"], b["rec"]
        p2p = self.transport == "p2p"
        ids, wts, _, _ = model.route[k]
        with model._t("ep_pack"):
            b["cnt"].zero_()
            ext.ep_pack(ids, wts, T, model.uq, model.usf, e_local, self.world, cap, rec, b["send"], b["cnt"],
                        b["pos_back"], b["peer_recv"] if p2p else None, self.rank, model.err,
                        b["sync0"] if p2p else None)
        with model._t("ep_exchange"):
            if p2p:
                ext.ep_wait(b["sig"], self.world, 0, b["epoch"], model.err)
            else:
                dist.all_to_all_single(b["rcnt"], b["cnt"], group=self.group)
                dist.all_to_all_single(b["recv"], b["send"], group=self.group)
        n = self.world * cap
        with model._t("ep_plan_unpack"):
            ext.ep_unpack_meta(b["recv"], b["rcnt"], self.world, cap, rec, D, b["ids"], b["wts"])
            # only the valid prefix of each peer's segment (rcnt) is visited
            ext.moe_plan(n, 1, e_local, 0, b["ids"], b["wts"], model.counts, model.seg, b["rank"], model.tile_rows,
                         2 * I, D, model.tiles13, model.nt13, model.tiles2, model.nt2, model.cap, b["pos"],
                         model.row_scale, model.err, b["rcnt"], cap)
            ext.ep_unpack_rows(b["recv"], b["rcnt"], self.world, cap, rec, D, b["pos"], model.xperm, model.xperm_sf)
        model._grouped(L, 1)
        with model._t("ep_combine"):
            ext.ep_combine_pack(model.yperm, b["pos"], b["rcnt"], cap, b["back_send"],
                                b["peer_back"] if p2p else None, self.rank, self.world, b["sync1"] if p2p else None)
        if not p2p:
            with model._t("ep_exchange"):
                dist.all_to_all_single(b["back_recv"], b["back_send"], group=self.group)
        with model._t("shared_expert"):
            model._shared_expert(L, T)
        if p2p:
            # the shared expert ran while the peers' rows were in flight
            with model._t("ep_exchange"):
                ext.ep_wait(b["sig"], self.world, 1, b["epoch"][1:], model.err)
        return b["back_recv"], b["pos_back"], k
