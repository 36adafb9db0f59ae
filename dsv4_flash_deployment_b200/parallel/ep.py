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
sides; ``fused`` (the default of the benchmark) = three kernels per MoE layer
and no copy on either side (:meth:`EPGroup.moe_fused`):

  ep_dispatch  router top-k + each pair claims a row of its expert on the owner
               (system-scope atomic) and stores the token's MXFP8 row there
  ep_plan      waits for every rank's dispatch, builds the GEMM tile lists
  grouped W13 / W2  the W2 epilogue stores each expert row into the source
               rank's return buffer; the next mHC boundary kernel waits and
               combines

Capacity per peer (``nccl``/``p2p``) is the worst case ``T * k`` pairs (every
pair of a rank to one peer), and per expert (``fused``) every token of every
rank, so no routing can overflow; an overflow would be reported through the
device error word, never dropped silently.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops.gemm import EPI_BF16, EPI_SWIGLU
from ..ops.layout import ceil_to


class EPGroup:
    def __init__(self, rank: int, world: int, group=None, device=None, transport: str = "nccl",
                 shared_first: bool | None = None):
        """``shared_first`` (fused transport): run the shared expert between the
        dispatch and the plan's wait instead of after the W2 GEMM (default from
        ``DSV4_EP_SHARED_FIRST``, off)."""
        import os

        self.shared_first = (os.environ.get("DSV4_EP_SHARED_FIRST", "0") == "1") if shared_first is None \
            else shared_first
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

    # ------------------------------------------------------------ fused path
    def _alloc_fused(self, T: int, k: int, D: int, I: int, e_local: int, tile_rows: int, shared: bool = False):
        """One symmetric allocation per rank: [expert rows e4m3 | their scale chunks |
        row weights f32 | row origins int32 | per-expert counters | return rows bf16
        (T*k pairs) | signal words]; expert e owns rows [e*cap_e, (e+1)*cap_e) with
        cap_e = every token of every rank (no routing can overflow it).  Local:
        the SwiGLU intermediate in the same row layout and the tile lists.

        ``shared``: the shared expert rides in the grouped GEMMs.  Its input segment
        (this rank's T tokens) follows the expert rows at ``shared_row0`` (row weight
        1, return destination row T*k + t of this rank's own return buffer, both
        constant) and its output rows follow the T*k pair rows of the return buffer."""
        import torch.distributed._symmetric_memory as symm_mem

        W = self.world
        # rows per expert: every pair of every rank, in the GEMM tiles' row layout
        # (tiles under 128 rows each take a 128-row slot)
        pairs = max(1, T) * W
        cap_e = ceil_to(pairs if tile_rows >= 128 else -(-pairs // tile_rows) * 128, 256)
        rows = e_local * cap_e
        srows = ceil_to(max(1, T), 256) if shared else 0
        xrows = rows + srows
        ret0 = max(1, T * k)                       # first shared output row of the return buffer
        kt = D // 128
        sizes = [xrows * D, (xrows // 128) * kt * 512, xrows * 4, xrows * 4, e_local * 4, (ret0 + srows) * D * 2,
                 2 * W * 4]
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
        e = lambda *s_, dt: torch.empty(*s_, dtype=dt, device=self.dev)
        tiles_max = (T * W * k) // tile_rows + e_local + 1   # sum over experts of ceil(rows / tile_rows)
        tiles_max += srows // tile_rows
        b = dict(
            cap_e=cap_e, rows=rows, xrows=xrows, k=k, tile_rows=tile_rows, symm=buf, symm_handle=hdl,
            shared=shared, shared_row0=rows if shared else -1, ret0=ret0,
            x=view(0).view(xrows, D), xsf=view(1), rscale=view(2).view(torch.float32),
            meta=view(3).view(torch.int32), cnt=view(4).view(torch.int32),
            back=view(5).view(torch.bfloat16).view(ret0 + srows, D), sig=view(6).view(torch.int32),
            tables=[table(i) for i in range(5)], peer_back=table(5), peer_sig=table(6),
            done=torch.zeros(2, dtype=torch.int32, device=self.dev),
            epoch=torch.zeros(2, dtype=torch.int32, device=self.dev),
            h=e(xrows, I, dt=torch.uint8), hsf=torch.zeros((xrows // 128) * (I // 128) * 512, dtype=torch.uint8,
                                                           device=self.dev),
            tiles13=e(tiles_max * (2 * I // 128), 4, dt=torch.int32),
            tiles2=e(tiles_max * (D // 128), 4, dt=torch.int32),
            nt13=torch.zeros(1, dtype=torch.int32, device=self.dev),
            nt2=torch.zeros(1, dtype=torch.int32, device=self.dev),
            # the return buffer holds pair (t, slot) at row t * k + slot: the combine's positions
            pos_id=torch.arange(max(1, T * k), dtype=torch.int32, device=self.dev).view(-1, k) if T * k else None,
        )
        if shared:
            # constant per shared row: weight 1, returned to this rank's row ret0 + t
            b["rscale"][rows:xrows].fill_(1.0)
            b["meta"][rows:xrows].copy_((self.rank << 24) + ret0 + torch.arange(srows, dtype=torch.int32,
                                                                               device=self.dev))
            torch.cuda.synchronize(self.dev)
        b["tab_cpu"] = torch.tensor([t.data_ptr() for t in b["tables"]], dtype=torch.int64)
        sync = lambda ph: torch.tensor([b["peer_sig"].data_ptr(), b["sig"].data_ptr(), b["done"].data_ptr() + 4 * ph,
                                        b["epoch"].data_ptr() + 4 * ph, ph, W, self.rank], dtype=torch.int64)
        b["sync0"], b["sync1"] = sync(0), sync(1)
        # mHC boundary descriptor: wait for phase 1, then the local combine (tp_mode 4)
        b["hc_desc"] = torch.cat([torch.tensor([4], dtype=torch.int64), b["sync1"],
                                  torch.zeros(5, dtype=torch.int64)])
        self._fb = b

    def moe_fused(self, model, L, T: int, k: int, logits: torch.Tensor):
        """Fused expert-parallel MoE block (router top-k included); returns
        (rows, positions, topk, hc_post descriptor) for the next mHC boundary."""
        cfg, ext = model.cfg, model.ext
        D = cfg.dim
        I = L.experts.inter
        E = cfg.n_experts_for(L.layer_id)
        _, e_local = self.expert_range(E)
        if getattr(self, "_fb", None) is None:
            self._alloc_fused(model.max_tokens, k, D, I, e_local, model.tile_rows, shared=model.merge_shared)
        b = self._fb
        if b["k"] != k:
            raise NotImplementedError("fused expert parallelism with several routing widths")
        merged = b["shared"] and L.shared_w13 is not None
        ids, wts, _, _ = model.route[k]
        with model._t("ep_dispatch"):
            ext.ep_dispatch(logits[:T], T, L.gate_b, k, 1 if cfg.score_func == "sigmoid" else 0, cfg.route_scale,
                            ids, wts, model.uq, model.usf, e_local, b["cap_e"], b["tile_rows"], b["ret0"],
                            b["tab_cpu"], model.err, b["sync0"], b["shared_row0"] if merged else -1)
        if self.shared_first and not merged:
            # the shared expert runs while the peers' dispatched rows are in flight
            with model._t("shared_expert"):
                model._shared_expert(L, T)
        with model._t("ep_plan"):
            ext.ep_plan(b["sync0"], b["cnt"], b["cap_e"], b["tile_rows"], 2 * I, D, b["tiles13"], b["nt13"],
                        b["tiles2"], b["nt2"], model.err, T if merged else 0, b["shared_row0"] if merged else 0)
        ex = L.experts
        a13 = (L.shared_w13.q, L.shared_w13.sf) if merged else (None, None)
        a2 = (L.shared_w2.q, L.shared_w2.sf) if merged else (None, None)
        with model._t("grouped_w13"):
            ext.gemm_a2(ex.w13.kind, EPI_SWIGLU, ex.w13.q, ex.w13.sf, b["x"], b["xsf"], None, ex.w13.q.shape[0],
                        b["xrows"], D, b["tile_rows"], 1, b["tiles13"], b["nt13"], b["rscale"], b["h"], b["hsf"],
                        cfg.swiglu_limit, 2 * I, 0, None, None, model.err, 0, 1, None, None, None, *a13)
        with model._t("grouped_w2"):
            ext.gemm_a2(ex.w2.kind, EPI_BF16, ex.w2.q, ex.w2.sf, b["h"].view(b["xrows"], I), b["hsf"], None,
                        ex.w2.q.shape[0], b["xrows"], I, b["tile_rows"], 1, b["tiles2"], b["nt2"], None, None, None,
                        0.0, D, D, None, None, model.err, 0, 1, b["sync1"], b["meta"], b["peer_back"], *a2)
        if merged:
            # the shared expert's rows came back with the routed ones (rows ret0 + t)
            model.shared_y = b["back"][b["ret0"]:b["ret0"] + T]
        else:
            if not self.shared_first:
                # the shared expert runs while the expert rows travel back
                with model._t("shared_expert"):
                    model._shared_expert(L, T)
            model.shared_y = model.shared_out
        return b["back"], b["pos_id"], k, b["hc_desc"]

    def release(self) -> None:
        """Drops the exchange buffers (symmetric memory) once the device is idle."""
        torch.cuda.synchronize(self.dev)
        self._bufs = None
        self._fb = None

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
                         model.row_scale, model.err, b["rcnt"], cap, 0, 0)
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
