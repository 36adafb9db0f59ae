"""DeepSeek-V4-family model step on the sm_100a kernels.

One call of :meth:`DSV4Model.forward` runs a *mixed batch*: any number of
sequences, each contributing a contiguous run of tokens (one for a decoding
sequence, a chunk for a prefilling one).  Per layer (reference
``_block_step`` reference.py:840-891):

  hc_step (post of previous MoE + mixes + collapse + RMSNorm + MXFP8)
  -> [wq_a|wkv] GEMM -> qkv_post (q norm+quant, kv norm+RoPE+FP8 round trip)
  -> wq_b GEMM -> compressor (kv sources) -> indexer (index sources)
  -> sparse attention over window ring + this step's rows + compressed rows
  -> window ring update -> grouped wo_a (bf16) -> MXFP8 wo_b
  -> hc_step -> router GEMM + top-k -> dispatch plan -> grouped W13 (SwiGLU
     epilogue requantizes to MXFP8) -> grouped W2 -> shared expert
and the next layer's hc_step consumes the expert outputs (combine fused).

All buffers are allocated once for a maximum token count, so a step replays
inside a CUDA graph.  Expert parallelism is a parameter of the MoE block
(``ep_rank, ep_size``): tokens routed to experts of another rank travel in the
dispatch/combine exchange of :mod:`..parallel.ep`.
"""

from __future__ import annotations

import contextlib
import itertools
import os
from dataclasses import dataclass

import numpy as np
import torch

from ..ops import _ext
from ..ops.gemm import (EPI_BF16, EPI_F32, EPI_SWIGLU, ErrorWord, MxWeight, gemm_bf16, gemm_mx,
                        pick_bn)
from ..ops.layout import ceil_to
from ..ref import numerics as N
from .kv_format import ik4_bytes, kv4_bytes, kv8_bytes
from .sampling import LOGPROB_TOP_N, chosen_logprob, gumbel_, logprob_top, seed_key, top_k_top_p_mask_
from .weights import LayerW

ROUTER_SMALL_T = 4   # steps of at most this many tokens route with csrc/moe.cu router_small


# --------------------------------------------------------------------------
# step metadata
# --------------------------------------------------------------------------
@dataclass
class SeqChunk:
    slot: int
    start_pos: int
    tokens: list[int]
    sample: bool = True        # produce logits for the last token of the chunk
    sample_all: bool = False   # produce logits for every token (speculative verify, draft blocks)
    temperature: float = 0.0   # > 0: sample the next token (Gumbel-max) instead of the argmax
    top_k: int = 0             # > 0: sample among the k most likely tokens only (temperature > 0)
    top_p: float = 1.0         # < 1: sample within the top-p nucleus only (temperature > 0)
    logprobs: int | None = None  # n >= 0: also return the sampled token's log-probability and n alternatives
    seed: int | None = None    # samples depend on (seed, position) only (temperature > 0)


class StepMeta:
    """Host description of one mixed step, and its pinned/device mirrors."""

    # per-chunk numeric fields, one column each (built in one pass over the chunks)
    _FIELDS = ("len", "start", "slot", "sample", "sample_all", "temperature", "top_k", "top_p")

    @staticmethod
    def _columns(chunks: list[SeqChunk]) -> np.ndarray:
        if not chunks:
            return np.zeros((0, len(StepMeta._FIELDS)))
        return np.array([(len(c.tokens), c.start_pos, c.slot, c.sample, c.sample_all, c.temperature, c.top_k, c.top_p)
                         for c in chunks], dtype=np.float64)

    def __init__(self, cfg, chunks: list[SeqChunk], ring_pad_slot: int | None = None, _cols=None, _ids=None):
        self.cfg = cfg
        self.chunks = chunks
        n = len(chunks)
        cols = self._columns(chunks) if _cols is None else _cols
        self._cols = cols
        lens = cols[:, 0].astype(np.int64)
        starts = cols[:, 1].astype(np.int64)
        slots = cols[:, 2].astype(np.int64)
        samp = cols[:, 3] != 0
        row0 = np.zeros(n, np.int64)
        if n:
            row0[1:] = np.cumsum(lens)[:-1]
        T = int(lens.sum())
        self.T = T
        self.ids = (np.fromiter(itertools.chain.from_iterable(c.tokens for c in chunks), np.int32, T)
                    if _ids is None else _ids)
        offs = np.arange(T, dtype=np.int64) - np.repeat(row0, lens)
        self.pos = (np.repeat(starts, lens) + offs).astype(np.int32)
        self.slot = np.repeat(slots, lens).astype(np.int32)
        self.chunk_start = np.repeat(starts, lens).astype(np.int32)
        self.step_row0 = np.repeat(row0, lens).astype(np.int32)
        self.last_pos = np.repeat(starts + lens - 1, lens).astype(np.int32)
        sall = cols[:, 4] != 0
        if sall.any():
            rows = [np.arange(row0[i], row0[i] + lens[i]) if sall[i] else
                    (np.array([row0[i] + lens[i] - 1]) if samp[i] else np.zeros(0, np.int64)) for i in range(n)]
            self.sample_rows = np.concatenate(rows).astype(np.int32)
        else:
            self.sample_rows = (row0 + lens - 1)[samp].astype(np.int32)
        # per sampled row: 0 = greedy, > 0 = temperature (one value per chunk)
        temps = cols[:, 5].astype(np.float32)
        per_chunk = np.where(sall, lens, samp.astype(np.int64))
        self.temps = np.repeat(temps, per_chunk).astype(np.float32)
        self.sampling = bool((self.temps > 0).any())
        # top-k / top-p per sampled row (0 / 1.0: off); they only act on rows with T > 0
        topk = cols[:, 6].astype(np.int32)
        topp = cols[:, 7].astype(np.float32)
        self.topk = np.repeat(topk, per_chunk).astype(np.int32)
        self.topp = np.repeat(topp, per_chunk).astype(np.float32)
        self.filtering = bool(((self.temps > 0) & ((self.topk > 0) | (self.topp < 1.0))).any())
        S = len(self.sample_rows)
        if any(c.seed is not None or c.logprobs is not None for c in chunks):
            # seeded rows: the noise key of (seed, position of the sampled token)
            seeds = [c.seed for c, k in zip(chunks, per_chunk) for _ in range(int(k))]
            spos = self.pos[self.sample_rows] if S else np.zeros(0, np.int32)
            self.has_seed = np.array([sd is not None for sd in seeds], dtype=bool)
            self.seedkey = np.array([seed_key(sd, int(p)) if sd is not None else 0 for sd, p in zip(seeds, spos)],
                                    dtype=np.int64)
            # alternatives wanted per sampled row (None: no log-probabilities)
            self.lp_want = [c.logprobs for c, k in zip(chunks, per_chunk) for _ in range(int(k))]
        else:
            self.has_seed = np.zeros(S, bool)
            self.seedkey = np.zeros(S, np.int64)
            self.lp_want = [None] * S
        self.seeded = bool((self.has_seed & (self.temps > 0)).any())
        self.want_lp = any(w is not None for w in self.lp_want)
        self.max_pos = int(self.pos.max()) if T else 0
        # compressor groups closed in this step, per ratio (token order)
        self.groups = {}
        for r in sorted({cfg.ratio(l) for l in cfg.kv_source_layer_ids}):
            mask = (self.pos + 1) % r == 0
            self.groups[r] = (self.slot[mask], (self.pos[mask] // r).astype(np.int32), self.chunk_start[mask],
                              self.step_row0[mask])
        self.clen = {r: ((self.pos + 1) // r).astype(np.int32) for r in self.groups}
        self._lens = lens

    def index_bypass(self, r: int) -> bool:
        """True when every token's compressed length <= index_topk: top-k selects all."""
        return int(self.clen[r].max(initial=0)) <= self.cfg.index_topk

    n_out = None   # sampled rows the caller wants (None: all); set by :meth:`padded`

    @property
    def chunk_bound(self) -> int:
        """Bucketed chunk count: launch sizes that depend on the chunk count (the
        compressor's group grid) are computed from this bound, not the exact count."""
        return token_bucket(len(self.chunks), max(1, self.T))

    def max_groups(self, r: int) -> int:
        """Upper bound of the compressor groups ratio ``r`` can close in this step: a
        chunk of l tokens closes at most l // r + 1 of them."""
        return min(self.T, self.T // r + self.chunk_bound)

    def key(self):
        """Graph key: the launch shapes and control flow of the step (token count,
        sampled rows, chunk-count bucket, indexer bypass per ratio, sampling) and
        nothing else, so steps of different batch compositions share a graph."""
        return (self.T, len(self.sample_rows), self.chunk_bound,
                tuple(self.index_bypass(r) for r in self.groups), self.sampling, self.filtering, self.want_lp,
                self.seeded)

    def padded(self, max_tokens: int, max_sample: int, pad_slot: int) -> "StepMeta":
        """This step padded to bucketed shapes (:func:`token_bucket`): a padding chunk
        of ``T_b - T`` tokens at positions 0.. of the scratch slot ``pad_slot`` (its
        caches absorb the writes), and extra sampled rows repeating row 0.  The
        result's ``n_out`` is the number of real sampled rows."""
        T_b = token_bucket(self.T, max_tokens)
        S = len(self.sample_rows)
        chunks = list(self.chunks)
        cols, ids = self._cols, self.ids
        if T_b > self.T:
            pad = SeqChunk(pad_slot, 0, [0] * (T_b - self.T), sample=False)
            chunks.append(pad)
            cols = np.concatenate([cols, self._columns([pad])])
            ids = np.concatenate([ids, np.zeros(T_b - self.T, np.int32)])
        m = StepMeta(self.cfg, chunks, _cols=cols, _ids=ids)
        S_b = token_bucket(S, max(S, min(max_sample, T_b)))
        if S_b > S:
            extra = S_b - S
            m.sample_rows = np.concatenate([m.sample_rows, np.full(extra, m.sample_rows[0] if S else 0, np.int32)])
            m.temps = np.concatenate([m.temps, np.zeros(extra, np.float32)])
            m.topk = np.concatenate([m.topk, np.zeros(extra, np.int32)])
            m.topp = np.concatenate([m.topp, np.ones(extra, np.float32)])
            m.lp_want = m.lp_want + [None] * extra
            m.has_seed = np.concatenate([m.has_seed, np.zeros(extra, bool)])
            m.seedkey = np.concatenate([m.seedkey, np.zeros(extra, np.int64)])
        m.n_out = S
        return m


def token_bucket(n: int, cap: int) -> int:
    """Padded size of a token / row count: powers of two up to 64, then multiples
    of 64, never above ``cap`` (a count already above ``cap`` stays as it is)."""
    if n <= 0:
        return 0
    b = 1 << (n - 1).bit_length() if n <= 64 else ceil_to(n, 64)
    return max(n, min(b, cap))


# --------------------------------------------------------------------------
# model
# --------------------------------------------------------------------------
class DSV4Model:
    def __init__(self, cfg, layers: list[LayerW], embed: torch.Tensor, head: torch.Tensor, norm_w: torch.Tensor,
                 max_tokens: int, n_slots: int, max_seq_len: int, device, ep=None, max_sample: int | None = None,
                 head_vocab: int | None = None, tp=None, kv_block: int = 0, kv_pool_tokens: int = 0,
                 merge_shared: bool | None = None):
        self.cfg = cfg
        self._want_merge = merge_shared
        self.layers = layers
        self.dev = torch.device(device)
        self.embed = embed
        self.head = head                      # bf16 [pad128(V), D]
        self.vocab = head_vocab or cfg.vocab_size
        self.norm_w = norm_w
        self.max_tokens = max_tokens
        self.n_slots = n_slots
        self.max_seq_len = max_seq_len
        self.ep = ep
        self.tp = tp                          # tensor-parallel group (parallel/tp.py) or None
        self.max_sample = max_sample or max_tokens
        self.pager = None                     # paged compressed caches (models/kv_pages.py) or None
        if kv_block:
            from .kv_pages import KvPager
            self.pager = KvPager(cfg, self.dev, n_slots + 1, max_seq_len, kv_block, kv_pool_tokens)
        self.err = ErrorWord.get(self.dev)
        self.ext = _ext.load()
        self._alloc()

    # ------------------------------------------------------------- buffers
    def _alloc(self):
        cfg, dev, T = self.cfg, self.dev, self.max_tokens
        D = cfg.dim
        Tp = ceil_to(T, 128)
        bf, f32, u8, i32 = torch.bfloat16, torch.float32, torch.uint8, torch.int32
        e = lambda *s, dt=bf: torch.empty(*s, dtype=dt, device=dev)
        z = lambda *s, dt=bf: torch.zeros(*s, dtype=dt, device=dev)
        self.X = e(T, cfg.hc_mult, D)
        self.hc_c = e(T, D)
        self.hc_part = e(T * self.ext.hc_num_slices(D) * 50, dt=f32)
        self.mix_raw = e(T, 48, dt=f32)
        self.mixA, self.mixF = z(T, 24, dt=f32), z(T, 24, dt=f32)
        init = torch.zeros(T, 24, dtype=f32, device=dev)
        init[:, 0] = 1.0
        self.mix0 = init
        self.u = e(T, D)
        self.uq = e(Tp, D, dt=u8)
        self.usf = z(Tp // 128, D // 128, 512, dt=u8)
        qa = cfg.q_lora_rank
        self.qkv = e(T, qa + cfg.head_dim)
        self.qr_q = e(Tp, qa, dt=u8)
        self.qr_sf = z(Tp // 128, qa // 128, 512, dt=u8)
        self.kv_step = z(T, kv8_bytes(cfg.head_dim), dt=u8)   # KV8 records (models/kv_format.py)
        tpw = self.tp.world if self.tp is not None else 1
        self.n_heads_local = cfg.n_heads // tpw
        o_inter = cfg.o_inter // tpw
        self.q = e(T, self.n_heads_local, cfg.head_dim)
        self.o = e(T, self.n_heads_local, cfg.head_dim)
        self.oa = e(T, o_inter)
        self.oa_q = e(Tp, o_inter, dt=u8)
        self.oa_sf = z(Tp // 128, o_inter // 128, 512, dt=u8)
        self.attn_out = e(T, D)
        self.proj = {co: e(T, 2 * co * cfg.head_dim, dt=f32)
                     for co in sorted({cfg.overlap(l) for l in cfg.kv_source_layer_ids})}
        nih = cfg.index_n_heads
        self.qidx = e(T, nih, cfg.index_head_dim)
        self.widx_raw = e(T, nih, dt=f32)
        self.widx = e(T, nih, dt=f32)
        self.comp_idx = e(T, cfg.index_topk, dt=i32)
        self.comp_cnt = e(T, dt=i32)
        self.dense_cnt = e(T, dt=i32)
        max_c = max([self.max_seq_len // cfg.ratio(l) for l in cfg.kv_source_layer_ids] or [1])
        self.cand = z(T, max(1, max_c // max(1, cfg.candidate_block_size)), dt=u8)
        # MoE
        # the tensor-parallel layout runs the backbone only (no MTP stages, whose
        # routing width differs)
        mtp = cfg.n_mtp_layers if self.tp is None else 0
        E = max(cfg.n_routed_experts, cfg.dspark_n_routed_experts if mtp else 0)
        k = max(cfg.n_activated_experts, cfg.dspark_n_activated_experts if mtp else 0)
        self.router_logits = {}
        self.route = {}   # top-k -> (ids, wts, pos, rank)
        for lid in range(cfg.n_layers + mtp):
            ee, kk = cfg.n_experts_for(lid), cfg.topk_for(lid)
            if ee not in self.router_logits:
                self.router_logits[ee] = e(T, ee, dt=f32)
            if kk not in self.route:
                self.route[kk] = (e(T, kk, dt=i32), e(T, kk, dt=f32), e(T, kk, dt=i32), e(T, kk, dt=i32))
        self.counts = e(E, dt=i32)
        self.seg = e(E, dt=i32)
        e_local = E
        if self.ep is not None:
            e_local = self.ep.experts_per_rank(E)
        elif self.tp is not None:
            e_local = self.tp.experts_per_rank(E)
        recv_rows = T * k if self.ep is None else self.ep.recv_rows(T, k)
        # 128-row expert tiles keep two accumulators in TMEM (epilogue overlaps the
        # next tile); 256-row tiles halve weight re-reads when experts get many rows
        # (decided on the expected rows per rank, T*k, not on the worst-case capacity);
        # DSV4_EXPERT_TILE_ROWS=32/64/128/256 overrides (32/64-row tiles take a
        # 128-row slot each and a deeper shared-memory pipeline)
        self.tile_rows = int(os.environ.get("DSV4_EXPERT_TILE_ROWS", "0")) or (
            128 if T * k <= 192 * e_local else 256)
        if self.tile_rows not in (32, 64, 128, 256):
            raise ValueError(f"expert tile rows {self.tile_rows}: 32, 64, 128 or 256")
        # worst-case permuted rows: every expert's segment rounded up (seg_rows in common.cuh)
        if self.tile_rows >= 128:
            self.cap = ceil_to(recv_rows + e_local * 127 + 128, 128)
        else:
            self.cap = ceil_to(-(-recv_rows // self.tile_rows) * 128 + e_local * 128 + 128, 128)
        tiles_rows_max = recv_rows // self.tile_rows + e_local + 1
        # expert intermediate width on this rank (a tensor-parallel expert split keeps 1/N)
        I = self.tp.inter_local(cfg.moe_inter_dim) if self.tp is not None else cfg.moe_inter_dim
        self.inter_local = I
        si = cfg.n_shared_experts * cfg.moe_inter_dim     # the shared expert is never split
        # the shared expert (MXFP8) rides in the routed experts' grouped GEMMs (its tiles
        # read a second weight operand, beside MXFP8 or MXFP4 experts) when it has their
        # intermediate width: its input rows follow the routed rows of the permuted
        # buffers (shared_row0), its output rows are read there by the next mHC
        # boundary.  Not with tensor parallelism, the p2p / NCCL exchanges or token
        # tiles under 128 rows.
        ep_ok = self.ep is None or self.ep.transport == "fused"
        # The two forms round differently (one K pass vs split-K, then the MXFP8 hidden),
        # and random-init V4.1 models amplify that through near-tied indexer picks, so
        # their logits can part (cosine 0.98 at one position) while both keep the same
        # agreement with the fp32 oracle.  ``merge_shared`` False / DSV4_MERGE_SHARED=0:
        # separate GEMMs.
        want = self._want_merge
        if want is None:
            want = os.environ.get("DSV4_MERGE_SHARED", "1") == "1"
        self.merge_shared = bool(want and si == I and self.tile_rows >= 128 and self.tp is None and ep_ok)
        self.shared_row0 = ceil_to(self.cap, 256)
        rows_all = self.shared_row0 + ceil_to(T, 256) if self.merge_shared else self.cap
        self.perm_rows = rows_all
        if self.merge_shared:
            tiles_rows_max += -(-T // self.tile_rows)
        self.tiles13 = e(tiles_rows_max * (2 * I // 128), 4, dt=i32)
        self.tiles2 = e(tiles_rows_max * (D // 128), 4, dt=i32)
        self.nt13, self.nt2 = z(1, dt=i32), z(1, dt=i32)
        self.xperm = e(rows_all, D, dt=u8)
        self.xperm_sf = z(rows_all // 128, D // 128, 512, dt=u8)
        self.hperm = e(rows_all, I, dt=u8)
        self.hperm_sf = z(rows_all // 128, I // 128, 512, dt=u8)
        self.yperm = e(rows_all, D)
        self.row_scale = z(rows_all, dt=f32)
        self.hs = e(Tp, si, dt=u8)
        self.hs_sf = z(Tp // 128, si // 128, 512, dt=u8)
        self.shared_out = e(T, D)
        self.shared_y = self.shared_out   # the shared expert's rows for the next mHC boundary
        self.router_counter = z(1, dt=i32)   # router_small's last-CTA counter (left at zero)
        # head
        self.u_sample = e(self.max_sample, D)
        self.logits = e(self.max_sample, self.head.shape[0], dt=f32)
        self.next_ids = e(self.max_sample, dt=i32)
        self.m_temp = z(self.max_sample, dt=f32)
        self.m_topk = z(self.max_sample, dt=i32)
        self.m_topp = torch.ones(self.max_sample, dtype=f32, device=dev)
        self.m_seedkey = z(self.max_sample, dt=torch.int64)
        self.m_hasseed = torch.zeros(self.max_sample, dtype=torch.bool, device=dev)
        # log-probabilities of the sampled rows (written only by steps that ask for them)
        self.lp_chosen = z(self.max_sample, dt=f32)
        self.lp_vals = z(self.max_sample, LOGPROB_TOP_N, dt=f32)
        self.lp_ids = z(self.max_sample, LOGPROB_TOP_N, dt=i32)
        # multi-CTA argmax: partials [2 * max(S, 296)] + zeroed per-row counters at the end
        self.argmax_scratch = z(2 * max(self.max_sample, 296) + self.max_sample, dt=i32)
        if self.tp is not None:
            # buffers peers read (expert rows, pair rows) live in symmetric memory
            if len(self.route) != 1:
                raise NotImplementedError("tensor parallelism with several routing widths (MTP stages)")
            self.tp.alloc(T, D, self.cap, k, self.max_sample)
            self.yperm = self.tp.buf("yperm")
            ids_, wts_, _, rank_ = self.route[k]
            self.route[k] = (ids_, wts_, self.tp.buf("pos"), rank_)
        # split-K scratch (reused sequentially on the stream)
        self.ws = e(8 * 1024 * 1024, dt=f32)
        self.counters = z(65536, dt=i32)
        # split-row attention at decode sizes: T <= 8 tokens x up to 32 splits
        self.attn_splits = int(os.environ.get("DSV4_ATTN_SPLITS", "16"))
        if not 1 <= self.attn_splits <= 32:
            raise ValueError("DSV4_ATTN_SPLITS must be 1..32")
        self.attn_ws = e(max(1, min(T, 8)) * max(16, self.attn_splits) * 64 * 514, dt=f32)
        # step metadata (device)
        self.m_ids, self.m_pos, self.m_slot = e(T, dt=i32), e(T, dt=i32), e(T, dt=i32)
        self.m_cstart, self.m_row0, self.m_last = e(T, dt=i32), e(T, dt=i32), e(T, dt=i32)
        self.m_sample = e(self.max_sample, dt=torch.int64)
        self.m_groups = {}
        self.m_clen = {}
        self.m_ngroups = {}
        for r in sorted({cfg.ratio(l) for l in cfg.kv_source_layer_ids}):
            self.m_groups[r] = tuple(e(T, dt=i32) for _ in range(4))
            self.m_clen[r] = e(T, dt=i32)
            self.m_ngroups[r] = z(1, dt=i32)
        self._alloc_cache()
        # rope tables on device
        tabs = N.layer_rope_tables(cfg, self.max_seq_len + 8)
        self.rope = {k_: (c.to(dev).contiguous(), s.to(dev).contiguous()) for k_, (c, s) in tabs.items()}

    def _alloc_cache(self):
        cfg, dev = self.cfg, self.dev
        S = self.n_slots + 1  # last slot absorbs padding tokens
        self.ring = {}
        self.comp = {}
        self.idx_cache = {}
        self.comp_ring = {}
        for l in range(cfg.n_layers):
            self.ring[l] = torch.zeros(S, cfg.sliding_window, kv8_bytes(cfg.head_dim), dtype=torch.uint8, device=dev)
        for l in cfg.kv_source_layer_ids:
            r, co = cfg.ratio(l), cfg.overlap(l)
            # contiguous: [slot, entry, dim]; paged: one pool [1, blocks * block, dim] per layer
            shape = (S, max(1, self.max_seq_len // r)) if self.pager is None else (1, self.pager.rows(r))
            self.comp[l] = torch.zeros(*shape, kv4_bytes(cfg.head_dim), dtype=torch.uint8, device=dev)
            if l in cfg.index_source_layer_ids:
                self.idx_cache[l] = torch.zeros(*shape, ik4_bytes(cfg.index_head_dim), dtype=torch.uint8, device=dev)
            self.comp_ring[l] = torch.zeros(S, co * r, 2 * co * cfg.head_dim, dtype=torch.float32, device=dev)
        # order keys of the indexer scores, [T, widest index cache] (scoring CTAs -> select CTA)
        kc = max([max(1, self.max_seq_len // cfg.ratio(l)) for l in self.idx_cache] or [1])
        self.idx_keys = torch.empty(self.max_tokens, kc, dtype=torch.int32, device=dev)

    def _pages(self, lid: int):
        """Page descriptor of layer ``lid``'s compressed caches (None: contiguous)."""
        return None if self.pager is None else self.pager.desc[self.cfg.ratio(lid)]

    def cache_bytes(self) -> int:
        tot = 0
        for d in (self.ring, self.comp, self.idx_cache, self.comp_ring):
            tot += sum(t.numel() * t.element_size() for t in d.values())
        return tot

    # ------------------------------------------------------------- metadata
    def upload(self, m: StepMeta, pinned: dict | None = None) -> None:
        """Host -> device copy of the step metadata (async on the current stream)."""
        T = m.T
        self.last_upload_bytes = 0

        def put(dst, arr):
            self.last_upload_bytes += arr.nbytes
            src = torch.from_numpy(arr)
            if pinned is not None:
                key = id(dst)
                buf = pinned.get(key)
                if buf is None or buf.numel() < dst.numel():
                    buf = torch.empty(dst.numel(), dtype=dst.dtype).pin_memory()
                    pinned[key] = buf
                buf[: len(arr)].copy_(src)
                src = buf[: len(arr)]
            dst[: len(arr)].copy_(src, non_blocking=True)

        if self.pager is not None:
            self.pager.sync()
        put(self.m_ids, m.ids)
        put(self.m_pos, m.pos)
        put(self.m_slot, m.slot)
        put(self.m_cstart, m.chunk_start)
        put(self.m_row0, m.step_row0)
        put(self.m_last, m.last_pos)
        put(self.m_sample, m.sample_rows.astype(np.int64))
        if m.sampling:
            put(self.m_temp, m.temps)
        if m.filtering:
            put(self.m_topk, m.topk)
            put(self.m_topp, m.topp)
        if m.seeded:
            put(self.m_seedkey, m.seedkey)
            put(self.m_hasseed, m.has_seed)
        for r, g in m.groups.items():
            for dst, arr in zip(self.m_groups[r], g):
                if len(arr):
                    put(dst, arr)
            put(self.m_clen[r], m.clen[r])
            put(self.m_ngroups[r], np.asarray([len(g[0])], np.int32))

    last_upload_bytes = 0
    op_timer: dict | None = None
    engram = None            # EngramRuntime for configs with Engram layers

    dev_trace = None         # utils.devtrace.DeviceTrace: a timestamp mark after every op group

    @contextlib.contextmanager
    def _t(self, name: str):
        """CUDA-event timing of one op group (eager runs only; off by default), or a
        device timestamp mark at its end (``dev_trace``; captured with the step)."""
        if self.op_timer is None:
            yield
            if self.dev_trace is not None:
                self.dev_trace.mark(name)
            return
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(name)     # named ranges for timeline profilers
        s.record()
        yield
        e.record()
        torch.cuda.nvtx.range_pop()
        self.op_timer.setdefault(name, []).append((s, e))

    # --------------------------------------------------------------- helpers
    def _gemm(self, xq, xsf, n_tok, w: MxWeight, out, epi=EPI_BF16, **kw):
        """Block-scaled GEMM; few output tiles -> split-K inside a thread-block cluster
        (each split keeps >= 2 k-tiles; the kernel binding trims the split count to
        what the GPU can keep resident)."""
        # splits=-1: the binding picks the split count from the tile count of the
        # weight-tile height it chooses (128 or 256 rows)
        return gemm_mx(xq, xsf, n_tok, w, out, epi, splits=-1, **kw)

    def _gemm_bf16(self, x, w, out, n_tok, f32_out=False, groups=1, m_valid=None):
        bn = pick_bn(n_tok)
        tiles = (w.shape[0] // 128) * ((n_tok + bn - 1) // bn)
        k_tiles = x.shape[1] // groups // 64
        splits = 1
        if tiles < 100:
            splits = max(1, min(8, k_tiles // 2, 148 // max(tiles, 1)))
        return gemm_bf16(x, w, out, f32_out=f32_out, groups=groups, n_tokens=n_tok, m_valid=m_valid, splits=splits,
                         bn=bn)

    def _hc(self, T, Y=None, yperm=None, pos=None, topk=0, prev=None, mixes=None, cw=None, norm=None,
            mix_out=None, u=None, uq=None, usf=None, tap=None, tp=None):
        """One mHC boundary: post/combine/collapse + tensor-core mixes, then Sinkhorn + norm + quant.
        ``tp``: tensor-parallel descriptor; the sublayer output is reduced from the peers."""
        cfg, ext = self.cfg, self.ext
        fnhl = scale = base = None
        if mixes is not None:
            fnhl, scale, base = mixes
        with self._t("hc_post"):
            ext.hc_post(self.X, Y, yperm, pos, topk, prev, fnhl, cw, 24, self.hc_c, self.hc_part, tap, T, tp,
                        self.err)
        if mixes is not None or (cw is not None and u is not None):
            with self._t("hc_finish"):
                ext.hc_finish(self.X, fnhl, scale, base, cw, norm, mix_out, self.hc_c, self.hc_part, u, uq, usf, T,
                              self.sinkhorn_iters, cfg.hc_eps, cfg.rms_norm_eps)

    sinkhorn_iters = None

    # --------------------------------------------------------------- forward
    def forward(self, m: StepMeta, taps: dict | None = None, trace: dict | None = None,
                defer_rings: bool = False) -> torch.Tensor:
        """Runs one step whose metadata is already uploaded; returns next ids [n_sample] (device).

        ``taps``: {layer id: [T, D] bf16 buffer} receives the mean of the four
        streams entering that layer (the DSpark drafter's main hidden).
        ``defer_rings``: a speculative verify step; the per-sequence rings
        (attention window, compressor projections, Engram tokens) are left as
        they are and this step's rows are parked, so that :meth:`commit_rings`
        stores only the accepted prefix.  Position-indexed caches (compressed
        KV, indexer keys) are written as usual: an entry of a rejected token
        is rewritten before any later token can read it.
        """
        cfg = self.cfg
        self._defer = defer_rings
        if self.sinkhorn_iters is None:
            self.sinkhorn_iters = cfg.hc_sinkhorn_iters
        T = m.T
        ext = self.ext
        with self._t("embed"):
            self.ext.embed_streams(self.embed, self.m_ids, T, self.X)
        eng = self.engram
        if eng is not None:
            with self._t("engram_gather"):
                eng.prepare(self, T, update_ring=not defer_rings)
        prev, cw = None, self.mix0
        moe_state = None
        for li, L in enumerate(self.layers):
            lid = L.layer_id
            tap = None
            if taps is not None and lid in cfg.dspark_target_layer_ids:
                tap = taps[lid]
            if eng is not None and lid in eng.layer_index:
                # the streams take the previous MoE output, then the Engram update, and
                # only then this block's mixes and collapse (reference.py:925-931)
                if moe_state is not None:
                    yp, ps, kk, td = moe_state
                    self._hc(T, Y=self.shared_y, yperm=yp, pos=ps, topk=kk, prev=self.mixF, tp=td)
                with self._t("engram"):
                    eng.apply(self, lid, T)
                self._hc(T, prev=None, mixes=L.hc_attn, cw=cw if moe_state is None else self.mixF,
                         norm=L.attn_norm, mix_out=self.mixA, u=self.u, uq=self.uq, usf=self.usf, tap=tap)
            elif moe_state is None:
                self._hc(T, prev=None, mixes=L.hc_attn, cw=cw, norm=L.attn_norm, mix_out=self.mixA, u=self.u,
                         uq=self.uq, usf=self.usf, tap=tap)
            else:
                yp, ps, kk, td = moe_state
                self._hc(T, Y=self.shared_y, yperm=yp, pos=ps, topk=kk, prev=self.mixF, mixes=L.hc_attn,
                         cw=self.mixF, norm=L.attn_norm, mix_out=self.mixA, u=self.u, uq=self.uq, usf=self.usf,
                         tap=tap, tp=td)
            if trace is not None:
                trace[lid] = self.X[:T].clone()
            self._attention(L, m)
            if trace is not None:
                trace[f"attn{lid}"] = self.attn_out[:T].clone()
            tpa = self.tp.attn_desc() if self.tp is not None else None
            self._hc(T, Y=None if tpa is not None else self.attn_out, prev=self.mixA, mixes=L.hc_ffn, cw=self.mixA,
                     norm=L.ffn_norm, mix_out=self.mixF, u=self.u, uq=self.uq, usf=self.usf, tp=tpa)
            moe_state = self._moe(L, T)
        # final collapse + norm on all tokens, then head on the sampled rows
        yp, ps, kk, td = moe_state
        self._hc(T, Y=self.shared_y, yperm=yp, pos=ps, topk=kk, prev=self.mixF, mixes=None, cw=self.mixF,
                 norm=self.norm_w, u=self.u, tp=td)
        S = len(m.sample_rows)
        if S == 0:
            return self.next_ids[:0]
        with self._t("head"):
            torch.index_select(self.u[:T], 0, self.m_sample[:S], out=self.u_sample[:S])
            self._gemm_bf16(self.u_sample[:S], self.head, self.logits[:S], S, f32_out=True)
            if (m.filtering or m.want_lp) and self.tp is not None:
                raise NotImplementedError("top-k / top-p / log-probabilities with the vocab-parallel head")
            if m.want_lp:
                raw = self._raw_logits(S)
                n_top = min(LOGPROB_TOP_N, self.vocab)
                lse, vals, ids = logprob_top(raw, n_top)
                self.lp_vals[:S, :n_top].copy_(vals)
                self.lp_ids[:S, :n_top].copy_(ids)
            if m.filtering:
                top_k_top_p_mask_(self.logits[:S, :self.vocab], self.m_temp[:S], self.m_topk[:S], self.m_topp[:S])
            if m.sampling:
                self._gumbel(S, seeded=m.seeded)
            if self.tp is None:
                ext.argmax_rows(self.logits[:S], S, self.vocab, self.next_ids[:S], self.argmax_scratch, None, 0)
                if m.want_lp:
                    self.lp_chosen[:S].copy_(chosen_logprob(raw, self.next_ids[:S], lse))
            else:
                # vocab-parallel head: best (value, index) of this shard, then the merge over ranks
                tp = self.tp
                r0, rows = tp.vocab_rows(self.vocab)
                valid = max(0, min(rows, self.vocab - r0))
                ext.argmax_rows(self.logits[:S], S, valid, tp.buf("aidx")[:S], self.argmax_scratch,
                                tp.buf("aval")[:S], r0)
                ext.tp_argmax_merge(tp.sync(2), tp.buf("peer_aval"), tp.buf("peer_aidx"), S, self.next_ids[:S],
                                    self.err)
        return self.next_ids[:S]

    def _gumbel(self, S: int, seeded: bool = False) -> None:
        """Temperature sampling by the Gumbel-max rule: the argmax of
        logits + T * g (g ~ Gumbel(0, 1) per vocabulary entry) is a sample of
        softmax(logits / T); rows with T = 0 keep their logits, so they stay
        greedy.  The noise comes from the device generator (captured with the
        step's CUDA graph); under the vocab-parallel head each rank draws the
        noise of its own rows and the cross-rank merge keeps the best."""
        if self._gnoise is None:   # first sampling step runs eagerly, before any capture of it
            self._gnoise = torch.empty_like(self.logits)
        sd = None
        v0 = 0
        if seeded:    # rows with a request seed: noise from (seed, position, vocabulary index) only
            sd = (self.m_seedkey[:S], self.m_hasseed[:S])
            if self.tp is not None:
                v0 = self.tp.vocab_rows(self.vocab)[0]
        gumbel_(self.logits[:S], self.m_temp[:S], self._gnoise[:S], sd, v0)

    _gnoise = None

    def _raw_logits(self, S: int) -> torch.Tensor:
        """Copy of the sampled rows' raw logits (the real vocabulary columns), kept for
        the log-probabilities while filtering and noise change ``logits`` in place.
        Allocated by the first step that asks for log-probabilities (an eager step:
        a step shape's first run precedes its capture)."""
        if self._lp_raw is None:
            self._lp_raw = torch.empty(self.max_sample, self.vocab, dtype=torch.float32, device=self.dev)
        raw = self._lp_raw[:S]
        raw.copy_(self.logits[:S, :self.vocab])
        return raw

    _lp_raw = None

    # ------------------------------------------------- deferred ring commits
    _defer = False
    pending_rows = 256

    def _pending(self, kind: str, lid: int, src: torch.Tensor, T: int) -> None:
        if T > self.pending_rows:
            raise ValueError(f"deferred-ring step of {T} tokens exceeds {self.pending_rows}")
        store = self.__dict__.setdefault("_pend", {})
        buf = store.get((kind, lid))
        if buf is None:
            buf = torch.empty(self.pending_rows, src.shape[1], dtype=src.dtype, device=self.dev)
            store[(kind, lid)] = buf
        buf[:T].copy_(src[:T])

    def commit_rings(self, T: int, last_commit: torch.Tensor) -> None:
        """After a deferred (verify) step: store the rows of positions <= last_commit[t]
        into every ring.  The step's metadata must still be the uploaded one."""
        ext = self.ext
        for (kind, lid), buf in self.__dict__.get("_pend", {}).items():
            ring = self.ring[lid] if kind == "kv" else self.comp_ring[lid]
            ext.ring_update(ring, buf, T, self.m_slot, self.m_pos, last_commit)
        if self.engram is not None:
            self.engram.commit_ring(self, T, last_commit)

    # ------------------------------------------------------------- attention
    def _attention(self, L: LayerW, m: StepMeta, ring: torch.Tensor | None = None, win_len: int = 0):
        """Attention sublayer.  ``ring``/``win_len``: a DSpark draft stage attends to its
        own ring plus every row of the draft block (window ending at the block's
        last position) and stores nothing."""
        cfg, ext = self.cfg, self.ext
        T = m.T
        lid = L.layer_id
        draft = ring is not None
        if ring is None:
            ring = self.ring[lid]
        r = cfg.ratio(lid)
        cos, sin = self.rope["yarn" if r > 0 else "swa"]
        qa = cfg.q_lora_rank
        with self._t("gemm_wqkv_a"):
            self._gemm(self.uq, self.usf, T, L.wqkv_a, self.qkv)
        with self._t("qkv_post"):
            ext.qkv_post(self.qkv, qa, cfg.head_dim, L.q_norm, L.kv_norm, cfg.rms_norm_eps, self.qr_q, self.qr_sf, cos,
                     sin, self.m_pos, self.kv_step, T)
        with self._t("gemm_wq_b"):
            self._gemm(self.qr_q, self.qr_sf, T, L.wq_b, self.q.view(self.q.shape[0], -1))
        comp = None
        comp_idx = None
        comp_cnt = None
        if r > 0:
            src = cfg.kv_source_for(lid)
            if lid in cfg.kv_source_layer_ids:
                self._compress(L, m, r)
            clen = self.m_clen[r]
            if lid in cfg.index_source_layer_ids:
                if m.index_bypass(r):
                    self._idx_sel = None
                else:
                    self._indexer(L, m, r)
                    self._idx_sel = (self.comp_idx, self.comp_cnt)
            if lid in cfg.index_source_layer_ids or lid not in cfg.kv_source_layer_ids:
                sel = getattr(self, "_idx_sel", None)
                if sel is None:
                    comp_cnt = clen
                else:
                    comp_idx, comp_cnt = sel
            else:
                comp_cnt = clen   # owns a compressor but no indexer: dense over its entries
            comp = self.comp[src]
        splits = 1
        if T <= 8:
            splits = self.attn_splits
        tctx = self._t("attention")
        tctx.__enter__()
        ext.attention(self.q, cos, sin, None, cfg.q_head_norm, cfg.rms_norm_eps, self.kv_step, ring, comp,
                      self.m_slot, self.m_pos, self.m_cstart, self.m_row0, comp_idx, comp_cnt, L.sink,
                      cfg.head_dim ** -0.5, self.o, self.attn_ws if splits > 1 else None, T, splits,
                      self.m_last if draft else None, win_len, self._pages(src) if comp is not None else None)
        tctx.__exit__(None, None, None)
        # draft blocks read the window but leave the ring alone (the verify step writes it)
        if not draft and self._defer:
            self._pending("kv", lid, self.kv_step, T)
        elif not draft:
            with self._t("ring_update"):
                ext.ring_update(ring, self.kv_step, T, self.m_slot, self.m_pos, self.m_last)
        groups = cfg.o_groups if self.tp is None else self.tp.groups(cfg.o_groups)
        with self._t("gemm_wo_a"):
            self._gemm_bf16(self.o.view(self.o.shape[0], -1), L.wo_a, self.oa, T, groups=groups)
        with self._t("quant_oa"):
            ext.act_quant_mx(self.oa[:T], self.oa_q, self.oa_sf)
        with self._t("gemm_wo_b"):
            if self.tp is None:
                self._gemm(self.oa_q, self.oa_sf, T, L.wo_b, self.attn_out)
            else:
                # this rank's wo_b input columns -> f32 partial in symmetric memory, published
                # to the peers when the last tile is stored (reduced in the next mHC boundary)
                self._gemm(self.oa_q, self.oa_sf, T, L.wo_b, self.tp.buf("part"), EPI_F32,
                           publish=self.tp.sync(0))

    def _compress(self, L: LayerW, m: StepMeta, r: int):
        cfg, ext = self.cfg, self.ext
        T = m.T
        lid = L.layer_id
        co = cfg.overlap(lid)
        width = 2 * co * cfg.head_dim
        proj = self.proj[co]
        with self._t("comp_gemm"):
            self._gemm_bf16(self.u, L.comp_wkvg, proj, T, f32_out=True, m_valid=width)
        g = self.m_groups[r]
        cos, sin = self.rope["yarn"]
        # grid covers every token that could close a group; the kernel reads the real count
        max_groups = m.max_groups(r)
        if max_groups:
            with self._t("comp_pool"):
                ext.compress_pool(max_groups, self.m_ngroups[r], g[0], g[1], g[2], g[3], r, co, proj, L.comp_ape,
                                  self.comp_ring[lid], L.comp_norm, cfg.rms_norm_eps, cos, sin, self.comp[lid],
                                  L.idx_wk, L.idx_knorm, self.idx_cache.get(lid) if L.idx_wk is not None else None,
                                  self._pages(lid))
        if self._defer:
            self._pending("proj", lid, proj, T)
        else:
            with self._t("comp_ring"):
                ext.ring_update(self.comp_ring[lid], proj, T, self.m_slot, self.m_pos, self.m_last)

    def _indexer(self, L: LayerW, m: StepMeta, r: int):
        cfg, ext = self.cfg, self.ext
        T = m.T
        lid = L.layer_id
        nih, hd = cfg.index_n_heads, cfg.index_head_dim
        with self._t("idx_gemm"):
            self._gemm(self.qr_q, self.qr_sf, T, L.idx_wq_b, self.qidx.view(self.qidx.shape[0], -1))
            self._gemm_bf16(self.u, L.idx_wproj, self.widx_raw, T, f32_out=True)
        cos, sin = self.rope["yarn"]
        with self._t("idx_q_prep"):
            ext.idx_q_prep(self.qidx, T, nih, hd, cos, sin, self.m_pos, self.widx_raw,
                           (hd ** -0.5) * (nih ** -0.5), self.widx)
        # widx_raw rows are 128 wide; idx_q_prep reads [T, nih] with row stride nih
        src = self._k_source(lid)
        cand_mode = 0
        if lid == cfg.candidate_source_layer_id:
            cand_mode = 1
        elif 0 <= cfg.candidate_source_layer_id < lid:
            cand_mode = 2
        alt = self._k_alt(lid)
        tk = self._t("idx_topk")
        tk.__enter__()
        ext.indexer_topk(self.qidx, self.widx, self.idx_cache[src], self.m_slot, self.m_clen[r], cfg.index_topk,
                         self.comp_idx, self.comp_cnt, self.cand if cand_mode else None, cand_mode,
                         cfg.candidate_block_size, cfg.candidate_topk_blocks, T, self.err,
                         self.idx_cache[alt] if alt is not None else None, self.m_pos, self.m_cstart, self.m_last, r,
                         self.idx_keys, self._pages(src), self._pages(alt) if alt is not None else None)
        tk.__exit__(None, None, None)

    def _k_alt(self, lid: int) -> int | None:
        """K cache read by tokens that do not close a group at ``lid`` this step.

        With ``index_k_mode == "reference"`` the indexer reads the K cache of the
        most recent K producer (reference.py:645-654).  A layer that owns K only
        produces it on positions closing a group; for the other positions the
        most recent producer is the last ratio-1 K owner (it produces every
        position).  Returns None when every token reads the layer's own cache.
        """
        cfg = self.cfg
        if cfg.index_k_mode != "reference" or lid not in cfg.kv_source_layer_ids or cfg.ratio(lid) == 1:
            return None
        r1 = [s for s in self.idx_cache if cfg.ratio(s) == 1]
        if not r1:
            raise NotImplementedError("reference index_k_mode needs a ratio-1 K owner; use index_k_mode='intended'")
        return max(r1)

    def _k_source(self, lid: int) -> int:
        cfg = self.cfg
        src = cfg.kv_source_for(lid)
        # layers that own an indexer but no K projection read the newest K producer
        while src not in self.idx_cache:
            cands = [s for s in self.idx_cache if s <= lid]
            src = max(cands)
        return src

    # ------------------------------------------------------------------- MoE
    def _moe(self, L: LayerW, T: int):
        cfg, ext = self.cfg, self.ext
        lid = L.layer_id
        E = cfg.n_experts_for(lid)
        k = cfg.topk_for(lid)
        D = cfg.dim
        I = L.experts.inter
        logits = self.router_logits[E]
        rctx = self._t("router")
        rctx.__enter__()
        ids, wts, pos, rank = self.route[k]
        sfn = 1 if cfg.score_func == "sigmoid" else 0
        fused = self.ep is not None and self.ep.transport == "fused"
        if T <= ROUTER_SMALL_T and not fused:
            # decode-sized steps: gate GEMV and top-k in one launch
            ext.router_small(self.u, L.gate_w, T, logits, L.gate_b, k, sfn, cfg.route_scale, ids, wts,
                             self.router_counter)
        else:
            self._gemm_bf16(self.u, L.gate_w, logits, T, f32_out=True)
        if fused:
            # (also at world size 1: the same kernels with this GPU as the only peer)
            rctx.__exit__(None, None, None)
            # top-k, dispatch, plan, grouped GEMMs and the return of the rows (parallel/ep.py)
            return self.ep.moe_fused(self, L, T, k, logits)
        if T > ROUTER_SMALL_T:
            ext.router_topk(logits, T, L.gate_b, k, sfn, cfg.route_scale, ids, wts)
        rctx.__exit__(None, None, None)
        if self.ep is not None and self.ep.world > 1:
            return self.ep.moe(self, L, T, k) + (None,)
        e_begin, e_local = (0, E) if self.tp is None else self.tp.expert_range(E)
        pctx = self._t("moe_plan_scatter")
        pctx.__enter__()
        merged = self.merge_shared and L.shared_w13 is not None
        s_rows, s_row0 = (T, self.shared_row0) if merged else (0, 0)
        ext.moe_plan(T, k, e_local, e_begin, ids, wts, self.counts, self.seg, rank, self.tile_rows, 2 * I, D,
                     self.tiles13, self.nt13, self.tiles2, self.nt2, self.cap, pos, self.row_scale, self.err,
                     None, 0, s_rows, s_row0)
        ext.moe_scatter(self.uq, self.usf, T, k, pos, self.xperm, self.xperm_sf, s_row0 if merged else -1)
        pctx.__exit__(None, None, None)
        self._grouped(L, k, shared=merged)
        if merged:
            self.shared_y = self.yperm[self.shared_row0:self.shared_row0 + T]
        else:
            with self._t("shared_expert"):
                self._shared_expert(L, T)
            self.shared_y = self.shared_out
        if self.tp is not None:
            # the next mHC boundary reads every pair's row from the rank owning its expert
            # (expert ownership) or sums every rank's partial row of each pair (expert split)
            return None, pos, k, self.tp.moe_desc(ids, e_local)
        return self.yperm, pos, k, None

    def _shared_expert(self, L: LayerW, T: int):
        cfg = self.cfg
        self._gemm(self.uq, self.usf, T, L.shared_w13, None, EPI_SWIGLU, hq=self.hs, hsf=self.hs_sf,
                   swiglu_limit=cfg.swiglu_limit)
        self._gemm(self.hs, self.hs_sf, T, L.shared_w2, self.shared_out)

    def _grouped(self, L: LayerW, k: int, shared: bool = False):
        """Grouped expert GEMMs over the permuted rows; ``shared``: the tile lists also
        hold the shared expert's tiles (second weight operand)."""
        cfg, ext = self.cfg, self.ext
        I, D = L.experts.inter, cfg.dim
        ex = L.experts
        bn = self.tile_rows
        rows = self.perm_rows
        a13 = (L.shared_w13.q, L.shared_w13.sf) if shared else (None, None)
        a2 = (L.shared_w2.q, L.shared_w2.sf) if shared else (None, None)
        c13 = self._t("grouped_w13")
        c13.__enter__()
        ext.gemm_a2(ex.w13.kind, EPI_SWIGLU, ex.w13.q, ex.w13.sf, self.xperm, self.xperm_sf, None, ex.w13.q.shape[0],
                    rows, D, bn, 1, self.tiles13, self.nt13, self.row_scale, self.hperm, self.hperm_sf,
                    cfg.swiglu_limit, 2 * I, 0, None, None, self.err, 0, 1, None, None, None, *a13)
        c13.__exit__(None, None, None)
        c2 = self._t("grouped_w2")
        c2.__enter__()
        split = self.tp is not None and self.tp.moe == "tp"   # f32 partial rows, summed over ranks
        ext.gemm_a2(ex.w2.kind, EPI_F32 if split else EPI_BF16, ex.w2.q, ex.w2.sf, self.hperm, self.hperm_sf,
                    self.yperm, ex.w2.q.shape[0], rows, I, bn, 1, self.tiles2, self.nt2, None, None, None, 0.0, D, D,
                    None, None, self.err, 0, 1, self.tp.sync(1) if self.tp is not None else None, None, None, *a2)
        c2.__exit__(None, None, None)
