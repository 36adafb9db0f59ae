// Host launchers and parameter blocks of the fused kernels (one .cu file each).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "peer.h"

namespace dsv4 {

// Cache row records.  The attention caches hold each row in the quantized form
// of the round trip it went through.  KV8 (window rows): d e4m3 codes, then
// d/32 ue8m0 scale bytes.  KV4 (compressed rows): d/2 bytes of e2m1 codes
// (column 2i in the low nibble of byte i, 2i+1 in the high nibble), then d/16
// e4m3 scale bytes.  IK4 (indexer keys): the same packed e2m1 codes, then d/32
// ue8m0 scale bytes.  All decode exactly to the bf16 values of the round trip
// (at most 6 significant bits).
__host__ __device__ constexpr int kv8_bytes(int d) { return d + d / 32; }
__host__ __device__ constexpr int kv4_bytes(int d) { return d / 2 + d / 16; }
__host__ __device__ constexpr int ik4_bytes(int d) { return d / 2 + d / 32; }

// Grouped-GEMM tile records {a_row0, b_row0, valid, out_col0}: a_row0 with this
// bit set reads the GEMM's second weight operand (the shared expert riding in
// the routed experts' tile list).
constexpr int kTileA2 = 1 << 30;

// Block table of a paged compressed cache: entry ci of sequence slot s lives in
// pool row table[s * ld + (ci >> shift)] << shift | (ci & (2^shift - 1)).
// table == nullptr: contiguous per-slot cache, row s * max_c + ci.
struct KvPages {
  const int* table;
  int ld;
  int shift;
};

// ------------------------------------------------------------ misc.cu (debug bounds)
// Points every translation unit's debug-bounds error pointer at `err` (current
// device).  Returns the number of units set (0 in the default build, which has
// no checks), or -cudaError on failure.
int dbg_bounds_attach(uint32_t* err);
int dbg_bounds_units();   // translation units with index checks (0 in the default build)

// ------------------------------------------------------------ quant.cu
cudaError_t act_quant_mx(const __nv_bfloat16* x, int ldx, int T, int K, uint8_t* q, int ldq, uint8_t* sf,
                         int k_tiles, cudaStream_t st);
cudaError_t act_roundtrip(const __nv_bfloat16* x, __nv_bfloat16* y, long long n, cudaStream_t st);
cudaError_t fp4_roundtrip(const __nv_bfloat16* x, __nv_bfloat16* y, long long n, int block, int e4m3_scale,
                          cudaStream_t st);

// -------------------------------------------------------------- mhc.cu
struct HcParams {
  int T, D;
  __nv_bfloat16* X;                 // [T, 4, D] residual streams (updated in place)
  const __nv_bfloat16* Y;           // sublayer output [T, D] (or the shared-expert term with yperm)
  const __nv_bfloat16* yperm;       // MoE: expert outputs in permuted-row order [R, D]
  const int* pos;                   // MoE: [T, topk] permuted row per slot (-1 = none)
  int topk;
  const float* prev_mix;            // [T, 24] (pre | post | comb) of the previous boundary
  const __nv_bfloat16* fn_hilo;     // [128, 4D] bf16 hi rows 0..23, lo rows 24..47 of hc_fn (null = no mixes)
  const float* scale;               // [3]
  const float* base;                // [24]
  const float* cw;                  // collapse weights: cw[t * cw_stride + i]
  int cw_stride;
  const __nv_bfloat16* norm_w;      // [D]
  float* mix_out;                   // [T, 24]
  __nv_bfloat16* c;                 // scratch [T, D]
  float* partials;                  // scratch [T, n_slices, 50]
  __nv_bfloat16* u;                 // [T, D] normalized collapse
  uint8_t* uq;                      // [T_pad, D] e4m3 (optional)
  uint8_t* usf;                     // scale chunks of uq
  __nv_bfloat16* tap;               // optional [T, D] mean of the updated streams
  int iters;
  float hc_eps, norm_eps;
  // tensor parallel (hc_post): tp_mode 1 = the sublayer output is the rank-order
  // sum of every rank's f32 partial (peer_y, rows D apart); tp_mode 2 = each
  // (token, slot) pair's expert row is read from the rank owning its expert
  // (peer_yperm / peer_pos; ids are identical on every rank); tp_mode 3 = experts
  // split by intermediate index: every rank's f32 partial row of each pair
  // (peer_y tables, at row peer_pos[rank][t, slot] of that rank's own plan)
  // summed in rank order; tp_mode 4 = expert parallelism with rows returned by
  // the owners' W2 epilogues: the local yperm / pos combine once every rank has
  // published the phase.  All wait first
  // (bounded) until every rank has published the phase.
  int tp_mode;
  const float* const* peer_y;
  const __nv_bfloat16* const* peer_yperm;
  const int* const* peer_pos;
  const int* ids;
  int e_local;
  PeerSync wait;
  uint32_t* err;
};
int hc_num_slices(int D);
cudaError_t hc_post(const HcParams& p, cudaStream_t st);
cudaError_t hc_finish(const HcParams& p, cudaStream_t st);

// -------------------------------------------------------- attention.cu
constexpr int kAttnMaxRows = 768;   // window (<= 256) + selected compressed rows
struct AttnParams {
  int T;
  const __nv_bfloat16* q;           // [T, n_heads, 512] rows q_stride apart
  int q_stride;
  int n_heads;                      // <= 64 (tensor parallel: this rank's heads; the rest of the
                                    // 64-head tile computes on zero queries and is not stored)
  int out_stride;
  const float* rope_cos;            // [positions, 32]
  const float* rope_sin;
  const int* rope_pos;              // optional rope position (default pos)
  int q_head_norm;
  float norm_eps;
  const uint8_t* kv_step;           // this step's window rows [R, 528] (KV8 records)
  const uint8_t* ring;              // [slots, W, 528] KV8 records
  int W;
  const uint8_t* comp;              // [slots, max_c, 288] KV4 records or a paged pool, or null
  int max_c;
  KvPages comp_pages;
  const int* slot;
  const int* pos;
  const int* chunk_start;           // first position of this step for the token's sequence
  const int* step_row0;             // kv_step row holding chunk_start
  const int* comp_idx;              // [T, comp_k] selected compressed rows (null = dense 0..cnt)
  int comp_k;
  const int* comp_cnt;              // [T] number of valid compressed rows
  const int* win_end;               // optional last window position per token (default pos): a
                                    // draft block attends to all of its rows (bidirectional)
  int win_len;                      // window rows (default W)
  const float* sink;                // [n_heads]
  float scale;
  __nv_bfloat16* out;               // [T, n_heads, 512] rows out_stride apart
  float* workspace;                 // split partials
};
size_t attn_smem_bytes();
cudaError_t attention(const AttnParams& p, int nsplit, cudaStream_t st);

// -------------------------------------------------------- norm_rope.cu
struct QkvParams {
  int T, q_dim, kv_dim;
  const __nv_bfloat16* in;          // [T, q_dim + kv_dim] fused wq_a|wkv output
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* kv_norm_w;
  float eps;
  uint8_t* qr_q;                    // [T_pad, q_dim] e4m3
  uint8_t* qr_sf;
  const float* rope_cos;
  const float* rope_sin;
  const int* pos;
  uint8_t* kv_out;                  // [T, kv8_bytes(kv_dim)] KV8 records
};
cudaError_t qkv_post(const QkvParams& p, cudaStream_t st);

// Indexer query: per head RoPE on the last 64 dims + e2m1 round trip (block 32,
// ue8m0); weights: bf16(w * scale).
cudaError_t idx_q_prep(__nv_bfloat16* q, int T, int n_heads, int head_dim, const float* cos, const float* sin,
                       const int* pos, const float* w_in, float w_scale, float* w_out, cudaStream_t st);

// -------------------------------------------------------- compressor.cu
struct CompParams {
  int n_groups;                     // grid size (upper bound)
  const int* n_groups_dev;          // actual number of closed groups (device)
  const int* g_slot;
  const int* g_index;               // compressed entry index g (closes at position g*r + r - 1)
  const int* g_chunk_start;         // first position of this step for the group's sequence
  const int* g_row0;                // proj_step row of g_chunk_start
  int r, co, dh;
  const float* proj;                // [T, 2*co*dh] (kv | score) this step
  const float* ape;                 // [r, co*dh] or null
  const float* ring;                // [slots, co*r, 2*co*dh]
  const __nv_bfloat16* norm_w;
  float eps;
  const float* rope_cos;
  const float* rope_sin;
  uint8_t* comp_out;                // [slots, max_c, kv4_bytes(dh)] KV4 records or a paged pool (pages)
  int max_c;
  KvPages pages;                    // rows of comp_out and idx_out
  const __nv_bfloat16* wk;          // indexer K projection [idx_dim, dh] (null = none)
  const __nv_bfloat16* k_norm_w;
  uint8_t* idx_out;                 // [slots, max_c, ik4_bytes(idx_dim)] IK4 records
  int idx_dim;
};
cudaError_t compress_pool(const CompParams& p, cudaStream_t st);
// ring[slot][pos % depth] = proj[row] for tokens whose position is among the
// last ``depth`` positions of their sequence in this step.
cudaError_t ring_update_f32(float* ring, int depth, int width, const float* src, int T, const int* slot,
                            const int* pos, const int* last_pos, cudaStream_t st);
cudaError_t ring_update_bf16(__nv_bfloat16* ring, int depth, int width, const __nv_bfloat16* src, int T,
                             const int* slot, const int* pos, const int* last_pos, cudaStream_t st);
cudaError_t ring_update_rec(uint8_t* ring, int depth, int width, const uint8_t* src, int T, const int* slot,
                            const int* pos, const int* last_pos, cudaStream_t st);

// ------------------------------------------------------------ moe.cu
// Router GEMV + top-k in one launch for T <= kRouterSmallMaxT tokens; counter: one
// zeroed device int (the kernel leaves it zero).
constexpr int kRouterSmallMaxT = 4;
struct RouterSmallParams {
  const __nv_bfloat16* u;           // [T, D] normalized activations
  const __nv_bfloat16* w;           // [E, D] gate weights
  int T, D, E;
  float* logits;                    // [T, E] out
  const float* bias;
  int topk, score_func;
  float route_scale;
  int* ids;
  float* wts;
  int* counter;
};
cudaError_t router_small(const RouterSmallParams& p, cudaStream_t st);
cudaError_t router_topk(const float* logits, int T, int E, const float* bias, int topk, int score_func,
                        float route_scale, int* ids, float* wts, cudaStream_t st);
struct MoePlanParams {
  int T, topk, E_local, e_begin;    // experts [e_begin, e_begin + E_local) live here
  const int* ids;                   // [T, topk] global expert ids
  const float* wts;
  int* counts;                      // [E_local] scratch (zeroed by the plan)
  int* seg_start;                   // [E_local]
  int* rank;                        // [T, topk] scratch
  int tile_rows;                    // token rows per GEMM tile: 32, 64 (one 128-row slot each), 128 or 256
  int m13, m2;                      // W13 / W2 output rows per expert
  int4* tiles13;
  int* n_tiles13;
  int4* tiles2;
  int* n_tiles2;
  int max_tiles13, max_tiles2;
  int cap_rows;                     // capacity of the permuted buffers
  int* pos;                         // [T, topk] permuted row (-1 if the expert is not local)
  float* row_scale;                 // [cap_rows]
  uint32_t* err;
  // optional: the T*topk entries are segments of seg_cap slots of which the
  // first seg_cnt[s] are valid (expert-parallel receive buffers); others are skipped
  const int* seg_cnt;
  int seg_cap;
  // optional: shared_rows > 0 appends the shared expert's tiles (flagged
  // kTileA2) for rows [shared_row0, shared_row0 + shared_rows) of the permuted
  // buffers (token t at row shared_row0 + t, row_scale 1); tile_rows >= 128
  int shared_rows, shared_row0;
  int rs_rows;                      // rows of row_scale (the debug-bounds build checks every write)
};
cudaError_t moe_plan(const MoePlanParams& p, cudaStream_t st);
// Copies quantized token rows (e4m3 + scale chunks) into permuted-row order;
// shared_row0 >= 0 also copies token t to row shared_row0 + t.
cudaError_t moe_scatter(const uint8_t* xq, const uint8_t* xsf, int T, int D, int topk, const int* pos, uint8_t* pq,
                        uint8_t* psf, int shared_row0, int pq_rows, cudaStream_t st);

// ----------------------------------------------------------- indexer.cu
struct IdxParams {
  int T, n_heads, head_dim;
  const __nv_bfloat16* q;           // [T, n_heads, head_dim]
  const float* w;                   // [T, n_heads] (already bf16-rounded)
  const uint8_t* kcache;            // [slots, max_c, ik4_bytes(head_dim)] IK4 records or a paged pool
  int max_c;
  KvPages pages;
  const int* slot;
  const int* clen;                  // [T] causal number of compressed entries
  int topk;
  int* out_idx;                     // [T, topk]
  int* out_cnt;                     // [T]
  uint8_t* cand;                    // [T, max_c/cand_block] candidate block mask (optional)
  int cand_mode;                    // 0 none, 1 build, 2 apply
  int cand_block, cand_topk;
  uint32_t* err;
  // tokens whose position does not close a group of ratio own_r read kcache_alt
  const uint8_t* kcache_alt;
  int alt_max_c;
  KvPages alt_pages;
  const int* pos;
  const int* chunk_start;           // alt only applies to single-token (decode) chunks
  const int* last_pos;
  int own_r;
};
// keys: [T, keys_ld] uint32 scratch (keys_ld >= max_c) for the order keys of the scores
cudaError_t indexer_topk(const IdxParams& p, uint32_t* keys, int keys_ld, cudaStream_t st);

// ---------------------------------------------------------------- ep.cu
// Completion signalling of the NVLink (peer-store) transport; all null for the
// NCCL transport.
struct EpSync {
  uint32_t* const* peer_sig;   // [world] each rank's signal array (uint32 [2 * world])
  int* const* peer_cnt;        // [world] each rank's receive-count array (dispatch only)
  int* done;                   // this rank's CTA completion counter for the phase
  uint32_t* epoch;             // this rank's epoch counter for the phase
  int phase;                   // 0 dispatch, 1 combine
};
cudaError_t ep_wait(const uint32_t* sig, int world, int phase, const uint32_t* epoch, uint32_t* err,
                    cudaStream_t st);
cudaError_t ep_pack(const int* ids, const float* wts, int T, int topk, const uint8_t* xq, const uint8_t* xsf, int D,
                    int e_local, int world, int cap, int rec, uint8_t* send, int* cnt, int* pos_back,
                    uint8_t* const* peer_recv, int my_rank, uint32_t* err, const EpSync& sync, cudaStream_t st);
cudaError_t ep_unpack_meta(const uint8_t* recv, const int* cnt, int world, int cap, int rec, int D, int* ids,
                           float* wts, cudaStream_t st);
// cnt: received records per peer (slot p * cap + j is valid for j < cnt[p])
cudaError_t ep_unpack_rows(const uint8_t* recv, const int* cnt, int world, int cap, int rec, int D, const int* pos,
                           uint8_t* pq, uint8_t* psf, cudaStream_t st);
cudaError_t ep_combine_pack(const __nv_bfloat16* yperm, const int* pos, const int* cnt, int D, int cap,
                            __nv_bfloat16* back, __nv_bfloat16* const* peer_back, int my_rank, int world,
                            const EpSync& sync, cudaStream_t st);

// Fused expert-parallel path (ep.cu): router top-k + direct stores into the
// owners' expert rows, then a one-CTA plan that waits for every rank.
struct EpDispatchParams {
  const float* logits;        // [T, E] router logits (fp32)
  const float* bias;          // [E] selection bias (optional)
  int T, E, topk, score_func;
  float route_scale;
  int* ids;                   // optional local copy of the routing [T, topk]
  float* wts;
  const uint8_t* xq;          // [>= T, D] e4m3 token rows
  const uint8_t* xsf;         // their scale chunks
  int D, e_local, cap_e, world, rank;
  int tile_rows;              // GEMM tile rows (the row layout of an expert segment, seg_row)
  int rows;                   // expert rows of every rank (e_local * cap_e), for the debug-bounds build
  int ret_rows;               // return rows of every rank (max tokens * topk), for the debug-bounds build
  uint8_t* const* peer_x;     // [world] expert rows [e_local * cap_e, D] of each rank
  uint8_t* const* peer_xsf;   // [world] their scale chunks
  float* const* peer_rscale;  // [world] routing weight per expert row
  int* const* peer_meta;      // [world] (source rank << 24) | pair index per expert row
  int* const* peer_cnt;       // [world] rows claimed per local expert (zero at rest)
  uint32_t* err;
  PeerSync pub;               // phase 0
  int shared_row0;            // >= 0: each token row is also stored at this rank's expert row
                              // shared_row0 + t (the shared expert's input segment)
};
cudaError_t ep_dispatch(const EpDispatchParams& p, cudaStream_t st);

struct EpPlanParams {
  PeerSync wait;              // phase 0
  int* cnt;                   // this rank's counters [e_local]
  int e_local, cap_e, tile_rows, m13, m2;
  int4* tiles13;
  int* n_tiles13;
  int4* tiles2;
  int* n_tiles2;
  int max_tiles13, max_tiles2;
  uint32_t* err;
  // shared_rows > 0: the shared expert's tiles (kTileA2) for this rank's rows
  // [shared_row0, shared_row0 + shared_rows) follow the routed tiles
  int shared_rows, shared_row0;
};
cudaError_t ep_plan(const EpPlanParams& p, cudaStream_t st);

// ------------------------------------------------------------ engram.cu
constexpr int kEngramMaxLayers = 4;
struct EngramParams {
  int T, nl, N, H, hd;              // tokens, Engram layers, max n-gram, heads per order, row bytes
  const int* ids;                   // [T] this step's token ids
  const int* pos;
  const int* slot;
  const int* chunk_start;
  const int* step_row0;
  const int* last_pos;
  const int64_t* token_map;         // [vocab] compressed id (-1 = dead token)
  int64_t* ring;                    // [slots, N-1] compressed ids by position % (N-1)
  const int64_t* mult;              // [nl, N]
  const int64_t* primes;            // [nl, N-1, H]
  const int64_t* offsets;           // [nl, (N-1)*H]
  int64_t pad;                      // compressed pad id
  int64_t* rows;                    // [T, nl, (N-1)*H] row ids (out)
  const uint8_t* table[kEngramMaxLayers];     // device-mapped host tables [n_emb, hd] e4m3
  const uint8_t* table_sf[kEngramMaxLayers];  // [n_emb, hd/32] ue8m0
  int64_t n_emb[kEngramMaxLayers];
  uint8_t* a_q;                     // [nl] x [T_pad, K] e4m3 (K = (N-1)*H*hd)
  uint8_t* a_sf;                    // [nl] x scale chunks
  size_t a_stride_q, a_stride_sf;   // per-layer strides (bytes)
};
cudaError_t engram_prepare(const EngramParams& p, int mode, cudaStream_t st);   // bits: 1 hash, 2 ring, 4 gather
cudaError_t engram_gate(__nv_bfloat16* X, const __nv_bfloat16* kv, const float* wgt, int T, int D, int hc, float eps,
                        cudaStream_t st);

// -------------------------------------------------------------- misc.cu
cudaError_t embed_streams(const __nv_bfloat16* table, const int* ids, int T, int D, int hc, __nv_bfloat16* X,
                          cudaStream_t st);
// ws_v/ws_i: >= max(T, 296) entries; counters: >= T ints, zero (left zero); all null = one CTA per row
int argmax_splits(int T);
// out_val (optional) receives the best value; idx_base is added to every index
cudaError_t argmax_rows(const float* logits, int T, int V, int ld, int* out, float* ws_v, int* ws_i, int* counters,
                        float* out_val, int idx_base, cudaStream_t st);
// stamps: [1 + 2 * ctas] u64 (see misc.cu)
cudaError_t pdl_probe(unsigned long long* stamps, int ctas, unsigned long long ns, cudaStream_t st);
cudaError_t ts_mark(unsigned long long* ring, int slot, cudaStream_t st);
cudaError_t tp_argmax_merge(const PeerSync& s, const float* const* peer_val, const int* const* peer_idx, int T,
                            int* out, uint32_t* err, cudaStream_t st);
cudaError_t markov_step(const float* logits, int ld, int blk, int i, const float* mlog, int mld, int V, int n,
                        int* toks, int ts, const __nv_bfloat16* memb, int R, __nv_bfloat16* emb, cudaStream_t st);

}  // namespace dsv4
