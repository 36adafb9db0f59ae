// Python bindings of the sm_100a kernels.  Every entry point checks device,
// dtype and layout, then launches on the current CUDA stream; nothing here
// allocates device memory (callers own all buffers).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "gemm.h"
#include "kernels.h"

#include <algorithm>
#include <cstdlib>

namespace {

using at::Tensor;
using c10::optional;

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CUDA_OK(expr)                                                                \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    TORCH_CHECK(_e == cudaSuccess, #expr " failed: ", cudaGetErrorString(_e));       \
  } while (0)

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

const uint8_t* u8ptr(const optional<Tensor>& t) { return t ? t->data_ptr<uint8_t>() : nullptr; }

int tma_elem_of(const Tensor& t, bool e2m1) {
  if (e2m1) return dsv4::TMA_E2M1;
  if (t.scalar_type() == at::kBFloat16) return dsv4::TMA_BF16;
  return dsv4::TMA_U8;
}

// Generic tcgen05 GEMM entry.
//   kind 0: bf16 x bf16; 1: e4m3 x e4m3 (MXFP8); 2: e2m1 (A) x e4m3 (B).
//   A [a_rows, K] (packed e2m1: [a_rows, K/2]); B [b_rows, K].
//   grouped: tiles int32 [n, 4] + n_tiles int32 [1] device tensors.
// Optional int64 CPU tensor [block table address, ld, shift, logical max_c] of a
// paged compressed cache -> KvPages; the logical per-slot capacity replaces the
// pool tensor's size(1).  None = contiguous per-slot cache.
static dsv4::KvPages kv_pages_of(const optional<Tensor>& d, int* max_c) {
  dsv4::KvPages pg{};
  if (!d) return pg;
  TORCH_CHECK(!d->is_cuda() && d->scalar_type() == at::kLong && d->numel() >= 4, "pages: int64 CPU [4]");
  const int64_t* v = d->data_ptr<int64_t>();
  pg.table = reinterpret_cast<const int*>(v[0]);
  pg.ld = (int)v[1];
  pg.shift = (int)v[2];
  *max_c = (int)v[3];
  TORCH_CHECK(pg.table != nullptr && pg.ld > 0 && pg.shift >= 0 && pg.shift < 16 && *max_c > 0 &&
              ((int64_t)pg.ld << pg.shift) >= *max_c, "bad page descriptor");
  return pg;
}

// DSV4_GEMM_BM256=0 keeps every GEMM on 128-row weight tiles (A/B timing).
static bool bm256_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("DSV4_GEMM_BM256");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

// Optional int64 CPU tensor [peer_sig table, sig, done, epoch, phase, world, rank] of device
// addresses / values -> PeerSync (all zero = none)
static dsv4::PeerSync peer_sync_of(const optional<Tensor>& t) {
  dsv4::PeerSync s{};
  if (!t) return s;
  TORCH_CHECK(!t->is_cuda() && t->scalar_type() == at::kLong && t->numel() >= 7, "peer sync: int64 CPU [7]");
  const int64_t* v = t->data_ptr<int64_t>();
  s.peer_sig = reinterpret_cast<uint32_t* const*>(v[0]);
  s.sig = reinterpret_cast<const uint32_t*>(v[1]);
  s.done = reinterpret_cast<int*>(v[2]);
  s.epoch = reinterpret_cast<uint32_t*>(v[3]);
  s.phase = (int)v[4];
  s.world = (int)v[5];
  s.rank = (int)v[6];
  return s;
}

// A2 / A2_sf (grouped GEMMs, optional): a second weight matrix of the same K and
// kind; tile records whose a_row0 carries kTileA2 read it (the shared expert in
// the routed experts' tile list).
void gemm_a2(int64_t kind, int64_t epi, const Tensor& A, const optional<Tensor>& A_sf, const Tensor& B,
             const optional<Tensor>& B_sf, const optional<Tensor>& out, int64_t M, int64_t N, int64_t K, int64_t bn,
             int64_t splits, const optional<Tensor>& tiles, const optional<Tensor>& n_tiles,
             const optional<Tensor>& row_scale, const optional<Tensor>& hq, const optional<Tensor>& hsf,
             double swiglu_limit, int64_t m_valid, int64_t ldo, const optional<Tensor>& workspace,
             const optional<Tensor>& counters, const Tensor& err, int64_t max_grid, int64_t groups,
             const optional<Tensor>& publish, const optional<Tensor>& ret_meta, const optional<Tensor>& ret_peer,
             const optional<Tensor>& A2, const optional<Tensor>& A2_sf) {
  CHECK_CUDA(A);
  CHECK_CUDA(B);
  CHECK_CONTIG(A);
  CHECK_CONTIG(B);
  TORCH_CHECK(K % 128 == 0, "K must be a multiple of 128");
  const bool grouped = tiles.has_value();
  const bool e2m1 = kind == dsv4::KIND_MX4A;
  const c10::cuda::CUDAGuard guard(A.device());
  const int64_t b_cols = B.size(1);  // full activation width (groups * K in batched mode)
  TORCH_CHECK(b_cols == K * std::max<int64_t>(1, groups), "B width must be groups * K");
  // 256-row weight tiles: two M=128 MMAs per stage share the token tile.  Measured
  // faster only without split-K on long K with enough tiles to fill the GPU (e.g.
  // wo_b at 1023 tokens: 53 vs 61 us); with split-K the cluster reduction doubles
  // and the single accumulator serializes the epilogue, so those stay at 128 rows.
  const bool caller_ws = workspace.has_value() && counters.has_value();
  const int k_tiles_mx = (int)(K / 128);
  const int tiles256 = (int)(M / 256) * (int)((N + bn - 1) / bn);
  const int bm = (kind != dsv4::KIND_BF16 && !grouped && groups <= 1 && epi != dsv4::EPI_SWIGLU && M % 256 == 0 &&
                  (bn == 64 || bn == 128) && !caller_ws && splits <= 1 && k_tiles_mx >= 64 && tiles256 >= 96 &&
                  bm256_enabled())
                     ? 256 : 128;
  dsv4::AMaps ta{};
  dsv4::BMaps tb;
  TORCH_CHECK(dsv4::make_tma_2d(&ta.m[0], A.data_ptr(), tma_elem_of(A, e2m1), A.size(0), K, (uint32_t)bm),
              "TMA(A) encode failed");
  // MXFP4 weights (A packed [rows, K/2]) may take an MXFP8 second operand ([rows, K])
  const bool a2_e4m3 = A2 && e2m1 && A2->size(1) == K;
  if (A2) {
    TORCH_CHECK(grouped && bm == 128 && A2->is_cuda() && A2->is_contiguous() && A2->dim() == 2 && A2->size(0) % 128 == 0,
                "A2: grouped GEMMs only, [rows (multiple of 128), K] contiguous");
    TORCH_CHECK(A2->scalar_type() == A.scalar_type() && (A2->size(1) == A.size(1) || a2_e4m3),
                "A2 must match A's type and K (or be MXFP8 beside MXFP4 weights)");
    TORCH_CHECK(kind == dsv4::KIND_BF16 || A2_sf.has_value(), "block-scaled A2 needs A2_sf");
    TORCH_CHECK(dsv4::make_tma_2d(&ta.m[1], A2->data_ptr(), tma_elem_of(*A2, e2m1 && !a2_e4m3), A2->size(0), K,
                                  (uint32_t)bm),
                "TMA(A2) encode failed");
  }
  if (grouped) {
    const uint32_t boxes[4] = {32, 64, 128, 256};
    for (int i = 0; i < 4; ++i)
      TORCH_CHECK(dsv4::make_tma_2d(&tb.m[i], B.data_ptr(), tma_elem_of(B, false), B.size(0), b_cols, boxes[i]),
                  "TMA(B) encode failed");
  } else {
    TORCH_CHECK(dsv4::make_tma_2d(&tb.m[0], B.data_ptr(), tma_elem_of(B, false), B.size(0), b_cols, (uint32_t)bn),
                "TMA(B) encode failed");
    TORCH_CHECK(N <= bn || bn >= 128, "dense GEMM with several token tiles needs bn >= 128");
  }
  dsv4::GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  const int elem_bytes = kind == dsv4::KIND_BF16 ? 2 : 1;
  p.k_tiles = (int)(K * elem_bytes / 128);
  if (splits < 0 && !grouped) {
    // automatic: split K when the output tiles cannot fill the SMs (each split keeps
    // >= 2 k-tiles; at most 8 splits, one cluster per tile)
    const int tiles_auto = (int)(M / bm) * (int)((N + bn - 1) / bn);
    splits = tiles_auto < 100 ? std::max(1, std::min({8, p.k_tiles / 2, 148 / std::max(tiles_auto, 1)})) : 1;
  }
  p.splits = (int)std::max<int64_t>(1, splits);
  p.sfa = u8ptr(A_sf);
  p.sfa_ktiles = (int)(K / 128);
  p.sfa2 = A2 ? (A2_sf ? u8ptr(A2_sf) : reinterpret_cast<const uint8_t*>(A2->data_ptr())) : nullptr;
  p.M2 = A2 ? (int)A2->size(0) : 0;
  p.a2_e4m3 = a2_e4m3 ? 1 : 0;
  p.sfb = u8ptr(B_sf);
  p.sfb_ktiles = (int)(b_cols / 128);
  if (groups > 1) {
    TORCH_CHECK(!grouped && M % groups == 0 && (M / groups) % 128 == 0, "batched GEMM: M must split into groups");
    p.group_rows = (int)(M / groups);
    p.group_k = (int)K;
  } else {
    p.group_rows = 1 << 30;
    p.group_k = 0;
  }
  if (kind != dsv4::KIND_BF16) TORCH_CHECK(A_sf && B_sf, "block-scaled GEMM needs A_sf and B_sf");
  p.out = out ? out->data_ptr() : nullptr;
  p.ldo = (int)ldo;
  p.m_valid = (int)m_valid;
  p.row_scale = row_scale ? row_scale->data_ptr<float>() : nullptr;
  p.hq = hq ? hq->data_ptr<uint8_t>() : nullptr;
  p.ldh = hq ? (int)hq->size(1) : 0;
  p.hsf = hsf ? hsf->data_ptr<uint8_t>() : nullptr;
  p.h_ktiles = hq ? (int)(hq->size(1) / 128) : 0;
  p.swiglu_limit = (float)swiglu_limit;
  p.workspace = workspace ? workspace->data_ptr<float>() : nullptr;
  p.tile_counters = counters ? counters->data_ptr<int>() : nullptr;
  p.err = reinterpret_cast<uint32_t*>(err.data_ptr<int>());
  p.pub = peer_sync_of(publish);
  if (ret_meta || ret_peer) {
    TORCH_CHECK(ret_meta && ret_peer && grouped && epi == dsv4::EPI_BF16, "return rows: grouped bf16 GEMMs with both tables");
    TORCH_CHECK(ret_meta->is_cuda() && ret_meta->scalar_type() == at::kInt && ret_meta->numel() >= B.size(0),
                "ret_meta: int32 device [B rows]");
    TORCH_CHECK(ret_peer->is_cuda() && ret_peer->scalar_type() == at::kLong, "ret_peer: int64 device pointer table");
    TORCH_CHECK(M % 128 == 0 && m_valid % 128 == 0 && (ldo * 2) % 16 == 0,
                "return rows: whole 128-row tiles, 16-byte rows");
    p.ret_meta = ret_meta->data_ptr<int>();
    p.ret_peer = reinterpret_cast<__nv_bfloat16* const*>(ret_peer->data_ptr<int64_t>());
    p.ret_world = (int)ret_peer->numel();
  }
  if (p.splits > 1 && !(workspace && counters)) {
    // split-K through a thread-block cluster per tile (dense GEMMs, <= 8 splits).
    // Halve the split count until every tile's cluster is resident at once.
    TORCH_CHECK(!grouped, "cluster split-K: dense GEMMs only");
    TORCH_CHECK(M % 128 == 0, "M must be a multiple of 128");
    const int tiles = (int)(M / bm) * (int)((N + bn - 1) / bn);
    int s = 1;
    while (s * 2 <= std::min(p.splits, 8)) s *= 2;
    while (s >= 2 && dsv4::gemm_max_clusters((int)kind, (int)epi, (int)bn, s, bm) < tiles) s /= 2;
    p.splits = s >= 2 ? s : 1;
    p.cluster_split = p.splits > 1;
  }
  int units;
  if (grouped) {
    p.tiles = reinterpret_cast<const int4*>(tiles->data_ptr<int>());
    p.n_tiles_ptr = n_tiles->data_ptr<int>();
    units = (int)tiles->size(0) * p.splits;
  } else {
    TORCH_CHECK(M % 128 == 0, "M must be a multiple of 128");
    p.n_tiles = (int)(M / bm) * (int)((N + bn - 1) / bn);
    units = p.n_tiles * p.splits;
  }
  if (units == 0) {
    TORCH_CHECK(!publish, "a publishing GEMM must launch");
    return;
  }
  int grid = p.cluster_split ? units : std::min(units, max_grid > 0 ? (int)max_grid : num_sms());
  CUDA_OK(dsv4::gemm_launch((int)kind, (int)epi, grouped, (int)bn, bm, ta, tb, p, grid, cur_stream()));
}

void gemm(int64_t kind, int64_t epi, const Tensor& A, const optional<Tensor>& A_sf, const Tensor& B,
          const optional<Tensor>& B_sf, const optional<Tensor>& out, int64_t M, int64_t N, int64_t K, int64_t bn,
          int64_t splits, const optional<Tensor>& tiles, const optional<Tensor>& n_tiles,
          const optional<Tensor>& row_scale, const optional<Tensor>& hq, const optional<Tensor>& hsf,
          double swiglu_limit, int64_t m_valid, int64_t ldo, const optional<Tensor>& workspace,
          const optional<Tensor>& counters, const Tensor& err, int64_t max_grid, int64_t groups,
          const optional<Tensor>& publish, const optional<Tensor>& ret_meta, const optional<Tensor>& ret_peer) {
  gemm_a2(kind, epi, A, A_sf, B, B_sf, out, M, N, K, bn, splits, tiles, n_tiles, row_scale, hq, hsf, swiglu_limit,
          m_valid, ldo, workspace, counters, err, max_grid, groups, publish, ret_meta, ret_peer, c10::nullopt,
          c10::nullopt);
}

void act_quant_mx(const Tensor& x, Tensor& q, Tensor& sf) {
  CHECK_CUDA(x);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x: bf16 [T, K] row-major");
  const int T = (int)x.size(0), K = (int)x.size(1);
  TORCH_CHECK(K % 128 == 0, "K must be a multiple of 128");
  TORCH_CHECK(q.size(0) >= T && q.size(1) == K, "q shape");
  const c10::cuda::CUDAGuard guard(x.device());
  CUDA_OK(dsv4::act_quant_mx(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int)x.stride(0), T, K,
                             q.data_ptr<uint8_t>(), (int)q.stride(0), sf.data_ptr<uint8_t>(), K / 128,
                             cur_stream()));
}

void act_roundtrip(const Tensor& x, Tensor& y) {
  CHECK_CUDA(x);
  CHECK_CONTIG(x);
  CHECK_CONTIG(y);
  TORCH_CHECK(x.numel() % 32 == 0, "numel must be a multiple of 32");
  CUDA_OK(dsv4::act_roundtrip(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                              reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), x.numel(), cur_stream()));
}

void fp4_roundtrip(const Tensor& x, Tensor& y, int64_t block, bool e4m3_scale) {
  CHECK_CUDA(x);
  CHECK_CONTIG(x);
  CHECK_CONTIG(y);
  TORCH_CHECK(block == 16 || block == 32, "block 16 or 32");
  CUDA_OK(dsv4::fp4_roundtrip(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                              reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), x.numel(), (int)block, e4m3_scale,
                              cur_stream()));
}

int64_t gemm_smem(int64_t bn) { return dsv4::gemm_smem_bytes((int)bn); }

template <typename T>
T* ptr(const optional<Tensor>& t) {
  return t ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}
template <typename T>
T* ptr(const Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
using bf16 = __nv_bfloat16;

dsv4::HcParams hc_params(const Tensor& X, const optional<Tensor>& Y, const optional<Tensor>& yperm,
                         const optional<Tensor>& pos, int64_t topk, const optional<Tensor>& prev_mix,
                         const optional<Tensor>& fn_hilo, const optional<Tensor>& scale, const optional<Tensor>& base,
                         const optional<Tensor>& cw, int64_t cw_stride, const optional<Tensor>& norm_w,
                         const optional<Tensor>& mix_out, const Tensor& c, const Tensor& partials,
                         const optional<Tensor>& u, const optional<Tensor>& uq, const optional<Tensor>& usf,
                         const optional<Tensor>& tap, int64_t T, int64_t iters, double hc_eps, double norm_eps) {
  CHECK_CUDA(X);
  TORCH_CHECK(X.size(1) == 4, "hc_mult must be 4");
  dsv4::HcParams p{};
  p.T = (int)T;
  p.D = (int)X.size(2);
  TORCH_CHECK(p.D % 128 == 0, "D % 128");
  TORCH_CHECK(partials.numel() >= T * dsv4::hc_num_slices(p.D) * 50, "partials too small");
  p.X = ptr<bf16>(X);
  p.Y = ptr<const bf16>(Y);
  p.yperm = ptr<const bf16>(yperm);
  p.pos = ptr<const int>(pos);
  p.topk = (int)topk;
  p.prev_mix = ptr<const float>(prev_mix);
  p.fn_hilo = ptr<const bf16>(fn_hilo);
  p.scale = ptr<const float>(scale);
  p.base = ptr<const float>(base);
  p.cw = ptr<const float>(cw);
  p.cw_stride = (int)cw_stride;
  p.norm_w = ptr<const bf16>(norm_w);
  p.mix_out = ptr<float>(mix_out);
  p.c = ptr<bf16>(c);
  p.partials = ptr<float>(partials);
  p.u = ptr<bf16>(u);
  p.uq = ptr<uint8_t>(uq);
  p.usf = ptr<uint8_t>(usf);
  p.tap = ptr<bf16>(tap);
  p.iters = (int)iters;
  p.hc_eps = (float)hc_eps;
  p.norm_eps = (float)norm_eps;
  return p;
}

void hc_post(const Tensor& X, const optional<Tensor>& Y, const optional<Tensor>& yperm, const optional<Tensor>& pos,
             int64_t topk, const optional<Tensor>& prev_mix, const optional<Tensor>& fn_hilo,
             const optional<Tensor>& cw, int64_t cw_stride, const Tensor& c, const Tensor& partials,
             const optional<Tensor>& tap, int64_t T, const optional<Tensor>& tp, const optional<Tensor>& err) {
  auto p = hc_params(X, Y, yperm, pos, topk, prev_mix, fn_hilo, c10::nullopt, c10::nullopt, cw, cw_stride,
                     c10::nullopt, c10::nullopt, c, partials, c10::nullopt, c10::nullopt, c10::nullopt, tap, T, 0, 0,
                     0);
  if (tp) {
    // int64 CPU [mode, peer_sig, sig, done, epoch, phase, world, rank, peer_y, peer_yperm, peer_pos, ids, e_local]
    TORCH_CHECK(!tp->is_cuda() && tp->scalar_type() == at::kLong && tp->numel() >= 13, "tp: int64 CPU [13]");
    TORCH_CHECK(err.has_value(), "tp mode needs the error word");
    const int64_t* v = tp->data_ptr<int64_t>();
    p.tp_mode = (int)v[0];
    p.wait = peer_sync_of(tp->narrow(0, 1, 7));
    p.peer_y = reinterpret_cast<const float* const*>(v[8]);
    p.peer_yperm = reinterpret_cast<const bf16* const*>(v[9]);
    p.peer_pos = reinterpret_cast<const int* const*>(v[10]);
    p.ids = reinterpret_cast<const int*>(v[11]);
    p.e_local = (int)v[12];
    p.err = reinterpret_cast<uint32_t*>(err->data_ptr<int>());
    TORCH_CHECK(p.tp_mode == 1 ? p.peer_y != nullptr
                : p.tp_mode == 3 ? (p.peer_y != nullptr && p.peer_pos != nullptr && topk > 0)
                : p.tp_mode == 4 ? (p.yperm != nullptr && p.pos != nullptr && topk > 0)
                                 : (p.peer_yperm && p.peer_pos && p.ids && p.e_local > 0 && topk > 0),
                "tp mode tables missing");
    TORCH_CHECK(p.tp_mode >= 1 && p.tp_mode <= 4, "tp mode must be 1 .. 4");
  }
  const c10::cuda::CUDAGuard guard(X.device());
  CUDA_OK(dsv4::hc_post(p, cur_stream()));
}

void hc_finish(const Tensor& X, const optional<Tensor>& fn_hilo, const optional<Tensor>& scale,
               const optional<Tensor>& base, const optional<Tensor>& cw, const optional<Tensor>& norm_w,
               const optional<Tensor>& mix_out, const Tensor& c, const Tensor& partials, const optional<Tensor>& u,
               const optional<Tensor>& uq, const optional<Tensor>& usf, int64_t T, int64_t iters, double hc_eps,
               double norm_eps) {
  auto p = hc_params(X, c10::nullopt, c10::nullopt, c10::nullopt, 0, c10::nullopt, fn_hilo, scale, base, cw, 24,
                     norm_w, mix_out, c, partials, u, uq, usf, c10::nullopt, T, iters, hc_eps, norm_eps);
  const c10::cuda::CUDAGuard guard(X.device());
  CUDA_OK(dsv4::hc_finish(p, cur_stream()));
}

void attention(const Tensor& q, const Tensor& cos, const Tensor& sin, const optional<Tensor>& rope_pos,
               bool q_head_norm, double norm_eps, const Tensor& kv_step, const Tensor& ring,
               const optional<Tensor>& comp, const Tensor& slot, const Tensor& pos, const Tensor& chunk_start,
               const Tensor& step_row0, const optional<Tensor>& comp_idx, const optional<Tensor>& comp_cnt,
               const Tensor& sink, double scale, const Tensor& out, const optional<Tensor>& workspace, int64_t T,
               int64_t nsplit, const optional<Tensor>& win_end, int64_t win_len,
               const optional<Tensor>& comp_pages) {
  CHECK_CUDA(q);
  TORCH_CHECK(q.dim() == 3 && q.size(-1) == 512 && q.size(-2) <= 64 && q.stride(1) == 512 && q.stride(2) == 1,
              "q must be [T, H <= 64, 512]");
  TORCH_CHECK(out.dim() == 3 && out.size(1) == q.size(1) && out.stride(1) == 512 && out.stride(2) == 1,
              "out must be [T, H, 512]");
  TORCH_CHECK(sink.numel() >= q.size(1), "sink must hold every head");
  dsv4::AttnParams p{};
  p.T = (int)T;
  p.q = ptr<const bf16>(q);
  p.q_stride = (int)q.stride(0);
  p.n_heads = (int)q.size(1);
  p.out_stride = (int)out.stride(0);
  p.rope_cos = ptr<const float>(cos);
  p.rope_sin = ptr<const float>(sin);
  p.rope_pos = ptr<const int>(rope_pos);
  p.q_head_norm = q_head_norm;
  p.norm_eps = (float)norm_eps;
  // window rows are KV8 records, compressed rows KV4 records (csrc/common.cuh)
  TORCH_CHECK(kv_step.scalar_type() == at::kByte && kv_step.dim() == 2 && kv_step.size(1) == dsv4::kv8_bytes(512),
              "kv_step must be [R, 528] uint8 KV8 records");
  TORCH_CHECK(ring.scalar_type() == at::kByte && ring.dim() == 3 && ring.size(2) == dsv4::kv8_bytes(512),
              "ring must be [slots, W, 528] uint8 KV8 records");
  if (comp)
    TORCH_CHECK(comp->scalar_type() == at::kByte && comp->dim() == 3 && comp->size(2) == dsv4::kv4_bytes(512),
                "comp must be [slots, max_c, 288] uint8 KV4 records");
  p.kv_step = ptr<const uint8_t>(kv_step);
  p.ring = ptr<const uint8_t>(ring);
  p.W = (int)ring.size(1);
  p.comp = ptr<const uint8_t>(comp);
  p.max_c = comp ? (int)comp->size(1) : 0;
  if (comp) p.comp_pages = kv_pages_of(comp_pages, &p.max_c);
  p.slot = ptr<const int>(slot);
  p.pos = ptr<const int>(pos);
  p.chunk_start = ptr<const int>(chunk_start);
  p.step_row0 = ptr<const int>(step_row0);
  p.comp_idx = ptr<const int>(comp_idx);
  p.comp_k = comp_idx ? (int)comp_idx->size(1) : 0;
  p.comp_cnt = ptr<const int>(comp_cnt);
  if (comp) TORCH_CHECK(comp_cnt.has_value(), "comp_cnt required with comp");
  p.win_end = ptr<const int>(win_end);
  p.win_len = (int)win_len;
  TORCH_CHECK(win_len <= dsv4::kAttnMaxRows, "window longer than the attention row limit");
  p.sink = ptr<const float>(sink);
  p.scale = (float)scale;
  p.out = ptr<bf16>(out);
  p.workspace = ptr<float>(workspace);
  if (nsplit > 1) TORCH_CHECK(workspace && workspace->numel() >= T * nsplit * 64 * 514, "attention workspace");
  const c10::cuda::CUDAGuard guard(q.device());
  CUDA_OK(dsv4::attention(p, (int)nsplit, cur_stream()));
}

void qkv_post(const Tensor& in, int64_t q_dim, int64_t kv_dim, const Tensor& q_norm_w, const Tensor& kv_norm_w,
              double eps, const Tensor& qr_q, const Tensor& qr_sf, const Tensor& cos, const Tensor& sin,
              const Tensor& pos, const Tensor& kv_out, int64_t T) {
  dsv4::QkvParams p{};
  p.T = (int)T;
  p.q_dim = (int)q_dim;
  p.kv_dim = (int)kv_dim;
  TORCH_CHECK(q_dim % 128 == 0 && kv_dim % 32 == 0, "dims");
  p.in = ptr<const bf16>(in);
  p.q_norm_w = ptr<const bf16>(q_norm_w);
  p.kv_norm_w = ptr<const bf16>(kv_norm_w);
  p.eps = (float)eps;
  p.qr_q = ptr<uint8_t>(qr_q);
  p.qr_sf = ptr<uint8_t>(qr_sf);
  p.rope_cos = ptr<const float>(cos);
  p.rope_sin = ptr<const float>(sin);
  p.pos = ptr<const int>(pos);
  TORCH_CHECK(kv_out.scalar_type() == at::kByte && kv_out.size(-1) == dsv4::kv8_bytes((int)kv_dim),
              "kv_out must hold kv8_bytes(kv_dim) uint8 per row (KV8 records)");
  p.kv_out = ptr<uint8_t>(kv_out);
  const c10::cuda::CUDAGuard guard(in.device());
  CUDA_OK(dsv4::qkv_post(p, cur_stream()));
}

void idx_q_prep(const Tensor& q, int64_t T, int64_t n_heads, int64_t head_dim, const Tensor& cos, const Tensor& sin,
                const Tensor& pos, const optional<Tensor>& w_in, double w_scale, const optional<Tensor>& w_out) {
  CUDA_OK(dsv4::idx_q_prep(ptr<bf16>(q), (int)T, (int)n_heads, (int)head_dim, ptr<const float>(cos),
                           ptr<const float>(sin), ptr<const int>(pos), ptr<const float>(w_in), (float)w_scale,
                           ptr<float>(w_out), cur_stream()));
}

void compress_pool(int64_t n_groups, const Tensor& n_groups_dev, const Tensor& g_slot, const Tensor& g_index, const Tensor& g_chunk_start,
                   const Tensor& g_row0, int64_t r, int64_t co, const Tensor& proj, const optional<Tensor>& ape,
                   const Tensor& ring, const Tensor& norm_w, double eps, const Tensor& cos, const Tensor& sin,
                   const Tensor& comp_out, const optional<Tensor>& wk, const optional<Tensor>& k_norm_w,
                   const optional<Tensor>& idx_out, const optional<Tensor>& pages) {
  dsv4::CompParams p{};
  p.n_groups = (int)n_groups;
  p.n_groups_dev = ptr<const int>(n_groups_dev);
  p.g_slot = ptr<const int>(g_slot);
  p.g_index = ptr<const int>(g_index);
  p.g_chunk_start = ptr<const int>(g_chunk_start);
  p.g_row0 = ptr<const int>(g_row0);
  p.r = (int)r;
  p.co = (int)co;
  // comp_out holds KV4 records: 288 bytes per 512-dim row
  TORCH_CHECK(comp_out.scalar_type() == at::kByte && comp_out.size(2) == dsv4::kv4_bytes(512),
              "comp_out must be [slots, max_c, 288] uint8 KV4 records");
  p.dh = 512;
  p.proj = ptr<const float>(proj);
  p.ape = ptr<const float>(ape);
  p.ring = ptr<const float>(ring);
  p.norm_w = ptr<const bf16>(norm_w);
  p.eps = (float)eps;
  p.rope_cos = ptr<const float>(cos);
  p.rope_sin = ptr<const float>(sin);
  p.comp_out = ptr<uint8_t>(comp_out);
  p.max_c = (int)comp_out.size(1);
  p.wk = ptr<const bf16>(wk);
  p.k_norm_w = ptr<const bf16>(k_norm_w);
  if (idx_out)
    TORCH_CHECK(idx_out->scalar_type() == at::kByte && idx_out->size(2) == dsv4::ik4_bytes(128),
                "idx_out must be [slots, max_c, 68] uint8 IK4 records (128-dim keys)");
  p.idx_out = ptr<uint8_t>(idx_out);
  p.idx_dim = idx_out ? 128 : 0;
  p.pages = kv_pages_of(pages, &p.max_c);
  CUDA_OK(dsv4::compress_pool(p, cur_stream()));
}

void ring_update(const Tensor& ring, const Tensor& src, int64_t T, const Tensor& slot, const Tensor& pos,
                 const Tensor& last_pos) {
  const int depth = (int)ring.size(1);
  const int width = (int)ring.size(2);
  TORCH_CHECK(src.scalar_type() == ring.scalar_type() && src.size(-1) == width, "ring / source row mismatch");
  if (ring.scalar_type() == at::kFloat)
    CUDA_OK(dsv4::ring_update_f32(ptr<float>(ring), depth, width, ptr<const float>(src), (int)T, ptr<const int>(slot),
                                  ptr<const int>(pos), ptr<const int>(last_pos), cur_stream()));
  else if (ring.scalar_type() == at::kByte)
    CUDA_OK(dsv4::ring_update_rec(ptr<uint8_t>(ring), depth, width, ptr<const uint8_t>(src), (int)T,
                                  ptr<const int>(slot), ptr<const int>(pos), ptr<const int>(last_pos), cur_stream()));
  else
    CUDA_OK(dsv4::ring_update_bf16(ptr<bf16>(ring), depth, width, ptr<const bf16>(src), (int)T, ptr<const int>(slot),
                                   ptr<const int>(pos), ptr<const int>(last_pos), cur_stream()));
}

void router_topk(const Tensor& logits, int64_t T, const optional<Tensor>& bias, int64_t topk, int64_t score_func,
                 double route_scale, const Tensor& ids, const Tensor& wts) {
  CUDA_OK(dsv4::router_topk(ptr<const float>(logits), (int)T, (int)logits.size(1), ptr<const float>(bias), (int)topk,
                            (int)score_func, (float)route_scale, ptr<int>(ids), ptr<float>(wts), cur_stream()));
}

void router_small(const Tensor& u, const Tensor& w, int64_t T, const Tensor& logits, const optional<Tensor>& bias,
                  int64_t topk, int64_t score_func, double route_scale, const Tensor& ids, const Tensor& wts,
                  const Tensor& counter) {
  TORCH_CHECK(u.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && u.is_contiguous() &&
                  w.is_contiguous() && u.size(1) == w.size(1), "router_small: bf16 u [T, D] and gate [E, D]");
  // the gate matrix may carry padding rows past E (128-row GEMM tiles): E is the logits width
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(0) == logits.size(1) &&
                  logits.stride(1) == 1 && w.size(0) >= logits.size(1), "router_small: f32 logits [T, E], E <= gate rows");
  TORCH_CHECK(counter.scalar_type() == at::kInt && counter.is_cuda(), "router_small: int32 counter");
  dsv4::RouterSmallParams p{};
  p.u = ptr<const bf16>(u);
  p.w = ptr<const bf16>(w);
  p.T = (int)T;
  p.D = (int)u.size(1);
  p.E = (int)logits.size(1);
  p.logits = logits.data_ptr<float>();
  p.bias = ptr<const float>(bias);
  p.topk = (int)topk;
  p.score_func = (int)score_func;
  p.route_scale = (float)route_scale;
  p.ids = ptr<int>(ids);
  p.wts = ptr<float>(wts);
  p.counter = counter.data_ptr<int>();
  const c10::cuda::CUDAGuard guard(u.device());
  CUDA_OK(dsv4::router_small(p, cur_stream()));
}

void moe_plan(int64_t T, int64_t topk, int64_t e_local, int64_t e_begin, const Tensor& ids, const Tensor& wts,
              const Tensor& counts, const Tensor& seg_start, const Tensor& rank, int64_t tile_rows, int64_t m13,
              int64_t m2, const Tensor& tiles13, const Tensor& n_tiles13, const Tensor& tiles2,
              const Tensor& n_tiles2, int64_t cap_rows, const Tensor& pos, const Tensor& row_scale,
              const Tensor& err, const optional<Tensor>& seg_cnt, int64_t seg_cap, int64_t shared_rows,
              int64_t shared_row0) {
  dsv4::MoePlanParams p{};
  p.T = (int)T;
  p.topk = (int)topk;
  p.E_local = (int)e_local;
  p.e_begin = (int)e_begin;
  p.ids = ptr<const int>(ids);
  p.wts = ptr<const float>(wts);
  p.counts = ptr<int>(counts);
  p.seg_start = ptr<int>(seg_start);
  p.rank = ptr<int>(rank);
  p.tile_rows = (int)tile_rows;
  p.m13 = (int)m13;
  p.m2 = (int)m2;
  p.tiles13 = ptr<int4>(tiles13);
  p.n_tiles13 = ptr<int>(n_tiles13);
  p.tiles2 = ptr<int4>(tiles2);
  p.n_tiles2 = ptr<int>(n_tiles2);
  p.max_tiles13 = (int)tiles13.size(0);
  p.max_tiles2 = (int)tiles2.size(0);
  p.cap_rows = (int)cap_rows;
  p.pos = ptr<int>(pos);
  p.row_scale = ptr<float>(row_scale);
  p.err = ptr<uint32_t>(err);
  p.seg_cnt = ptr<const int>(seg_cnt);
  p.seg_cap = (int)seg_cap;
  p.shared_rows = (int)shared_rows;
  p.shared_row0 = (int)shared_row0;
  p.rs_rows = (int)row_scale.numel();
  if (shared_rows > 0)
    TORCH_CHECK(shared_row0 + shared_rows <= row_scale.numel(), "shared segment outside row_scale");
  CUDA_OK(dsv4::moe_plan(p, cur_stream()));
}

void moe_scatter(const Tensor& xq, const Tensor& xsf, int64_t T, int64_t topk, const Tensor& pos, const Tensor& pq,
                 const Tensor& psf, int64_t shared_row0) {
  if (shared_row0 >= 0) TORCH_CHECK(shared_row0 + T <= pq.size(0), "shared segment outside the permuted buffer");
  CUDA_OK(dsv4::moe_scatter(ptr<const uint8_t>(xq), ptr<const uint8_t>(xsf), (int)T, (int)xq.size(1), (int)topk,
                            ptr<const int>(pos), ptr<uint8_t>(pq), ptr<uint8_t>(psf), (int)shared_row0,
                            (int)pq.size(0), cur_stream()));
}

void indexer_topk(const Tensor& q, const Tensor& w, const Tensor& kcache, const Tensor& slot, const Tensor& clen,
                  int64_t topk, const Tensor& out_idx, const Tensor& out_cnt, const optional<Tensor>& cand,
                  int64_t cand_mode, int64_t cand_block, int64_t cand_topk, int64_t T, const Tensor& err,
                  const optional<Tensor>& kcache_alt, const optional<Tensor>& pos,
                  const optional<Tensor>& chunk_start, const optional<Tensor>& last_pos, int64_t own_r,
                  const Tensor& keys, const optional<Tensor>& pages, const optional<Tensor>& alt_pages) {
  dsv4::IdxParams p{};
  p.T = (int)T;
  p.n_heads = (int)q.size(1);
  p.head_dim = (int)q.size(2);
  p.q = ptr<const bf16>(q);
  p.w = ptr<const float>(w);
  // key caches hold IK4 records (kernels.h): 68 bytes per 128-dim key
  TORCH_CHECK(q.size(2) == 128, "indexer head dim must be 128");
  TORCH_CHECK(kcache.scalar_type() == at::kByte && kcache.dim() == 3 && kcache.size(2) == dsv4::ik4_bytes(128),
              "kcache must be [slots, max_c, 68] uint8 IK4 records");
  if (kcache_alt)
    TORCH_CHECK(kcache_alt->scalar_type() == at::kByte && kcache_alt->size(2) == dsv4::ik4_bytes(128),
                "kcache_alt must hold IK4 records");
  p.kcache = ptr<const uint8_t>(kcache);
  p.max_c = (int)kcache.size(1);
  p.slot = ptr<const int>(slot);
  p.clen = ptr<const int>(clen);
  p.topk = (int)topk;
  p.out_idx = ptr<int>(out_idx);
  p.out_cnt = ptr<int>(out_cnt);
  p.cand = ptr<uint8_t>(cand);
  p.cand_mode = (int)cand_mode;
  p.cand_block = (int)std::max<int64_t>(1, cand_block);
  p.cand_topk = (int)cand_topk;
  p.err = ptr<uint32_t>(err);
  p.kcache_alt = ptr<const uint8_t>(kcache_alt);
  p.alt_max_c = kcache_alt ? (int)kcache_alt->size(1) : 0;
  p.pages = kv_pages_of(pages, &p.max_c);
  if (kcache_alt) p.alt_pages = kv_pages_of(alt_pages, &p.alt_max_c);
  p.pos = ptr<const int>(pos);
  p.chunk_start = ptr<const int>(chunk_start);
  p.last_pos = ptr<const int>(last_pos);
  p.own_r = (int)std::max<int64_t>(1, own_r);
  if (kcache_alt) TORCH_CHECK(pos && chunk_start && last_pos, "pos/chunk_start/last_pos required with kcache_alt");
  TORCH_CHECK(keys.dim() == 2 && keys.size(0) >= T && keys.size(1) >= p.max_c && keys.element_size() == 4,
              "keys scratch must be [>=T, >=max_c] 32-bit");
  CUDA_OK(dsv4::indexer_topk(p, ptr<uint32_t>(keys), (int)keys.stride(0), cur_stream()));
}

// sync = optional int64 tensor [peer_sig_table, peer_cnt_table, done, epoch] of device addresses
static dsv4::EpSync ep_sync(const optional<Tensor>& sync, int phase) {
  dsv4::EpSync s{nullptr, nullptr, nullptr, nullptr, phase};
  if (!sync) return s;
  TORCH_CHECK(sync->device().is_cpu() && sync->dtype() == torch::kInt64 && sync->numel() == 4,
              "sync must be a CPU int64 tensor of 4 device addresses");
  const int64_t* a = sync->data_ptr<int64_t>();
  s.peer_sig = reinterpret_cast<uint32_t* const*>(a[0]);
  s.peer_cnt = reinterpret_cast<int* const*>(a[1]);
  s.done = reinterpret_cast<int*>(a[2]);
  s.epoch = reinterpret_cast<uint32_t*>(a[3]);
  return s;
}

void ep_pack(const Tensor& ids, const Tensor& wts, int64_t T, const Tensor& xq, const Tensor& xsf, int64_t e_local,
             int64_t world, int64_t cap, int64_t rec, const Tensor& send, const Tensor& cnt, const Tensor& pos_back,
             const optional<Tensor>& peer_recv, int64_t my_rank, const Tensor& err, const optional<Tensor>& sync) {
  CUDA_OK(dsv4::ep_pack(ptr<const int>(ids), ptr<const float>(wts), (int)T, (int)ids.size(1), ptr<const uint8_t>(xq),
                        ptr<const uint8_t>(xsf), (int)xq.size(1), (int)e_local, (int)world, (int)cap, (int)rec,
                        ptr<uint8_t>(send), ptr<int>(cnt), ptr<int>(pos_back), ptr<uint8_t* const>(peer_recv),
                        (int)my_rank, ptr<uint32_t>(err), ep_sync(sync, 0), cur_stream()));
}

void ep_wait(const Tensor& sig, int64_t world, int64_t phase, const Tensor& epoch, const Tensor& err) {
  CUDA_OK(dsv4::ep_wait(ptr<const uint32_t>(sig), (int)world, (int)phase, ptr<const uint32_t>(epoch),
                        ptr<uint32_t>(err), cur_stream()));
}

void ep_unpack_meta(const Tensor& recv, const Tensor& cnt, int64_t world, int64_t cap, int64_t rec, int64_t D,
                    const Tensor& ids, const Tensor& wts) {
  CUDA_OK(dsv4::ep_unpack_meta(ptr<const uint8_t>(recv), ptr<const int>(cnt), (int)world, (int)cap, (int)rec, (int)D,
                               ptr<int>(ids), ptr<float>(wts), cur_stream()));
}

// cnt: int32 [world] records received from each peer
void ep_unpack_rows(const Tensor& recv, const Tensor& cnt, int64_t world, int64_t cap, int64_t rec, int64_t D,
                    const Tensor& pos, const Tensor& pq, const Tensor& psf) {
  CUDA_OK(dsv4::ep_unpack_rows(ptr<const uint8_t>(recv), ptr<const int>(cnt), (int)world, (int)cap, (int)rec, (int)D,
                               ptr<const int>(pos), ptr<uint8_t>(pq), ptr<uint8_t>(psf), cur_stream()));
}

void ep_combine_pack(const Tensor& yperm, const Tensor& pos, const Tensor& cnt, int64_t cap, const Tensor& back,
                     const optional<Tensor>& peer_back, int64_t my_rank, int64_t world, const optional<Tensor>& sync) {
  CUDA_OK(dsv4::ep_combine_pack(ptr<const bf16>(yperm), ptr<const int>(pos), ptr<const int>(cnt),
                                (int)yperm.size(1), (int)cap, ptr<bf16>(back), ptr<bf16* const>(peer_back),
                                (int)my_rank, (int)world, ep_sync(sync, 1), cur_stream()));
}

// Fused expert-parallel dispatch.  tables: int64 CPU [5] = device addresses of
// the [world] pointer tables (expert rows, their scale chunks, row weights, row
// origins, per-expert counters) of every rank; pub: PeerSync of phase 0.
void ep_dispatch(const Tensor& logits, int64_t T, const optional<Tensor>& bias, int64_t topk, int64_t score_func,
                 double route_scale, const optional<Tensor>& ids, const optional<Tensor>& wts, const Tensor& xq,
                 const Tensor& xsf, int64_t e_local, int64_t cap_e, int64_t tile_rows, int64_t ret_rows,
                 const Tensor& tables, const Tensor& err, const Tensor& pub, int64_t shared_row0) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1 &&
                  logits.stride(0) == logits.size(1), "logits: f32 [T, E] contiguous");
  TORCH_CHECK(!tables.is_cuda() && tables.scalar_type() == at::kLong && tables.numel() == 5, "tables: int64 CPU [5]");
  TORCH_CHECK(xq.size(0) >= T && xq.size(1) % 128 == 0, "xq: [>= T, D]");
  TORCH_CHECK(ids.has_value() == wts.has_value(), "ids and wts together");
  const int64_t* tb = tables.data_ptr<int64_t>();
  dsv4::EpDispatchParams p{};
  p.logits = logits.data_ptr<float>();
  p.bias = ptr<const float>(bias);
  p.T = (int)T;
  p.E = (int)logits.size(1);
  p.topk = (int)topk;
  p.score_func = (int)score_func;
  p.route_scale = (float)route_scale;
  p.ids = ptr<int>(ids);
  p.wts = ptr<float>(wts);
  p.xq = ptr<const uint8_t>(xq);
  p.xsf = ptr<const uint8_t>(xsf);
  p.D = (int)xq.size(1);
  p.e_local = (int)e_local;
  p.cap_e = (int)cap_e;
  p.tile_rows = (int)tile_rows;
  p.rows = (int)(e_local * cap_e);
  p.ret_rows = (int)ret_rows;
  p.peer_x = reinterpret_cast<uint8_t* const*>(tb[0]);
  p.peer_xsf = reinterpret_cast<uint8_t* const*>(tb[1]);
  p.peer_rscale = reinterpret_cast<float* const*>(tb[2]);
  p.peer_meta = reinterpret_cast<int* const*>(tb[3]);
  p.peer_cnt = reinterpret_cast<int* const*>(tb[4]);
  p.err = ptr<uint32_t>(err);
  p.pub = peer_sync_of(pub);
  p.world = p.pub.world;
  p.rank = p.pub.rank;
  p.shared_row0 = (int)shared_row0;
  TORCH_CHECK(shared_row0 < 0 || shared_row0 >= p.rows, "dispatch: the shared segment follows the expert rows");
  TORCH_CHECK(p.pub.done != nullptr && p.E == p.e_local * p.world, "dispatch: phase-0 sync and E = e_local * world");
  const c10::cuda::CUDAGuard guard(logits.device());
  CUDA_OK(dsv4::ep_dispatch(p, cur_stream()));
}

// wait: PeerSync of phase 0; tiles: int32 [max, 4]; cnt: this rank's counters [e_local]
void ep_plan(const Tensor& wait, const Tensor& cnt, int64_t cap_e, int64_t tile_rows, int64_t m13, int64_t m2,
             const Tensor& tiles13, const Tensor& nt13, const Tensor& tiles2, const Tensor& nt2, const Tensor& err,
             int64_t shared_rows, int64_t shared_row0) {
  CHECK_CUDA(cnt);
  TORCH_CHECK(tiles13.dim() == 2 && tiles13.size(1) == 4 && tiles2.dim() == 2 && tiles2.size(1) == 4, "tiles [n, 4]");
  dsv4::EpPlanParams p{};
  p.wait = peer_sync_of(wait);
  p.cnt = cnt.data_ptr<int>();
  p.e_local = (int)cnt.numel();
  p.cap_e = (int)cap_e;
  p.tile_rows = (int)tile_rows;
  p.m13 = (int)m13;
  p.m2 = (int)m2;
  p.tiles13 = reinterpret_cast<int4*>(tiles13.data_ptr<int>());
  p.n_tiles13 = nt13.data_ptr<int>();
  p.tiles2 = reinterpret_cast<int4*>(tiles2.data_ptr<int>());
  p.n_tiles2 = nt2.data_ptr<int>();
  p.max_tiles13 = (int)tiles13.size(0);
  p.max_tiles2 = (int)tiles2.size(0);
  p.err = ptr<uint32_t>(err);
  p.shared_rows = (int)shared_rows;
  p.shared_row0 = (int)shared_row0;
  const c10::cuda::CUDAGuard guard(cnt.device());
  CUDA_OK(dsv4::ep_plan(p, cur_stream()));
}

// tables: int64 CPU tensor [nl, 3] = (device-mapped table address, scale table address, n_emb)
void engram_prepare(const Tensor& ids, const Tensor& pos, const Tensor& slot, const Tensor& chunk_start,
                    const Tensor& step_row0, const Tensor& last_pos, int64_t T, const Tensor& token_map,
                    const Tensor& ring, const Tensor& mult, const Tensor& primes, const Tensor& offsets, int64_t pad,
                    const Tensor& rows, const optional<Tensor>& tables, const optional<Tensor>& a_q,
                    const optional<Tensor>& a_sf, int64_t hd, int64_t mode) {
  dsv4::EngramParams p{};
  p.T = (int)T;
  p.nl = (int)mult.size(0);
  p.N = (int)mult.size(1);
  p.H = (int)primes.size(2);
  p.hd = (int)hd;
  p.ids = ptr<const int>(ids);
  p.pos = ptr<const int>(pos);
  p.slot = ptr<const int>(slot);
  p.chunk_start = ptr<const int>(chunk_start);
  p.step_row0 = ptr<const int>(step_row0);
  p.last_pos = ptr<const int>(last_pos);
  p.token_map = ptr<const int64_t>(token_map);
  p.ring = ptr<int64_t>(ring);
  p.mult = ptr<const int64_t>(mult);
  p.primes = ptr<const int64_t>(primes);
  p.offsets = ptr<const int64_t>(offsets);
  p.pad = pad;
  p.rows = ptr<int64_t>(rows);
  TORCH_CHECK(p.nl <= dsv4::kEngramMaxLayers, "too many Engram layers");
  const bool gather = (mode & 4) != 0;
  if (gather) {
    TORCH_CHECK(a_q && a_sf && tables->device().is_cpu() && tables->size(0) == p.nl, "bad Engram tables");
    const int64_t* t = tables->data_ptr<int64_t>();
    for (int l = 0; l < p.nl; ++l) {
      p.table[l] = reinterpret_cast<const uint8_t*>(t[3 * l]);
      p.table_sf[l] = reinterpret_cast<const uint8_t*>(t[3 * l + 1]);
      p.n_emb[l] = t[3 * l + 2];
    }
    p.a_q = ptr<uint8_t>(a_q);
    p.a_sf = ptr<uint8_t>(a_sf);
    p.a_stride_q = (size_t)a_q->stride(0);
    p.a_stride_sf = (size_t)a_sf->stride(0);
  }
  CUDA_OK(dsv4::engram_prepare(p, (int)mode, cur_stream()));
}

void engram_gate(const Tensor& X, const Tensor& kv, const Tensor& wgt, int64_t T, double eps) {
  CUDA_OK(dsv4::engram_gate(ptr<bf16>(X), ptr<const bf16>(kv), ptr<const float>(wgt), (int)T, (int)X.size(2),
                            (int)X.size(1), (float)eps, cur_stream()));
}

// Pins an existing host allocation and returns the device address that kernels read it through.
int64_t host_register(int64_t addr, int64_t bytes) {
  void* p = reinterpret_cast<void*>(addr);
  CUDA_OK(cudaHostRegister(p, (size_t)bytes, cudaHostRegisterMapped | cudaHostRegisterPortable));
  void* d = nullptr;
  CUDA_OK(cudaHostGetDevicePointer(&d, p, 0));
  return reinterpret_cast<int64_t>(d);
}

void host_unregister(int64_t addr) { CUDA_OK(cudaHostUnregister(reinterpret_cast<void*>(addr))); }

// Device address of page-locked host memory (e.g. a pinned torch tensor).
int64_t host_device_ptr(int64_t addr) {
  void* d = nullptr;
  CUDA_OK(cudaHostGetDevicePointer(&d, reinterpret_cast<void*>(addr), 0));
  return reinterpret_cast<int64_t>(d);
}

void embed_streams(const Tensor& table, const Tensor& ids, int64_t T, const Tensor& X) {
  CUDA_OK(dsv4::embed_streams(ptr<const bf16>(table), ptr<const int>(ids), (int)T, (int)table.size(1),
                              (int)X.size(1), ptr<bf16>(X), cur_stream()));
}

void markov_step(const Tensor& logits, int64_t blk, int64_t i, const Tensor& mlog, int64_t V, int64_t n,
                 const Tensor& toks, const Tensor& memb, const Tensor& emb) {
  CUDA_OK(dsv4::markov_step(ptr<const float>(logits), (int)logits.stride(0), (int)blk, (int)i,
                            ptr<const float>(mlog), (int)mlog.stride(0), (int)V, (int)n, ptr<int>(toks),
                            (int)toks.stride(0), ptr<const bf16>(memb), (int)memb.size(1), ptr<bf16>(emb),
                            cur_stream()));
}

// scratch: optional int32 [2 * max(T, 296) + T]; its tail (T entries) must start zeroed and is left zeroed
void argmax_rows(const Tensor& logits, int64_t T, int64_t V, const Tensor& out, const optional<Tensor>& scratch,
                 const optional<Tensor>& out_val, int64_t idx_base) {
  float* wv = nullptr;
  int* wi = nullptr;
  int* cnt = nullptr;
  if (scratch) {
    const int64_t cap = std::max<int64_t>(T, 296);
    TORCH_CHECK(scratch->scalar_type() == at::kInt && scratch->numel() >= 2 * cap + T, "argmax scratch too small");
    const int64_t n = scratch->numel();
    int* base = ptr<int>(*scratch);
    const int64_t tail = n - T;   // counters live at the fixed end of the buffer
    wv = reinterpret_cast<float*>(base);
    wi = base + cap;
    cnt = base + tail;
    TORCH_CHECK(cap * 2 <= tail, "argmax scratch too small");
  }
  CUDA_OK(dsv4::argmax_rows(ptr<const float>(logits), (int)T, (int)V, (int)logits.stride(0), ptr<int>(out), wv, wi,
                            cnt, ptr<float>(out_val), (int)idx_base, cur_stream()));
}

// measurement: stamps int64 [1 + 2 * ctas]
void pdl_probe(const Tensor& stamps, int64_t ctas, int64_t ns) {
  TORCH_CHECK(stamps.numel() >= 1 + 2 * ctas && stamps.scalar_type() == at::kLong, "stamps: int64 [1 + 2 ctas]");
  CUDA_OK(dsv4::pdl_probe(reinterpret_cast<unsigned long long*>(stamps.data_ptr()), (int)ctas,
                          (unsigned long long)ns, cur_stream()));
}

// device timestamp ring: int64 [n]; ring[slot] = %globaltimer once the previous kernel has completed
void ts_mark(const Tensor& ring, int64_t slot) {
  TORCH_CHECK(ring.is_cuda() && ring.scalar_type() == at::kLong && slot >= 0 && slot < ring.numel(),
              "ts_mark: int64 device ring, slot in range");
  const c10::cuda::CUDAGuard guard(ring.device());
  CUDA_OK(dsv4::ts_mark(reinterpret_cast<unsigned long long*>(ring.data_ptr()), (int)slot, cur_stream()));
}

// sync: int64 CPU [7] (PeerSync); peer_val / peer_idx: int64 device tables of each rank's pairs
void tp_argmax_merge(const Tensor& sync, const Tensor& peer_val, const Tensor& peer_idx, int64_t T, const Tensor& out,
                     const Tensor& err) {
  CUDA_OK(dsv4::tp_argmax_merge(peer_sync_of(sync), reinterpret_cast<const float* const*>(peer_val.data_ptr()),
                                reinterpret_cast<const int* const*>(peer_idx.data_ptr()), (int)T, ptr<int>(out),
                                reinterpret_cast<uint32_t*>(err.data_ptr<int>()), cur_stream()));
}


}  // namespace

int64_t debug_bounds_attach(const Tensor& err) {
  TORCH_CHECK(err.is_cuda() && err.numel() >= 1 && err.element_size() == 4, "error word: int32 CUDA tensor");
  c10::cuda::CUDAGuard g(err.device());
  const int n = dsv4::dbg_bounds_attach(reinterpret_cast<uint32_t*>(err.data_ptr()));
  TORCH_CHECK(n >= 0, "debug bounds attach failed: ", cudaGetErrorString((cudaError_t)(-n)));
  return n;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "DeepSeek-V4 B200 kernels (sm_100a)";
  m.def("gemm", &gemm);
  m.def("gemm_a2", &gemm_a2);
  m.def("gemm_smem", &gemm_smem);
  m.def("act_quant_mx", &act_quant_mx);
  m.def("act_roundtrip", &act_roundtrip);
  m.def("fp4_roundtrip", &fp4_roundtrip);
  m.def("hc_post", &hc_post);
  m.def("hc_finish", &hc_finish);
  m.def("hc_num_slices", [](int64_t d) { return (int64_t)dsv4::hc_num_slices((int)d); });
  m.def("attention", &attention);
  m.def("debug_bounds_attach", &debug_bounds_attach);
  m.def("debug_bounds_units", []() { return (int64_t)dsv4::dbg_bounds_units(); });
#ifdef DSV4_DEBUG_BOUNDS
  m.attr("debug_bounds") = true;
#else
  m.attr("debug_bounds") = false;
#endif
  m.def("attn_smem", []() { return (int64_t)dsv4::attn_smem_bytes(); });
  m.def("qkv_post", &qkv_post);
  m.def("idx_q_prep", &idx_q_prep);
  m.def("compress_pool", &compress_pool);
  m.def("ring_update", &ring_update);
  m.def("router_topk", &router_topk);
  m.def("router_small", &router_small);
  m.def("moe_plan", &moe_plan);
  m.def("moe_scatter", &moe_scatter);
  m.def("indexer_topk", &indexer_topk);
  m.def("embed_streams", &embed_streams);
  m.def("engram_prepare", &engram_prepare);
  m.def("engram_gate", &engram_gate);
  m.def("host_register", &host_register);
  m.def("host_unregister", &host_unregister);
  m.def("host_device_ptr", &host_device_ptr);
  m.def("ep_pack", &ep_pack);
  m.def("ep_wait", &ep_wait);
  m.def("ep_unpack_meta", &ep_unpack_meta);
  m.def("ep_unpack_rows", &ep_unpack_rows);
  m.def("ep_combine_pack", &ep_combine_pack);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_plan", &ep_plan);
  m.def("argmax_rows", &argmax_rows);
  m.def("tp_argmax_merge", &tp_argmax_merge);
  m.def("pdl_probe", &pdl_probe);
  m.def("ts_mark", &ts_mark);
  m.def("markov_step", &markov_step);
}
