// Python bindings of the sm_100a kernels.  Every entry point checks device,
// dtype and layout, then launches on the current CUDA stream; nothing here
// allocates device memory (callers own all buffers).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "gemm.h"
#include "kernels.h"

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
void gemm(int64_t kind, int64_t epi, const Tensor& A, const optional<Tensor>& A_sf, const Tensor& B,
          const optional<Tensor>& B_sf, const optional<Tensor>& out, int64_t M, int64_t N, int64_t K, int64_t bn,
          int64_t splits, const optional<Tensor>& tiles, const optional<Tensor>& n_tiles,
          const optional<Tensor>& row_scale, const optional<Tensor>& hq, const optional<Tensor>& hsf,
          double swiglu_limit, int64_t m_valid, int64_t ldo, const optional<Tensor>& workspace,
          const optional<Tensor>& counters, const Tensor& err, int64_t max_grid, int64_t groups) {
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
  CUtensorMap ta;
  dsv4::BMaps tb;
  TORCH_CHECK(dsv4::make_tma_2d(&ta, A.data_ptr(), tma_elem_of(A, e2m1), A.size(0), K, 128), "TMA(A) encode failed");
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
  p.splits = (int)std::max<int64_t>(1, splits);
  p.sfa = u8ptr(A_sf);
  p.sfa_ktiles = (int)(K / 128);
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
  if (p.splits > 1) TORCH_CHECK(workspace && counters, "split-K needs workspace and counters");
  int units;
  if (grouped) {
    p.tiles = reinterpret_cast<const int4*>(tiles->data_ptr<int>());
    p.n_tiles_ptr = n_tiles->data_ptr<int>();
    units = (int)tiles->size(0) * p.splits;
  } else {
    TORCH_CHECK(M % 128 == 0, "M must be a multiple of 128");
    p.n_tiles = (int)(M / 128) * (int)((N + bn - 1) / bn);
    units = p.n_tiles * p.splits;
  }
  if (units == 0) return;
  int grid = std::min(units, max_grid > 0 ? (int)max_grid : num_sms());
  CUDA_OK(dsv4::gemm_launch((int)kind, (int)epi, grouped, (int)bn, ta, tb, p, grid, cur_stream()));
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

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "DeepSeek-V4 B200 kernels (sm_100a)";
  m.def("gemm", &gemm);
  m.def("gemm_smem", &gemm_smem);
  m.def("act_quant_mx", &act_quant_mx);
  m.def("act_roundtrip", &act_roundtrip);
  m.def("fp4_roundtrip", &fp4_roundtrip);
}
