// dsv4_gemm_mx8_noalloc: block-scaled FP8 GEMM with split-K that allocates nothing.
//
// This entry point has no counterpart in the reference (which ships no native
// code); it is an addition of this library.
//
// Who it is for: callers that cannot allocate device memory while they run.
// Examples are real-time serving loops that forbid cudaMalloc/cudaFree (both
// synchronize the device and can stall every stream), and embedders with a
// fixed, pre-sized memory budget that owns every byte.
// The regular `gemm` binding expects the caller to pass a split-K workspace and
// tile counters; this variant instead uses one scratch array that lives in the
// library itself.
//
// The public prototype, return codes, scratch limits and the full contract are
// in dsv4_noalloc.h, which this file includes so the definition is checked
// against it.
#include <cuda.h>

#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "dsv4_noalloc.h"
#include "gemm.h"

namespace {

constexpr size_t kScratchFloats = DSV4_NOALLOC_SCRATCH_FLOATS;
constexpr int kMaxTiles = DSV4_NOALLOC_MAX_TILES;
constexpr int kMaxDevices = 64;

struct ScratchArea {
  float partials[kScratchFloats];
  int counters[kMaxTiles];
};

static __device__ __align__(256) ScratchArea g_scratch;

// Looked-up address per device, valid for the context it was looked up in.
struct ScratchSlot {
  ScratchArea* ptr = nullptr;
  CUcontext ctx = nullptr;
};
ScratchSlot g_slots[kMaxDevices];
std::mutex g_setup_mutex;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime (the library does not link libcuda).
CUcontext current_context() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(p);
    return static_cast<CtxGetCurrentFn>(nullptr);
  }();
  CUcontext c = nullptr;
  if (fn != nullptr && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}

// Device address of the scratch array in the current device's current context.
// Looked up once, and again whenever the context differs from the one of the
// last lookup (a reset device gets a new context).
cudaError_t scratch_for_current_device(ScratchArea** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  // makes the runtime's context of this device current if no call has done so yet
  // (cudaSetDevice initializes the primary context since CUDA 12)
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return e;
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  ScratchSlot& s = g_slots[dev];
  if (s.ptr == nullptr || s.ctx != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return e;
    s.ptr = static_cast<ScratchArea*>(p);
    s.ctx = ctx;
  }
  *out = s.ptr;
  return cudaSuccess;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int dsv4_gemm_mx8_noalloc(
    const void* a, const void* a_sf, const void* b, const void* b_sf, void* out, int m, int n, int k, int b_rows,
    int ldo, int splits, void* err, cudaStream_t stream) {
  if (!a || !a_sf || !b || !b_sf || !out || !err || m <= 0 || n <= 0 || k <= 0 || m % 128 || k % 128 ||
      b_rows < n || b_rows % 128 || splits < 1 || splits > k / 128 || ldo < m) {
    std::fprintf(stderr, "dsv4_gemm_mx8_noalloc: invalid arguments (m=%d n=%d k=%d b_rows=%d ldo=%d splits=%d)\n", m,
                 n, k, b_rows, ldo, splits);
    return DSV4_NOALLOC_BAD_ARG;
  }
  const int bn = n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : 256;
  const int tiles = (m / 128) * ((n + bn - 1) / bn);
  const size_t need = (size_t)tiles * splits * 128 * bn;
  if (splits > 1 && (need > kScratchFloats || tiles > kMaxTiles)) {
    std::fprintf(stderr,
                 "dsv4_gemm_mx8_noalloc: problem too large for the built-in scratch: needs %zu partial floats "
                 "(max %zu) and %d tile counters (max %d); use fewer splits or the allocating entry point\n",
                 need, kScratchFloats, tiles, kMaxTiles);
    return DSV4_NOALLOC_TOO_LARGE;
  }
  ScratchArea* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return (int)e;
  dsv4::AMaps ta{};
  dsv4::BMaps tb;
  if (!dsv4::make_tma_2d(&ta.m[0], a, dsv4::TMA_U8, (uint64_t)m, (uint64_t)k, 128) ||
      !dsv4::make_tma_2d(&tb.m[0], b, dsv4::TMA_U8, (uint64_t)b_rows, (uint64_t)k, (uint32_t)bn)) {
    std::fprintf(stderr, "dsv4_gemm_mx8_noalloc: tensor map encoding failed (alignment of a or b?)\n");
    return DSV4_NOALLOC_BAD_ARG;
  }
  if (splits > 1) {
    // counters must start at zero; the previous call on this device left its values here
    e = cudaMemsetAsync(scratch->counters, 0, sizeof(int) * tiles, stream);
    if (e != cudaSuccess) return (int)e;
  }
  dsv4::GemmParams p{};
  p.M = m;
  p.N = n;
  p.k_tiles = k / 128;
  p.n_tiles = tiles;
  p.splits = splits;
  p.sfa = static_cast<const uint8_t*>(a_sf);
  p.sfa_ktiles = k / 128;
  p.sfb = static_cast<const uint8_t*>(b_sf);
  p.sfb_ktiles = k / 128;
  p.group_rows = 1 << 30;
  p.group_k = 0;
  p.out = out;
  p.ldo = ldo;
  p.m_valid = m;
  p.workspace = scratch->partials;
  p.tile_counters = scratch->counters;
  p.err = static_cast<uint32_t*>(err);
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int units = tiles * splits;
  const int grid = units < sms ? units : sms;
  return (int)dsv4::gemm_launch(dsv4::KIND_MX8, dsv4::EPI_BF16, false, bn, 128, ta, tb, p, grid, stream);
}
