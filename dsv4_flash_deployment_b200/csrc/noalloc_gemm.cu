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
// Contract:
//  * Scratch: a file-scope `static __device__` array of kScratchFloats floats
//    for the split-K partial tiles plus kMaxTiles int32 tile counters
//    (4 MiB + 16 KiB).  Every GPU that loads the library holds it until the
//    process exits.
//  * Set-up: the first call on a device looks up the array's device address
//    with cudaGetSymbolAddress while that device is current.  That first call
//    should happen before any stream capture starts.
//  * Sharing: all calls on a device share the one array, which keeps the
//    last call's contents.  Each call clears its tile counters before it
//    launches.  Calls that overlap on the GPU (different streams, or different
//    host threads on one device) race on the array and corrupt each other's
//    results: serialize them.
//  * Limits: problems whose split-K partials need more than kScratchFloats
//    floats, or more than kMaxTiles output tiles, are rejected with return
//    code DSV4_NOALLOC_TOO_LARGE and a message on stderr; nothing is launched.
//  * No cudaMalloc, cudaFree or allocating library call is made.
//
// Arguments (all device pointers, row-major, the caller owns them):
//   a      e4m3 weights [m, k] (m a multiple of 128)
//   a_sf   ue8m0 scale chunks of a [m/128][k/128][512]
//   b      e4m3 activations [b_rows, k] (b_rows >= n, a multiple of 128)
//   b_sf   ue8m0 scale chunks of b [b_rows/128][k/128][512]
//   out    bf16 [n, ldo]; out[t][j] = sum_k a[j][k] * b[t][k] for j < m
//   err    one uint32 device word (0 on success; a kernel-side error code otherwise)
// Returns 0 on success, DSV4_NOALLOC_TOO_LARGE, DSV4_NOALLOC_BAD_ARG, or a
// cudaError_t value.
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "gemm.h"

namespace {

constexpr size_t kScratchFloats = size_t(1) << 20;  // 4 MiB of fp32 split-K partials
constexpr int kMaxTiles = 4096;                      // tile counters (16 KiB)
constexpr int kMaxDevices = 64;

struct ScratchArea {
  float partials[kScratchFloats];
  int counters[kMaxTiles];
};

static __device__ __align__(256) ScratchArea g_scratch;

ScratchArea* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_setup_mutex;

constexpr int DSV4_NOALLOC_TOO_LARGE = -1;
constexpr int DSV4_NOALLOC_BAD_ARG = -2;

// Device address of this device's scratch array; looked up once per device.
cudaError_t scratch_for_current_device(ScratchArea** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<ScratchArea*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int dsv4_gemm_mx8_noalloc(
    const void* a, const void* a_sf, const void* b, const void* b_sf, void* out, int m, int n, int k, int b_rows,
    int ldo, int splits, void* err, cudaStream_t stream) {
  if (!a || !a_sf || !b || !b_sf || !out || !err || m <= 0 || n <= 0 || k <= 0 || m % 128 || k % 128 ||
      b_rows < n || b_rows % 128 || splits < 1 || ldo < m) {
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
  CUtensorMap ta;
  dsv4::BMaps tb;
  if (!dsv4::make_tma_2d(&ta, a, dsv4::TMA_U8, (uint64_t)m, (uint64_t)k, 128) ||
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
