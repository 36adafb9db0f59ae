// Streaming-rate probe: how fast can one CTA per SM pull a 4 GB weight-like
// matrix into shared memory with the copy engines the GEMMs use?
//
// Variants (each CTA keeps a ring of stages in flight, one thread issues and
// waits; every wait is bounded by %globaltimer and reports through an error word):
//   tma2d   2-D tensor tiles of 128 rows x 128 B (128-byte swizzle), the GEMM's
//           weight tile; 32 KB boxes of 256 rows
//   bulk    1-D bulk copies of contiguous 8 / 16 / 32 KB chunks
//   GEMM order   each CTA walks the 32 k-tiles of its own 128-row block, as a
//                GEMM tile does (DRAM row locality of the strided boxes)
//   GEMM stage   a weight tile plus a 4 KB activation tile from an L2-resident
//                region and two 512-byte scale chunks per stage
// Built and run by bench/tma_stream.py; prints one line per variant (GB/s of
// the streamed matrix, read only).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#define CK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { printf("CUDA %s at %d\n", cudaGetErrorString(e_), __LINE__); exit(1);} } while (0)

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t gtime() { uint64_t t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t; }
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t c) { asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(c)); }
__device__ __forceinline__ void expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool try_wait(uint64_t* b, uint32_t ph) {
  uint32_t ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok) : "r"(smem_u32(b)), "r"(ph) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait_bounded(uint64_t* b, uint32_t ph, int* err) {
  if (try_wait(b, ph)) return true;
  const uint64_t t0 = gtime();
  while (!try_wait(b, ph)) {
    if (gtime() - t0 > 2000000000ull) { atomicExch(err, 1); return false; }
  }
  return true;
}
__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
               ::"r"(smem_u32(dst)), "l"(m), "r"(smem_u32(bar)), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}


// mode 0: 2-D tiles [rows, 4096 B] box {128 B, BOXR rows}; mode 1: 1-D bulk of CHUNK bytes
template <int MODE, int BYTES, int S, int ORDER = 0>
__global__ void __launch_bounds__(32, 1) stream_kernel(const __grid_constant__ CUtensorMap map, const uint8_t* base,
                                                       long long n_units, int* err) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t* buf = (uint8_t*)(((uintptr_t)sm + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t full[S];
  if (threadIdx.x != 0) return;
  for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  long long u = blockIdx.x;
  int issued = 0, done = 0;
  // units per CTA: blockIdx.x, +grid, ...
  const long long n_rb = n_units / 32;   // 128-row blocks of 32 k-tiles (16 KB units only)
  auto issue = [&](long long unit0, int s) {
    long long unit = unit0;
    if (ORDER == 1) {
      // this CTA's j-th unit: row block b + grid*(j/32), k-tile j%32 (a GEMM tile walk)
      const long long j = (unit0 - blockIdx.x) / gridDim.x;
      const long long rb = blockIdx.x + (long long)gridDim.x * (j / 32);
      unit = rb < n_rb ? rb * 32 + (j % 32) : n_units;   // past the end: no unit
      if (unit >= n_units) unit = blockIdx.x;            // keep counts equal (rare tail)
    }
    expect_tx(&full[s], MODE == 2 ? BYTES + 4096 + 1024 : BYTES);
    if (MODE == 2) {
      const int tiles_per_row = 4096 / 128;
      const long long r = unit / tiles_per_row, c = unit % tiles_per_row;
      tma2d(buf + s * (BYTES + 8192), &map, &full[s], (int)(c * 128), (int)(r * (BYTES / 128)));
      bulk(buf + s * (BYTES + 8192) + BYTES, base + (c * 4096) % (1 << 20), 4096, &full[s]);
      bulk(buf + s * (BYTES + 8192) + BYTES + 4096, base + (2ll << 30) + unit * 512, 512, &full[s]);
      bulk(buf + s * (BYTES + 8192) + BYTES + 4608, base + (c * 512) % (1 << 16), 512, &full[s]);
    } else if (MODE == 0) {
      const int tiles_per_row = 4096 / 128;
      const long long r = unit / tiles_per_row, c = unit % tiles_per_row;
      tma2d(buf + s * BYTES, &map, &full[s], (int)(c * 128), (int)(r * (BYTES / 128)));
    } else {
      bulk(buf + s * BYTES, base + unit * (long long)BYTES, BYTES, &full[s]);
    }
  };
  for (; issued < S && u + (long long)issued * gridDim.x < n_units; ++issued) issue(u + (long long)issued * gridDim.x, issued);
  uint32_t phase = 0;
  int s = 0;
  while (done < issued) {
    if (!wait_bounded(&full[s], phase, err)) return;
    ++done;
    const long long nu = u + (long long)(done + S - 1) * gridDim.x;
    if (nu < n_units) { issue(nu, s); ++issued; }
    if (++s == S) { s = 0; phase ^= 1; }
  }
}

int main() {
  const size_t total = 4ull << 30;   // 4 GB
  uint8_t* d;
  CK(cudaMalloc(&d, total));
  CK(cudaMemset(d, 1, total));
  int* err;
  CK(cudaMalloc(&err, 4));
  CK(cudaMemset(err, 0, 4));
  int sms;
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0));
  const uint64_t rows = total / 4096;
  auto run = [&](const char* name, auto kern, int bytes, int box_rows, int ctas, int stages, int extra = 0) {
    CUtensorMap m;
    cuuint64_t dims[2] = {4096, rows};
    cuuint64_t strides[1] = {4096};
    cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = cuTensorMapEncodeTiled(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, d, dims, strides, box, es,
                                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { printf("encode failed %d\n", (int)r); exit(1); }
    const long long units = (long long)(total / bytes);
    const int smem = stages * (bytes + extra) + 1024;
    CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    kern<<<ctas, 32, smem>>>(m, d, units, err);
    CK(cudaDeviceSynchronize());
    cudaEventRecord(a);
    const int it = 5;
    for (int i = 0; i < it; ++i) kern<<<ctas, 32, smem>>>(m, d, units, err);
    cudaEventRecord(b);
    CK(cudaDeviceSynchronize());
    float ms;
    cudaEventElapsedTime(&ms, a, b);
    int e;
    CK(cudaMemcpy(&e, err, 4, cudaMemcpyDeviceToHost));
    const double gbs = (double)total * it / (ms / 1e3) / 1e9;
    printf("%-30s stages %2d (%3d KB in flight) ctas %4d  %8.1f GB/s  %6.1f GB/s/CTA  err=%d\n", name, stages,
           stages * bytes / 1024, ctas, gbs, gbs / ctas, e);
  };
  const int ctas = sms;
  run("tma2d box 128x128 (16 KB)", stream_kernel<0, 16384, 6>, 16384, 128, ctas, 6);
  run("tma2d box 128x128 (16 KB)", stream_kernel<0, 16384, 12>, 16384, 128, ctas, 12);
  run("tma2d box 128x256 (32 KB)", stream_kernel<0, 32768, 6>, 32768, 256, ctas, 6);
  run("bulk 16 KB", stream_kernel<1, 16384, 6>, 16384, 128, ctas, 6);
  run("bulk 16 KB", stream_kernel<1, 16384, 12>, 16384, 128, ctas, 12);
  run("bulk 32 KB", stream_kernel<1, 32768, 6>, 32768, 128, ctas, 6);
  run("bulk 8 KB", stream_kernel<1, 8192, 16>, 8192, 128, ctas, 16);
  run("GEMM order: tma2d strided 16 KB", stream_kernel<0, 16384, 6, 1>, 16384, 128, ctas, 6);
  run("GEMM order: tma2d strided 16 KB", stream_kernel<0, 16384, 12, 1>, 16384, 128, ctas, 12);
  run("GEMM order: bulk contiguous 16 KB", stream_kernel<1, 16384, 6, 1>, 16384, 128, ctas, 6);
  run("GEMM stage: A 16K + B 4K + 2 SF", stream_kernel<2, 16384, 6, 1>, 16384, 128, ctas, 6, 8192);
  run("GEMM stage: A 16K + B 4K + 2 SF", stream_kernel<2, 16384, 8, 1>, 16384, 128, ctas, 8, 8192);
  return 0;
}
