// Host launchers of the element-wise / fused kernels (one .cu file each).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dsv4 {

// quant.cu
cudaError_t act_quant_mx(const __nv_bfloat16* x, int ldx, int T, int K, uint8_t* q, int ldq, uint8_t* sf,
                         int k_tiles, cudaStream_t st);
cudaError_t act_roundtrip(const __nv_bfloat16* x, __nv_bfloat16* y, long long n, cudaStream_t st);
cudaError_t fp4_roundtrip(const __nv_bfloat16* x, __nv_bfloat16* y, long long n, int block, int e4m3_scale,
                          cudaStream_t st);

}  // namespace dsv4
