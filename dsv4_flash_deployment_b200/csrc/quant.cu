// Activation quantization kernels (block-scaled formats of the model contract).
//
// act_quant_mx:     bf16 [T, K] -> e4m3 [T, K] + ue8m0 per 32 columns, scales
//                   written in the GEMM's 512-byte chunk layout.  Scale rule:
//                   s = 2^ceil(log2(max(amax, 1e-4)/448)) from IEEE bits, q =
//                   e4m3_rne(clamp(x/s, +-448)) (reference quant.py:110-145).
// act_roundtrip:    the same quantization followed by dequantization back to
//                   bf16 (the window-KV "inplace" act_quant).
// fp4_roundtrip:    e2m1 quantization with exact midpoint rounding (ties to
//                   even), scale either ue8m0 per 32 or e4m3 per 16, then
//                   dequantized to bf16 (quant.py:212-350).
#include "common.cuh"
#include "kernels.h"

namespace dsv4 {

// 4 threads per 32-element block, 8 elements per thread.
__global__ void act_quant_mx_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int T, int K,
                                    uint8_t* __restrict__ q, int ldq, uint8_t* __restrict__ sf, int k_tiles) {
  pdl_entry();
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = K / 8;
  const long long total = (long long)T * per_row;
  const bool active = gid < total;
  const int row = active ? (int)(gid / per_row) : 0;
  const int c8 = active ? (int)(gid % per_row) : 0;
  float v[8];
  float amax = 0.f;
  if (active) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + (size_t)row * ldx + c8 * 8);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  if (!active) return;
  const uint32_t e = pow2_ceil_exp(fmaxf(amax, 1e-4f), 1.f / 448.f);
  const float s = exp_to_f32(e);
  uint32_t packed[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float t = fminf(fmaxf(v[i] / s, -448.f), 448.f);
    packed[i >> 2] |= (uint32_t)f32_to_e4m3(t) << (8 * (i & 3));
  }
  *reinterpret_cast<uint2*>(q + (size_t)row * ldq + c8 * 8) = make_uint2(packed[0], packed[1]);
  if ((c8 & 3) == 0) sf[sf_chunk_offset(row, c8 >> 2, k_tiles)] = (uint8_t)e;
}

__global__ void act_roundtrip_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                     long long total8) {
  pdl_entry();
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = gid < total8;
  float v[8];
  float amax = 0.f;
  if (active) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + gid * 8);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  if (!active) return;
  const uint32_t e = pow2_ceil_exp(fmaxf(amax, 1e-4f), 1.f / 448.f);
  const float s = exp_to_f32(e);
  uint4 out;
  __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = e4m3_to_f32(f32_to_e4m3(fminf(fmaxf(v[2 * i] / s, -448.f), 448.f))) * s;
    const float b = e4m3_to_f32(f32_to_e4m3(fminf(fmaxf(v[2 * i + 1] / s, -448.f), 448.f))) * s;
    o2[i] = __floats2bfloat162_rn(a, b);
  }
  *reinterpret_cast<uint4*>(y + gid * 8) = out;
}

DSV4_DEV float e2m1_quant_dequant(float x, float s) {
  const float ax = fabsf(x);
  int c = (ax > 0.25f * s) + (ax >= 0.75f * s) + (ax > 1.25f * s) + (ax >= 1.75f * s) + (ax > 2.5f * s) +
          (ax >= 3.5f * s) + (ax > 5.0f * s);
  const float mag = c <= 4 ? 0.5f * c : (c == 5 ? 3.f : (c == 6 ? 4.f : 6.f));
  return (signbit(x) ? -mag : mag) * s;
}

// One thread per block of 16 (e4m3 scale) or 32 (ue8m0 scale) elements.
__global__ void fp4_roundtrip_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                     long long n_blocks, int block, int e4m3_scale) {
  pdl_entry();
  const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n_blocks) return;
  const __nv_bfloat16* src = x + b * block;
  float v[32];
  float amax = 0.f;
  for (int i = 0; i < block; ++i) {
    v[i] = __bfloat162float(src[i]);
    amax = fmaxf(amax, fabsf(v[i]));
  }
  float s;
  if (e4m3_scale) {
    amax = fmaxf(amax, 6.f * 0.001953125f);  // 6 * 2^-9
    s = e4m3_to_f32(f32_to_e4m3(amax / 6.f));
  } else {
    amax = fmaxf(amax, 6.f * 1.1754943508222875e-38f);  // 6 * 2^-126
    s = exp_to_f32(pow2_ceil_exp(amax, 1.f / 6.f));
  }
  __nv_bfloat16* dst = y + b * block;
  for (int i = 0; i < block; ++i) dst[i] = __float2bfloat16(e2m1_quant_dequant(v[i], s));
}

cudaError_t act_quant_mx(const __nv_bfloat16* x, int ldx, int T, int K, uint8_t* q, int ldq, uint8_t* sf,
                         int k_tiles, cudaStream_t st) {
  const long long total = (long long)T * (K / 8);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  launch_pdl(act_quant_mx_kernel, (unsigned)((total + threads - 1) / threads), threads, 0, st, x, ldx, T, K, q, ldq, sf,
                                                                                        k_tiles);
  return cudaGetLastError();
}

cudaError_t act_roundtrip(const __nv_bfloat16* x, __nv_bfloat16* y, long long n, cudaStream_t st) {
  const long long total8 = n / 8;
  if (total8 == 0) return cudaSuccess;
  launch_pdl(act_roundtrip_kernel, (unsigned)((total8 + 255) / 256), 256, 0, st, x, y, total8);
  return cudaGetLastError();
}

cudaError_t fp4_roundtrip(const __nv_bfloat16* x, __nv_bfloat16* y, long long n, int block, int e4m3_scale,
                          cudaStream_t st) {
  const long long nb = n / block;
  if (nb == 0) return cudaSuccess;
  launch_pdl(fp4_roundtrip_kernel, (unsigned)((nb + 255) / 256), 256, 0, st, x, y, nb, block, e4m3_scale);
  return cudaGetLastError();
}

}  // namespace dsv4
