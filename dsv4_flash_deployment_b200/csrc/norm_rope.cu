// Post-projection normalization, RoPE and quantization of the attention inputs.
//
// qkv_post: the fused wq_a|wkv GEMM output row is split into
//   qr = bf16(rmsnorm(q part) * q_norm)   -> MXFP8 for the wq_b / indexer GEMMs
//   kv = bf16(rmsnorm(kv part) * kv_norm) -> RoPE at pos (fp32, rounded to bf16)
//        -> FP8 e4m3 / ue8m0-per-32 round trip (the window KV contract)
// (reference.py:704-731).  One warp per token; lane l owns column 32*b + l of
// every 32-column block b, so a block's amax is one warp reduction.
#include "common.cuh"
#include "kernels.h"

namespace dsv4 {

// One CTA (4 warps) per token: every warp reduces the row's sums of squares
// (16-byte loads), then warp w handles the 32-column blocks w, w+4, ... of both
// parts.
__global__ void __launch_bounds__(128) qkv_post_kernel(QkvParams p) {
  pdl_entry();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x;
  if (t >= p.T) return;
  const __nv_bfloat16* in = p.in + (size_t)t * (p.q_dim + p.kv_dim);
  auto sumsq = [&](const __nv_bfloat16* x, int n) {
    float ss = 0.f;
#pragma unroll 4
    for (int d = lane * 8; d < n; d += 256) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + d);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
    return warp_sum(ss);
  };
  // ---- q part
  if (p.q_dim > 0) {
    const float ss = sumsq(in, p.q_dim);
    const float r = rsqrtf(ss / (float)p.q_dim + p.eps);
    for (int b = warp; b < p.q_dim / 32; b += 4) {
      const int d = 32 * b + lane;
      const float y = __bfloat162float(__float2bfloat16(__bfloat162float(in[d]) * r *
                                                        __bfloat162float(p.q_norm_w[d])));
      const float amax = fmaxf(warp_max(fabsf(y)), 1e-4f);
      const uint32_t e = pow2_ceil_exp(amax, 1.f / 448.f);
      p.qr_q[(size_t)t * p.q_dim + d] = f32_to_e4m3(fminf(fmaxf(y / exp_to_f32(e), -448.f), 448.f));
      if (lane == 0) p.qr_sf[sf_chunk_offset(t, b, p.q_dim / 128)] = (uint8_t)e;
    }
  }
  // ---- kv part
  {
    const __nv_bfloat16* kin = in + p.q_dim;
    const float ss = sumsq(kin, p.kv_dim);
    const float r = rsqrtf(ss / (float)p.kv_dim + p.eps);
    const int pos = p.pos[t];
    for (int b = warp; b < p.kv_dim / 32; b += 4) {
      const int d = 32 * b + lane;
      float y = __bfloat162float(__float2bfloat16(__bfloat162float(kin[d]) * r * __bfloat162float(p.kv_norm_w[d])));
      if (d >= p.kv_dim - 64) {
        const int pi = (d - (p.kv_dim - 64)) >> 1;
        const float c = p.rope_cos[(size_t)pos * 32 + pi], s = p.rope_sin[(size_t)pos * 32 + pi];
        const float other = __shfl_xor_sync(0xffffffffu, y, 1);
        y = (lane & 1) ? (other * s + y * c) : (y * c - other * s);
        y = __bfloat162float(__float2bfloat16(y));
      } else {
        (void)__shfl_xor_sync(0xffffffffu, y, 1);
      }
      const float amax = fmaxf(warp_max(fabsf(y)), 1e-4f);
      const float sc = exp_to_f32(pow2_ceil_exp(amax, 1.f / 448.f));
      const float qv = e4m3_to_f32(f32_to_e4m3(fminf(fmaxf(y / sc, -448.f), 448.f))) * sc;
      p.kv_out[(size_t)t * p.kv_dim + d] = __float2bfloat16(qv);
    }
  }
}

cudaError_t qkv_post(const QkvParams& p, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  if (p.q_dim % 256 || p.kv_dim % 256) return cudaErrorInvalidValue;
  launch_pdl(qkv_post_kernel, p.T, 128, 0, st, p);
  return cudaGetLastError();
}

DSV4_DEV float e2m1_qdq(float x, float s) {
  const float ax = fabsf(x);
  const int c = (ax > 0.25f * s) + (ax >= 0.75f * s) + (ax > 1.25f * s) + (ax >= 1.75f * s) + (ax > 2.5f * s) +
                (ax >= 3.5f * s) + (ax > 5.0f * s);
  const float mag = c <= 4 ? 0.5f * c : (c == 5 ? 3.f : (c == 6 ? 4.f : 6.f));
  return (signbit(x) ? -mag : mag) * s;
}

// One warp per (token, head); head_dim = 32 * k.
__global__ void idx_q_prep_kernel(__nv_bfloat16* q, int T, int H, int hd, const float* cos, const float* sin,
                                  const int* pos, const float* w_in, float w_scale, float* w_out) {
  pdl_entry();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= T * H) return;
  const int t = gw / H, h = gw % H;
  __nv_bfloat16* row = q + ((size_t)t * H + h) * hd;
  const int ps = pos[t];
  for (int b = 0; b < hd / 32; ++b) {
    const int d = 32 * b + lane;
    float y = __bfloat162float(row[d]);
    if (d >= hd - 64) {
      const int pi = (d - (hd - 64)) >> 1;
      const float c = cos[(size_t)ps * 32 + pi], s = sin[(size_t)ps * 32 + pi];
      const float other = __shfl_xor_sync(0xffffffffu, y, 1);
      y = (lane & 1) ? (other * s + y * c) : (y * c - other * s);
      y = __bfloat162float(__float2bfloat16(y));
    } else {
      (void)__shfl_xor_sync(0xffffffffu, y, 1);
    }
    const float amax = fmaxf(warp_max(fabsf(y)), 6.f * 1.1754943508222875e-38f);
    const float s = exp_to_f32(pow2_ceil_exp(amax, 1.f / 6.f));
    row[d] = __float2bfloat16(e2m1_qdq(y, s));
  }
  if (lane == 0 && w_out) {
    const float w = __bfloat162float(__float2bfloat16(w_in[(size_t)t * H + h])) * w_scale;
    w_out[(size_t)t * H + h] = __bfloat162float(__float2bfloat16(w));
  }
}

cudaError_t idx_q_prep(__nv_bfloat16* q, int T, int n_heads, int head_dim, const float* cos, const float* sin,
                       const int* pos, const float* w_in, float w_scale, float* w_out, cudaStream_t st) {
  const long long warps = (long long)T * n_heads;
  if (warps == 0) return cudaSuccess;
  launch_pdl(idx_q_prep_kernel, (unsigned)((warps * 32 + 255) / 256), 256, 0, st, q, T, n_heads, head_dim, cos, sin, pos,
                                                                        w_in, w_scale, w_out);
  return cudaGetLastError();
}

}  // namespace dsv4
