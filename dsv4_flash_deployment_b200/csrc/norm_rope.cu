// Post-projection normalization, RoPE and quantization of the attention inputs.
//
// qkv_post: the fused wq_a|wkv GEMM output row is split into
//   qr = bf16(rmsnorm(q part) * q_norm)   -> MXFP8 for the wq_b / indexer GEMMs
//   kv = bf16(rmsnorm(kv part) * kv_norm) -> RoPE at pos (fp32, rounded to bf16)
//        -> FP8 e4m3 / ue8m0 per 32, stored as a KV8 record (kernels.h): the
//        window KV contract, kept in its quantized form
// (reference.py:704-731).
#include "common.cuh"
#include "kernels.h"

namespace dsv4 {

// One CTA (256 threads) per token.  Thread i owns the 8-column chunks i, i+256, ...
// of each part: every global load (row, norm weights, RoPE table) is issued up
// front as a 16-byte vector, one block reduction gives both sums of squares,
// and a 32-column scale block is 4 adjacent lanes (two shuffles).  At decode
// sizes the kernel is one memory round trip plus the reduction.
constexpr int kQkvThreads = 256;
constexpr int kQkvMaxJ = 1;   // chunks per thread: q_dim and kv_dim up to 2048

DSV4_DEV void ld8(const __nv_bfloat16* src, float* v) {
  const uint4 raw = *reinterpret_cast<const uint4*>(src);
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h2[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__global__ void __launch_bounds__(kQkvThreads) qkv_post_kernel(QkvParams p) {
  pdl_entry();
  const int t = blockIdx.x;
  if (t >= p.T) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nq = p.q_dim / 8, nk = p.kv_dim / 8;
  const __nv_bfloat16* in = p.in + (size_t)t * (p.q_dim + p.kv_dim);
  const __nv_bfloat16* kin = in + p.q_dim;
  const int pos = p.pos[t];
  float xq[kQkvMaxJ][8], wq[kQkvMaxJ][8], xk[kQkvMaxJ][8], wk[kQkvMaxJ][8], cs[kQkvMaxJ][8];
  float ssq = 0.f, ssk = 0.f;
#pragma unroll
  for (int j = 0; j < kQkvMaxJ; ++j) {
    const int c = tid + kQkvThreads * j;
    if (c < nq) {
      ld8(in + 8 * c, xq[j]);
      ld8(p.q_norm_w + 8 * c, wq[j]);
    }
    if (c < nk) {
      ld8(kin + 8 * c, xk[j]);
      ld8(p.kv_norm_w + 8 * c, wk[j]);
      if (8 * c >= p.kv_dim - 64) {   // RoPE on the last 64 dims: pairs (2i, 2i+1) -> table index i
        const int pi = (8 * c - (p.kv_dim - 64)) >> 1;
        const float4 co = *reinterpret_cast<const float4*>(p.rope_cos + (size_t)pos * 32 + pi);
        const float4 si = *reinterpret_cast<const float4*>(p.rope_sin + (size_t)pos * 32 + pi);
        cs[j][0] = co.x, cs[j][1] = co.y, cs[j][2] = co.z, cs[j][3] = co.w;
        cs[j][4] = si.x, cs[j][5] = si.y, cs[j][6] = si.z, cs[j][7] = si.w;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kQkvMaxJ; ++j) {
    const int c = tid + kQkvThreads * j;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (c < nq) ssq += xq[j][i] * xq[j][i];
      if (c < nk) ssk += xk[j][i] * xk[j][i];
    }
  }
  __shared__ float s_red[2][kQkvThreads / 32];
  ssq = warp_sum(ssq);
  ssk = warp_sum(ssk);
  if (lane == 0) {
    s_red[0][warp] = ssq;
    s_red[1][warp] = ssk;
  }
  __syncthreads();
  ssq = 0.f;
  ssk = 0.f;
#pragma unroll
  for (int w = 0; w < kQkvThreads / 32; ++w) {
    ssq += s_red[0][w];
    ssk += s_red[1][w];
  }
  const float rq = rsqrtf(ssq / (float)max(p.q_dim, 1) + p.eps);
  const float rk = rsqrtf(ssk / (float)p.kv_dim + p.eps);
#pragma unroll
  for (int j = 0; j < kQkvMaxJ; ++j) {
    const int c = tid + kQkvThreads * j;
    if (c < nq) {   // warp-uniform: nq is a multiple of 32
      float y[8], amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        y[i] = __bfloat162float(__float2bfloat16(xq[j][i] * rq * wq[j][i]));
        amax = fmaxf(amax, fabsf(y[i]));
      }
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const uint32_t e = pow2_ceil_exp(fmaxf(amax, 1e-4f), 1.f / 448.f);
      const float sc = exp_to_f32(e);
      uint32_t qb[2] = {0, 0};
#pragma unroll
      for (int i = 0; i < 8; ++i)
        qb[i >> 2] |= (uint32_t)f32_to_e4m3(fminf(fmaxf(y[i] / sc, -448.f), 448.f)) << (8 * (i & 3));
      *reinterpret_cast<uint2*>(p.qr_q + (size_t)t * p.q_dim + 8 * c) = make_uint2(qb[0], qb[1]);
      if ((lane & 3) == 0) p.qr_sf[sf_chunk_offset(t, c >> 2, p.q_dim / 128)] = (uint8_t)e;
    }
    if (c < nk) {   // warp-uniform: nk is a multiple of 32
      float y[8], amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = __bfloat162float(__float2bfloat16(xk[j][i] * rk * wk[j][i]));
      if (8 * c >= p.kv_dim - 64) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float ev = y[2 * i], od = y[2 * i + 1], co = cs[j][i], si = cs[j][4 + i];
          y[2 * i] = __bfloat162float(__float2bfloat16(ev * co - od * si));
          y[2 * i + 1] = __bfloat162float(__float2bfloat16(od * co + ev * si));
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(y[i]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const uint32_t e = pow2_ceil_exp(fmaxf(amax, 1e-4f), 1.f / 448.f);
      const float sc = exp_to_f32(e);
      // KV8 record: the e4m3 codes, then the ue8m0 exponent of each 32 columns
      uint8_t* rec = p.kv_out + (size_t)t * kv8_bytes(p.kv_dim);
      uint32_t qb[2] = {0, 0};
#pragma unroll
      for (int i = 0; i < 8; ++i)
        qb[i >> 2] |= (uint32_t)f32_to_e4m3(fminf(fmaxf(y[i] / sc, -448.f), 448.f)) << (8 * (i & 3));
      *reinterpret_cast<uint2*>(rec + 8 * c) = make_uint2(qb[0], qb[1]);
      if ((lane & 3) == 0) rec[p.kv_dim + (c >> 2)] = (uint8_t)e;
    }
  }
}

cudaError_t qkv_post(const QkvParams& p, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  if (p.q_dim % 256 || p.kv_dim % 256 || p.q_dim > 8 * kQkvThreads * kQkvMaxJ || p.kv_dim > 8 * kQkvThreads * kQkvMaxJ)
    return cudaErrorInvalidValue;
  launch_pdl(qkv_post_kernel, p.T, kQkvThreads, 0, st, p);
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
