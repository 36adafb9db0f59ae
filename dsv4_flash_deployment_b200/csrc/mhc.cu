// Manifold hyper-connection (mHC) boundary kernels.
//
// Between two sublayers the 4 residual streams X[t, 4, D] are updated and the
// next sublayer's input is formed (reference.py:81-125, _block_step :840-891):
//
//   y      = sublayer output (attention row, or MoE combine: sum_k y_perm[pos[t,k]]
//            + shared[t], rounded to bf16)
//   X'[j]  = bf16( post[j] * y + sum_i comb[i][j] * X[i] )      (post/comb from the
//            mixes computed at the previous boundary)
//   m      = (flat(X') . hc_fn^T) * rsqrt(mean(flat(X')^2) + eps)   (24 mixes)
//   pre, post, comb = split + 20-iteration Sinkhorn of m          (next boundary)
//   c      = bf16( sum_i w[i] * X'[i] )   with the collapse weights w handed over
//            from the previous boundary
//   u      = bf16( rmsnorm(c) * norm_w ), then MXFP8-quantized for the next GEMM.
//
// Three launches per boundary:
//   hc_post    (memory bound) X' and c for a (token tile, D slice), with per-slice
//              partial sums of squares of X' and c;
//   mixes GEMM (tensor cores, issued by the host) flat(X') [T, 4D] x fn^T where
//              fn is stored as bf16 hi + lo rows (fn = hi + lo to 2^-16), so the
//              fp32 projection runs on tcgen05 with split-K;
//   hc_finish  per token: fixed-order reduction of the partials, Sinkhorn with one
//              lane per comb entry, RMSNorm and MXFP8 quantization.
#include "common.cuh"
#include "kernels.h"

namespace dsv4 {

constexpr int HC = 4;
constexpr int kSlice = 512;       // D-columns per CTA
constexpr int kTokTile = 16;      // tokens per CTA

// 256 threads: each thread owns 2 consecutive columns of the slice.
__global__ void __launch_bounds__(256) hc_post_kernel(HcParams p, int n_slices) {
  const int slice = blockIdx.x;
  const int t0 = blockIdx.y * kTokTile;
  const int D = p.D;
  const int d = slice * kSlice + 2 * threadIdx.x;
  const bool has_y = p.Y != nullptr || p.yperm != nullptr;
  const bool collapse = p.cw != nullptr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float red[8][2];
  for (int tt = 0; tt < kTokTile; ++tt) {
    const int t = t0 + tt;
    if (t >= p.T) break;
    float ssx = 0.f, ssc = 0.f;
    if (d < D) {
      __nv_bfloat16* xt = p.X + (size_t)t * HC * D;
      float2 xv[HC];
#pragma unroll
      for (int i = 0; i < HC; ++i) xv[i] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xt + (size_t)i * D + d));
      if (has_y) {
        float2 y;
        if (p.yperm != nullptr) {
          float2 acc = make_float2(0.f, 0.f);
          for (int s = 0; s < p.topk; ++s) {
            const int r = p.pos[(size_t)t * p.topk + s];
            if (r >= 0) {
              const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p.yperm + (size_t)r * D + d));
              acc.x += v.x;
              acc.y += v.y;
            }
          }
          if (p.Y) {
            const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p.Y + (size_t)t * D + d));
            acc.x += v.x;
            acc.y += v.y;
          }
          y = __bfloat1622float2(__floats2bfloat162_rn(acc.x, acc.y));
        } else {
          y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p.Y + (size_t)t * D + d));
        }
        const float* pm = p.prev_mix + (size_t)t * 24;
        float2 nx[HC];
#pragma unroll
        for (int j = 0; j < HC; ++j) {
          const float po = pm[HC + j];
          float ax = po * y.x, ay = po * y.y;
#pragma unroll
          for (int i = 0; i < HC; ++i) {
            const float cb = pm[2 * HC + i * HC + j];
            ax += cb * xv[i].x;
            ay += cb * xv[i].y;
          }
          const __nv_bfloat162 b = __floats2bfloat162_rn(ax, ay);
          *reinterpret_cast<__nv_bfloat162*>(xt + (size_t)j * D + d) = b;
          nx[j] = __bfloat1622float2(b);
        }
#pragma unroll
        for (int j = 0; j < HC; ++j) xv[j] = nx[j];
      }
#pragma unroll
      for (int i = 0; i < HC; ++i) ssx += xv[i].x * xv[i].x + xv[i].y * xv[i].y;
      if (p.tap) {
        const float mx = (xv[0].x + xv[1].x + xv[2].x + xv[3].x) * 0.25f;
        const float my = (xv[0].y + xv[1].y + xv[2].y + xv[3].y) * 0.25f;
        *reinterpret_cast<__nv_bfloat162*>(p.tap + (size_t)t * D + d) = __floats2bfloat162_rn(mx, my);
      }
      if (collapse) {
        const float* w = p.cw + (size_t)t * p.cw_stride;
        float cx = 0.f, cy = 0.f;
#pragma unroll
        for (int i = 0; i < HC; ++i) {
          cx += w[i] * xv[i].x;
          cy += w[i] * xv[i].y;
        }
        const __nv_bfloat162 cb = __floats2bfloat162_rn(cx, cy);
        *reinterpret_cast<__nv_bfloat162*>(p.c + (size_t)t * D + d) = cb;
        const float2 cf = __bfloat1622float2(cb);
        ssc = cf.x * cf.x + cf.y * cf.y;
      }
    }
    if (p.partials != nullptr) {
      ssx = warp_sum(ssx);
      ssc = warp_sum(ssc);
      if (lane == 0) {
        red[warp][0] = ssx;
        red[warp][1] = ssc;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        float a = 0.f, b = 0.f;
        for (int w = 0; w < 8; ++w) {
          a += red[w][0];
          b += red[w][1];
        }
        float* dst = p.partials + ((size_t)t * n_slices + slice) * 2;
        dst[0] = a;
        dst[1] = b;
      }
      __syncthreads();
    }
  }
}

// One warp per token.  mix_raw: [T, 48] = (hi | lo) halves of the projection.
__global__ void __launch_bounds__(128) hc_finish_kernel(HcParams p, int n_slices) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + warp;
  if (t >= p.T) return;
  const int D = p.D;
  float ssx = 0.f, ssc = 0.f;
  for (int s = lane; s < n_slices; s += 32) {
    ssx += p.partials[((size_t)t * n_slices + s) * 2];
    ssc += p.partials[((size_t)t * n_slices + s) * 2 + 1];
  }
  ssx = warp_sum(ssx);
  ssc = warp_sum(ssc);
  if (p.mix_raw != nullptr) {
    // lanes 0-3 pre, 4-7 post, 16-31 comb[i][j] with i = (lane-16)/4, j = lane%4
    const int idx = lane < 8 ? lane : (lane >= 16 ? 8 + lane - 16 : -1);
    const float r = rsqrtf(ssx / (float)(HC * D) + p.norm_eps);
    float v = 0.f;
    if (idx >= 0) {
      const float* raw = p.mix_raw + (size_t)t * 48;
      v = (raw[idx] + raw[24 + idx]) * r * p.scale[idx < HC ? 0 : (idx < 2 * HC ? 1 : 2)] + p.base[idx];
    }
    float outv = 0.f;
    if (lane < HC) outv = 1.f / (1.f + expf(-v)) + p.hc_eps;
    else if (lane < 2 * HC) outv = 2.f / (1.f + expf(-v));
    // Sinkhorn on lanes 16..31 (other lanes carry dummies through the shuffles)
    float c = (lane >= 16) ? v : 0.f;
    if (p.iters > 0) {
      float mx = fmaxf(c, __shfl_xor_sync(0xffffffffu, c, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      c = expf(c - mx);
      float rs = c + __shfl_xor_sync(0xffffffffu, c, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
      c = c / rs + p.hc_eps;
      float cs = c + __shfl_xor_sync(0xffffffffu, c, 4);
      cs += __shfl_xor_sync(0xffffffffu, cs, 8);
      c = c / (cs + p.hc_eps);
      for (int it = 1; it < p.iters; ++it) {
        rs = c + __shfl_xor_sync(0xffffffffu, c, 1);
        rs += __shfl_xor_sync(0xffffffffu, rs, 2);
        c = c / (rs + p.hc_eps);
        cs = c + __shfl_xor_sync(0xffffffffu, c, 4);
        cs += __shfl_xor_sync(0xffffffffu, cs, 8);
        c = c / (cs + p.hc_eps);
      }
    }
    if (lane >= 16) outv = c;
    if (idx >= 0) p.mix_out[(size_t)t * 24 + idx] = outv;
  }
  if (p.cw == nullptr || p.u == nullptr) return;
  // RMSNorm of the collapse + MXFP8: lane owns 8 consecutive columns of each
  // 256-column chunk; 4 lanes cover one 32-column scale block.
  const float rr = rsqrtf(ssc / (float)D + p.norm_eps);
  const __nv_bfloat16* c = p.c + (size_t)t * D;
  for (int base = 0; base < D; base += 256) {
    const int d0 = base + lane * 8;
    const uint4 raw = *reinterpret_cast<const uint4*>(c + d0);
    const uint4 wr = *reinterpret_cast<const uint4*>(p.norm_w + d0);
    const __nv_bfloat162* c2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wr);
    float uf[8];
    uint4 uo;
    __nv_bfloat162* u2 = reinterpret_cast<__nv_bfloat162*>(&uo);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 cv = __bfloat1622float2(c2[i]);
      const float2 wv = __bfloat1622float2(w2[i]);
      u2[i] = __floats2bfloat162_rn(cv.x * rr * wv.x, cv.y * rr * wv.y);
      const float2 ub = __bfloat1622float2(u2[i]);
      uf[2 * i] = ub.x;
      uf[2 * i + 1] = ub.y;
      amax = fmaxf(amax, fmaxf(fabsf(ub.x), fabsf(ub.y)));
    }
    *reinterpret_cast<uint4*>(p.u + (size_t)t * D + d0) = uo;
    if (p.uq) {
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const uint32_t e = pow2_ceil_exp(fmaxf(amax, 1e-4f), 1.f / 448.f);
      const float s = exp_to_f32(e);
      uint32_t q[2] = {0, 0};
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i >> 2] |= (uint32_t)f32_to_e4m3(fminf(fmaxf(uf[i] / s, -448.f), 448.f)) << (8 * (i & 3));
      *reinterpret_cast<uint2*>(p.uq + (size_t)t * D + d0) = make_uint2(q[0], q[1]);
      if ((lane & 3) == 0) p.usf[sf_chunk_offset(t, d0 >> 5, D / 128)] = (uint8_t)e;
    }
  }
}

int hc_num_slices(int D) { return (D + kSlice - 1) / kSlice; }

cudaError_t hc_post(const HcParams& p, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  const int ns = hc_num_slices(p.D);
  dim3 g(ns, (p.T + kTokTile - 1) / kTokTile);
  hc_post_kernel<<<g, 256, 0, st>>>(p, ns);
  return cudaGetLastError();
}

cudaError_t hc_finish(const HcParams& p, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  hc_finish_kernel<<<(p.T + 3) / 4, 128, 0, st>>>(p, hc_num_slices(p.D));
  return cudaGetLastError();
}

}  // namespace dsv4
