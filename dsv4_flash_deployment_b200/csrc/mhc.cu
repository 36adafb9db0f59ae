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
// Kernel 1 (hc_partial) runs on a (D-slice, token-tile) grid with the slice of
// hc_fn held in shared memory, so hc_fn is read once per 64 tokens rather than
// once per token; it writes X', the collapse c, and per-slice partial sums.
// Kernel 2 (hc_finish) reduces the partials in a fixed order (deterministic),
// runs Sinkhorn and the norm/quantization per token.
#include "common.cuh"
#include "kernels.h"

namespace dsv4 {

constexpr int HC = 4;
constexpr int kSlice = 256;       // D-columns per CTA
constexpr int kTokTile = 32;      // tokens per CTA
constexpr int kNPart = 2 * HC + HC * HC + 2;  // 24 mixes + sumsq(X') + sumsq(c)

__global__ void __launch_bounds__(256) hc_partial_kernel(HcParams p) {
  extern __shared__ float fn_s[];  // [24][4][kSlice]
  const int slice = blockIdx.x;
  const int d0 = slice * kSlice;
  const int t0 = blockIdx.y * kTokTile;
  const int D = p.D;
  const bool mixes = p.fn != nullptr;
  if (mixes) {
    for (int e = threadIdx.x; e < 24 * HC * kSlice; e += blockDim.x) {
      const int m = e / (HC * kSlice), r = e % (HC * kSlice), i = r / kSlice, d = r % kSlice;
      fn_s[e] = (d0 + d < D) ? __ldg(p.fn + (size_t)m * HC * D + (size_t)i * D + d0 + d) : 0.f;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kPer = kSlice / 32;  // d's per lane
  for (int tt = warp; tt < kTokTile; tt += 8) {
    const int t = t0 + tt;
    if (t >= p.T) break;
    float part[24];
#pragma unroll
    for (int m = 0; m < 24; ++m) part[m] = 0.f;
    float ssx = 0.f, ssc = 0.f;
    float post[HC], comb[HC][HC], w[HC];
    const bool has_y = p.Y != nullptr || p.yperm != nullptr;
    if (has_y) {
#pragma unroll
      for (int i = 0; i < HC; ++i) post[i] = p.prev_mix[(size_t)t * 24 + HC + i];
#pragma unroll
      for (int i = 0; i < HC; ++i)
#pragma unroll
        for (int j = 0; j < HC; ++j) comb[i][j] = p.prev_mix[(size_t)t * 24 + 2 * HC + i * HC + j];
    }
    const bool collapse = p.cw != nullptr;
    if (collapse) {
#pragma unroll
      for (int i = 0; i < HC; ++i) w[i] = p.cw[(size_t)t * p.cw_stride + i];
    }
    __nv_bfloat16* xt = p.X + (size_t)t * HC * D;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int dl = lane + 32 * k;
      const int d = d0 + dl;
      if (d >= D) break;
      float xv[HC];
#pragma unroll
      for (int i = 0; i < HC; ++i) xv[i] = __bfloat162float(xt[(size_t)i * D + d]);
      if (has_y) {
        float y;
        if (p.yperm != nullptr) {
          float acc = 0.f;
          for (int s = 0; s < p.topk; ++s) {
            const int r = p.pos[(size_t)t * p.topk + s];
            if (r >= 0) acc += __bfloat162float(p.yperm[(size_t)r * D + d]);
          }
          if (p.Y) acc += __bfloat162float(p.Y[(size_t)t * D + d]);
          y = __bfloat162float(__float2bfloat16(acc));
        } else {
          y = __bfloat162float(p.Y[(size_t)t * D + d]);
        }
        float nx[HC];
#pragma unroll
        for (int j = 0; j < HC; ++j) {
          float a = post[j] * y;
#pragma unroll
          for (int i = 0; i < HC; ++i) a += comb[i][j] * xv[i];
          nx[j] = __bfloat162float(__float2bfloat16(a));
        }
#pragma unroll
        for (int j = 0; j < HC; ++j) {
          xv[j] = nx[j];
          xt[(size_t)j * D + d] = __float2bfloat16(nx[j]);
        }
      }
      if (p.tap) {
        const float mean = (xv[0] + xv[1] + xv[2] + xv[3]) * 0.25f;
        p.tap[(size_t)t * D + d] = __float2bfloat16(mean);
      }
      if (mixes) {
#pragma unroll
        for (int i = 0; i < HC; ++i) {
          ssx += xv[i] * xv[i];
#pragma unroll
          for (int m = 0; m < 24; ++m) part[m] += xv[i] * fn_s[(m * HC + i) * kSlice + dl];
        }
      }
      if (collapse) {
        float c = 0.f;
#pragma unroll
        for (int i = 0; i < HC; ++i) c += w[i] * xv[i];
        const __nv_bfloat16 cb = __float2bfloat16(c);
        p.c[(size_t)t * D + d] = cb;
        const float cf = __bfloat162float(cb);
        ssc += cf * cf;
      }
    }
    if (mixes || collapse) {
#pragma unroll
      for (int m = 0; m < 24; ++m) part[m] = warp_sum(part[m]);
      ssx = warp_sum(ssx);
      ssc = warp_sum(ssc);
      if (lane == 0) {
        float* dst = p.partials + ((size_t)t * gridDim.x + slice) * kNPart;
#pragma unroll
        for (int m = 0; m < 24; ++m) dst[m] = part[m];
        dst[24] = ssx;
        dst[25] = ssc;
      }
    }
  }
}

// One warp per token.
__global__ void __launch_bounds__(128) hc_finish_kernel(HcParams p, int n_slices) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + warp;
  if (t >= p.T) return;
  const int D = p.D;
  float ssc;
  {
    // fixed-order reduction over slices
    float v = 0.f;
    float mix[24];
    float ssx = 0.f;
    ssc = 0.f;
    for (int m = 0; m < 24; ++m) mix[m] = 0.f;
    for (int s = 0; s < n_slices; ++s) {
      const float* src = p.partials + ((size_t)t * n_slices + s) * kNPart;
      if (lane < kNPart) v = src[lane];
      for (int m = 0; m < 24; ++m) mix[m] += __shfl_sync(0xffffffffu, v, m);
      ssx += __shfl_sync(0xffffffffu, v, 24);
      ssc += __shfl_sync(0xffffffffu, v, 25);
    }
    if (p.fn != nullptr && lane == 0) {
      const float r = rsqrtf(ssx / (float)(HC * D) + p.norm_eps);
      float pre[HC], post[HC], comb[HC][HC];
      for (int i = 0; i < HC; ++i) {
        pre[i] = 1.f / (1.f + expf(-(mix[i] * r * p.scale[0] + p.base[i]))) + p.hc_eps;
        post[i] = 2.f / (1.f + expf(-(mix[HC + i] * r * p.scale[1] + p.base[HC + i])));
      }
      for (int i = 0; i < HC; ++i)
        for (int j = 0; j < HC; ++j) comb[i][j] = mix[2 * HC + i * HC + j] * r * p.scale[2] + p.base[2 * HC + i * HC + j];
      if (p.iters > 0) {
        for (int i = 0; i < HC; ++i) {
          float mx = comb[i][0];
          for (int j = 1; j < HC; ++j) mx = fmaxf(mx, comb[i][j]);
          float s = 0.f;
          for (int j = 0; j < HC; ++j) {
            comb[i][j] = expf(comb[i][j] - mx);
            s += comb[i][j];
          }
          for (int j = 0; j < HC; ++j) comb[i][j] = comb[i][j] / s + p.hc_eps;
        }
        for (int j = 0; j < HC; ++j) {
          float s = 0.f;
          for (int i = 0; i < HC; ++i) s += comb[i][j];
          for (int i = 0; i < HC; ++i) comb[i][j] /= (s + p.hc_eps);
        }
        for (int it = 1; it < p.iters; ++it) {
          for (int i = 0; i < HC; ++i) {
            float s = 0.f;
            for (int j = 0; j < HC; ++j) s += comb[i][j];
            for (int j = 0; j < HC; ++j) comb[i][j] /= (s + p.hc_eps);
          }
          for (int j = 0; j < HC; ++j) {
            float s = 0.f;
            for (int i = 0; i < HC; ++i) s += comb[i][j];
            for (int i = 0; i < HC; ++i) comb[i][j] /= (s + p.hc_eps);
          }
        }
      }
      float* o = p.mix_out + (size_t)t * 24;
      for (int i = 0; i < HC; ++i) {
        o[i] = pre[i];
        o[HC + i] = post[i];
      }
      for (int i = 0; i < HC; ++i)
        for (int j = 0; j < HC; ++j) o[2 * HC + i * HC + j] = comb[i][j];
    }
  }
  if (p.cw == nullptr || p.u == nullptr) return;
  // RMSNorm of the collapse, then MXFP8 quantization in 32-column blocks (one
  // block per lane-iteration: lane l covers columns 32*b + l).
  const float r = rsqrtf(ssc / (float)D + p.norm_eps);
  const __nv_bfloat16* c = p.c + (size_t)t * D;
  for (int b = 0; b < D / 32; ++b) {
    const int d = 32 * b + lane;
    const float y = __bfloat162float(c[d]) * r;
    const __nv_bfloat16 ub = __float2bfloat16(y * __bfloat162float(p.norm_w[d]));
    p.u[(size_t)t * D + d] = ub;
    if (p.uq) {
      const float uf = __bfloat162float(ub);
      const float amax = fmaxf(warp_max(fabsf(uf)), 1e-4f);
      const uint32_t e = pow2_ceil_exp(amax, 1.f / 448.f);
      p.uq[(size_t)t * D + d] = f32_to_e4m3(fminf(fmaxf(uf / exp_to_f32(e), -448.f), 448.f));
      if (lane == 0) p.usf[sf_chunk_offset(t, b, D / 128)] = (uint8_t)e;
    }
  }
}

int hc_num_slices(int D) { return (D + kSlice - 1) / kSlice; }

cudaError_t hc_step(const HcParams& p, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  const int ns = hc_num_slices(p.D);
  const int smem = p.fn ? 24 * HC * kSlice * 4 : 0;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(hc_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         24 * HC * kSlice * 4);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 g1(ns, (p.T + kTokTile - 1) / kTokTile);
  hc_partial_kernel<<<g1, 256, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (p.fn == nullptr && p.cw == nullptr) return cudaSuccess;
  hc_finish_kernel<<<(p.T + 3) / 4, 128, 0, st>>>(p, ns);
  return cudaGetLastError();
}

}  // namespace dsv4
