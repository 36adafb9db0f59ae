// Router top-k of one token, shared by the router kernel (moe.cu) and the fused
// expert-parallel dispatch (ep.cu).
//
// scores = sqrt(softplus(logit)) (V4 family) or sigmoid(logit); experts = top-k
// of (score + bias), ties to the lower expert id; weights = score / sum(score)
// * route_scale (reference.py:355-382).  One warp per token; register arrays
// are only indexed by unrolled loop counters (no local memory); lane k < topk
// ends up holding the k-th pick.  kMaxPer = experts per lane (ceil(E / 32)).
#pragma once
#include "common.cuh"

namespace dsv4 {

template <int kMaxPer>
DSV4_DEV void route_token(const float* __restrict__ logit_row, int E, const float* __restrict__ bias, int topk,
                          int score_func, float route_scale, int lane, int& my_id, float& my_w) {
  float sc[kMaxPer], key[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lane + 32 * i;
    sc[i] = 0.f;
    key[i] = -INFINITY;
    if (e < E) {
      const float x = logit_row[e];
      float sv;
      if (score_func == 1) {
        sv = 1.f / (1.f + expf(-x));
      } else {
        const float sp = x > 20.f ? x : log1pf(expf(x));
        sv = sqrtf(sp);
      }
      sc[i] = sv;
      key[i] = sv + (bias ? bias[e] : 0.f);
    }
  }
  float my_s = 0.f, total = 0.f;
  my_id = 0;
  uint32_t taken = 0;   // bit i: this lane's element i is already chosen
  for (int k = 0; k < topk; ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      if (!((taken >> i) & 1u) && key[i] > bv) {
        bv = key[i];
        bi = lane + 32 * i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    float sv = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
      if (i == (bi >> 5)) sv = sc[i];
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    sv = __shfl_sync(0xffffffffu, sv, bi & 31);
    if (lane == k) {
      my_s = sv;
      my_id = bi;
    }
    total += sv;
  }
  const float inv = topk > 1 ? 1.f / (total + 1e-20f) : 1.f;
  my_w = my_s * inv * route_scale;
}

}  // namespace dsv4
