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
// Two launches per boundary:
//   hc_post    one pass over X per (16-token, 128-column) tile: X', the collapse c,
//              sums of squares, and the tile's share of the 24-mix projection on
//              tensor cores (mma.sync, bf16 operands, fp32 accumulate): hc_fn is
//              stored as bf16 hi + lo rows (fn = hi + lo to 2^-16), 48 outputs;
//   hc_finish  per token: fixed-order reduction of the per-slice partials,
//              Sinkhorn with one lane per comb entry, RMSNorm, MXFP8 quantization.
#include "common.cuh"
#include "kernels.h"
#include "peer.cuh"

namespace dsv4 {

constexpr int HC = 4;
constexpr int kSlice = 128;       // D-columns per CTA
constexpr int kTokTile = 16;      // tokens per CTA (one m16 MMA tile)
constexpr int kK = HC * kSlice;   // 512 = projection depth per CTA
constexpr int kRowE = kK + 8;     // padded smem row (bf16 elements)
constexpr int kNMix = 48;         // hi | lo rows of hc_fn
constexpr int kNPart = kNMix + 2; // + sumsq(X'), sumsq(c)

DSV4_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
DSV4_DEV void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
DSV4_DEV void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 256 threads.  Thread -> (token tid/16, 8 columns (tid%16)*8 of the slice).
constexpr int kMaxCombine = 8;   // routed experts per token summed by the MoE combine

__global__ void __launch_bounds__(256, 3) hc_post_kernel(HcParams p, int n_slices) {
  pdl_entry();
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sFn = reinterpret_cast<__nv_bfloat16*>(smem);                 // [48][kRowE]
  __nv_bfloat16* sX = sFn + kNMix * kRowE;                                      // [16][kRowE]
  // [8 warps][16][48] cross-warp sums of the mixes; aliases sFn, which is dead
  // once every warp's MMAs have read it (barrier below)
  float* sRed = reinterpret_cast<float*>(sFn);
  const int slice = blockIdx.x;
  const int t0 = blockIdx.y * kTokTile;
  const int D = p.D;
  const int d0 = slice * kSlice;
  const bool mixes = p.fn_hilo != nullptr;
  const bool has_y = p.Y != nullptr || p.yperm != nullptr || p.tp_mode != 0;
  const bool collapse = p.cw != nullptr;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (mixes) {
    // fn slice: rows 0..47, k = i*128 + c  <-  fn_hilo[row][i*D + d0 + c]
    for (int e = tid; e < kNMix * HC * (kSlice / 8); e += 256) {
      const int row = e / (HC * 16), r = e % (HC * 16), i = r / 16, ch = r % 16;
      const uint4 v = *reinterpret_cast<const uint4*>(p.fn_hilo + (size_t)row * HC * D + (size_t)i * D + d0 + ch * 8);
      *reinterpret_cast<uint4*>(sFn + row * kRowE + i * kSlice + ch * 8) = v;
    }
  }
  if (p.tp_mode) peer_wait(p.wait, p.err, KID_COMM);   // the fn slice load above overlaps the wait
  const int tt = tid >> 4;            // token within the tile
  const int cc = (tid & 15) * 8;      // column offset within the slice
  const int t = t0 + tt;
  const int d = d0 + cc;
  float ssx = 0.f, ssc = 0.f;
  float xn[HC][8];
  if (t < p.T) {
    __nv_bfloat16* xt = p.X + (size_t)t * HC * D;
#pragma unroll
    for (int i = 0; i < HC; ++i) {
      const uint4 raw = *reinterpret_cast<const uint4*>(xt + (size_t)i * D + d);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h2[k]);
        xn[i][2 * k] = f.x;
        xn[i][2 * k + 1] = f.y;
      }
    }
    if (has_y) {
      float y[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) y[k] = 0.f;
      // MoE combine: every pair's row index first, then all rows in flight, summed
      // in slot order (a per-slot index -> row load chain is 2 x topk round trips)
      if (p.tp_mode == 2 || p.yperm != nullptr) {
        const int k = min(p.topk, kMaxCombine);
        int rr[kMaxCombine];
        const __nv_bfloat16* src[kMaxCombine];
#pragma unroll
        for (int s = 0; s < kMaxCombine; ++s) {
          rr[s] = -1;
          src[s] = nullptr;
          if (s < k) {
            const size_t pi = (size_t)t * p.topk + s;
            if (p.tp_mode == 2) {   // each pair's row lives on the rank that owns its expert
              const int owner = p.ids[pi] / p.e_local;
              rr[s] = p.peer_pos[owner][pi];
              src[s] = p.peer_yperm[owner];
            } else {
              rr[s] = p.pos[pi];
              src[s] = p.yperm;
            }
          }
        }
        uint4 raw[kMaxCombine];
#pragma unroll
        for (int s = 0; s < kMaxCombine; ++s)
          if (rr[s] >= 0) raw[s] = *reinterpret_cast<const uint4*>(src[s] + (size_t)rr[s] * D + d);
#pragma unroll
        for (int s = 0; s < kMaxCombine; ++s) {
          if (rr[s] < 0) continue;
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[s]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __bfloat1622float2(h2[q]);
            y[2 * q] += f.x;
            y[2 * q + 1] += f.y;
          }
        }
      }
      if (p.tp_mode == 3) {
        // experts split over the ranks by intermediate index: every rank holds an
        // f32 partial row for every routed pair, at the row its own MoE plan gave
        // the pair (the order inside an expert segment comes from atomics, so it
        // differs between ranks: read each rank's row index from its pos table).
        // A pair's row is the rank-order sum of its partials rounded to bf16, as
        // the whole expert's W2 output is on one GPU; rows add in slot order, so
        // every rank gets the same bits and one GPU's rounding is reproduced
        // (without the per-row rounding the FP8 re-quantizations downstream
        // amplify the difference).
        const int k = min(p.topk, kMaxCombine);
        for (int s = 0; s < k; ++s) {
          float r8[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) r8[q] = 0.f;
          for (int rk = 0; rk < p.wait.world; ++rk) {
            const int rw = p.peer_pos[rk][(size_t)t * p.topk + s];
            if (rw < 0) continue;
            const float4* src = reinterpret_cast<const float4*>(p.peer_y[rk] + (size_t)rw * D + d);
            const float4 a = src[0], b = src[1];
            r8[0] += a.x; r8[1] += a.y; r8[2] += a.z; r8[3] += a.w;
            r8[4] += b.x; r8[5] += b.y; r8[6] += b.z; r8[7] += b.w;
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) y[q] += __bfloat162float(__float2bfloat16(r8[q]));
        }
      }
      if (p.tp_mode == 1) {
        // rank-order sum of the f32 partials: the same bits on every rank
#pragma unroll 8
        for (int rr = 0; rr < p.wait.world; ++rr) {
          const float4* src = reinterpret_cast<const float4*>(p.peer_y[rr] + (size_t)t * D + d);
          const float4 a = src[0], b = src[1];
          y[0] += a.x; y[1] += a.y; y[2] += a.z; y[3] += a.w;
          y[4] += b.x; y[5] += b.y; y[6] += b.z; y[7] += b.w;
        }
      } else if (p.Y != nullptr) {
        const uint4 raw = *reinterpret_cast<const uint4*>(p.Y + (size_t)t * D + d);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(h2[k]);
          y[2 * k] += f.x;
          y[2 * k + 1] += f.y;
        }
      }
      if (p.yperm != nullptr || p.tp_mode != 0) {   // the sublayer output is a bf16 tensor
#pragma unroll
        for (int k = 0; k < 8; ++k) y[k] = __bfloat162float(__float2bfloat16(y[k]));
      }
      const float* pm = p.prev_mix + (size_t)t * 24;
      float nx[HC][8];
#pragma unroll
      for (int j = 0; j < HC; ++j) {
        const float po = pm[HC + j];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float a = po * y[k];
#pragma unroll
          for (int i = 0; i < HC; ++i) a += pm[2 * HC + i * HC + j] * xn[i][k];
          nx[j][k] = __bfloat162float(__float2bfloat16(a));
        }
      }
#pragma unroll
      for (int j = 0; j < HC; ++j) {
        uint4 o;
        __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) o2[k] = __floats2bfloat162_rn(nx[j][2 * k], nx[j][2 * k + 1]);
        *reinterpret_cast<uint4*>(xt + (size_t)j * D + d) = o;
#pragma unroll
        for (int k = 0; k < 8; ++k) xn[j][k] = nx[j][k];
      }
    }
#pragma unroll
    for (int i = 0; i < HC; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) ssx += xn[i][k] * xn[i][k];
    if (p.tap) {
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float a = (xn[0][2 * k] + xn[1][2 * k] + xn[2][2 * k] + xn[3][2 * k]) * 0.25f;
        const float b = (xn[0][2 * k + 1] + xn[1][2 * k + 1] + xn[2][2 * k + 1] + xn[3][2 * k + 1]) * 0.25f;
        o2[k] = __floats2bfloat162_rn(a, b);
      }
      *reinterpret_cast<uint4*>(p.tap + (size_t)t * D + d) = o;
    }
    if (collapse) {
      const float* w = p.cw + (size_t)t * p.cw_stride;
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float a = 0.f, b = 0.f;
#pragma unroll
        for (int i = 0; i < HC; ++i) {
          a += w[i] * xn[i][2 * k];
          b += w[i] * xn[i][2 * k + 1];
        }
        o2[k] = __floats2bfloat162_rn(a, b);
        const float2 f = __bfloat1622float2(o2[k]);
        ssc += f.x * f.x + f.y * f.y;
      }
      *reinterpret_cast<uint4*>(p.c + (size_t)t * D + d) = o;
    }
  } else {
#pragma unroll
    for (int i = 0; i < HC; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) xn[i][k] = 0.f;
  }
  // per-token sums of squares: the 16 threads of a token are 16 consecutive lanes
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) {
    ssx += __shfl_xor_sync(0xffffffffu, ssx, o);
    ssc += __shfl_xor_sync(0xffffffffu, ssc, o);
  }
  float* part = p.partials;
  if (t < p.T && (tid & 15) == 0) {
    part[((size_t)t * n_slices + slice) * kNPart + kNMix] = ssx;
    part[((size_t)t * n_slices + slice) * kNPart + kNMix + 1] = ssc;
  }
  if (!mixes) return;
  // X' tile into shared memory as the A operand [16 tokens][k = i*128 + c]
#pragma unroll
  for (int i = 0; i < HC; ++i) {
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) o2[k] = __floats2bfloat162_rn(xn[i][2 * k], xn[i][2 * k + 1]);
    *reinterpret_cast<uint4*>(sX + tt * kRowE + i * kSlice + cc) = o;
  }
  __syncthreads();
  // [16 x 512] x [512 x 48]: warp w takes k in [64w, 64w+64), all six n8 tiles
  float acc[6][4];
#pragma unroll
  for (int n = 0; n < 6; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int k0 = warp * 64 + ks * 16;
    uint32_t a0, a1, a2, a3;
    ldsm_x4(smem_u32(sX + ((lane & 7) + 8 * ((lane >> 3) & 1)) * kRowE + k0 + 8 * (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
    for (int n = 0; n < 6; ++n) {
      uint32_t b0, b1;
      ldsm_x2(smem_u32(sFn + (n * 8 + (lane & 7)) * kRowE + k0 + 8 * ((lane >> 3) & 1)), b0, b1);
      mma16816(acc[n], a0, a1, a2, a3, b0, b1);
    }
  }
  __syncthreads();   // every warp is done reading sFn before sRed overwrites it
  const int g = lane >> 2, cq = lane & 3;
#pragma unroll
  for (int n = 0; n < 6; ++n) {
    sRed[(warp * 16 + g) * kNMix + n * 8 + 2 * cq] = acc[n][0];
    sRed[(warp * 16 + g) * kNMix + n * 8 + 2 * cq + 1] = acc[n][1];
    sRed[(warp * 16 + g + 8) * kNMix + n * 8 + 2 * cq] = acc[n][2];
    sRed[(warp * 16 + g + 8) * kNMix + n * 8 + 2 * cq + 1] = acc[n][3];
  }
  __syncthreads();
  for (int e = tid; e < kTokTile * kNMix; e += 256) {
    const int r = e / kNMix, c = e % kNMix;
    if (t0 + r >= p.T) continue;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) v += sRed[(w * 16 + r) * kNMix + c];
    part[((size_t)(t0 + r) * n_slices + slice) * kNPart + c] = v;
  }
}

// One CTA (4 warps) per token.  Partials per slice: 48 projections (hi | lo
// rows of hc_fn), sumsq(X'), sumsq(c); every warp reduces them in slice order
// (8 slices' loads in flight), warp 0 forms the mixes and runs Sinkhorn, and the
// four warps share the RMSNorm + MXFP8 pass over the D columns.
constexpr int kFinMaxIt = 5;   // norm pass: 1024 columns per iteration, D <= 5120

__global__ void __launch_bounds__(128) hc_finish_kernel(HcParams p, int n_slices) {
  pdl_entry();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x;
  if (t >= p.T) return;
  const int D = p.D;
  const bool do_norm = p.cw != nullptr && p.u != nullptr;
  // the collapse row and the norm weights do not depend on the partials: load them first
  uint4 craw[kFinMaxIt], wraw[kFinMaxIt];
  if (do_norm) {
#pragma unroll
    for (int i = 0; i < kFinMaxIt; ++i) {
      const int d0 = warp * 256 + i * 1024 + lane * 8;
      if (d0 < D) {
        craw[i] = *reinterpret_cast<const uint4*>(p.c + (size_t)t * D + d0);
        wraw[i] = *reinterpret_cast<const uint4*>(p.norm_w + d0);
      }
    }
  }
  // partial sums: warp w adds slices w, w+4, ... (loads in flight), then the four
  // warp sums combine in warp order; lane holds columns lane and 32 + lane (< 50)
  const float* part = p.partials + (size_t)t * n_slices * kNPart;
  const bool hi_lane = lane + 32 < kNPart;
  float r0 = 0.f, r1 = 0.f;
#pragma unroll 4
  for (int s = warp; s < n_slices; s += 4) {
    r0 += part[s * kNPart + lane];
    if (hi_lane) r1 += part[s * kNPart + 32 + lane];
  }
  __shared__ float s_part[4][64];
  s_part[warp][lane] = r0;
  s_part[warp][32 + lane] = r1;
  __syncthreads();
  r0 = ((s_part[0][lane] + s_part[1][lane]) + s_part[2][lane]) + s_part[3][lane];
  r1 = ((s_part[0][32 + lane] + s_part[1][32 + lane]) + s_part[2][32 + lane]) + s_part[3][32 + lane];
  const float ssx = __shfl_sync(0xffffffffu, r1, kNMix - 32);
  const float ssc = __shfl_sync(0xffffffffu, r1, kNMix + 1 - 32);
  if (p.fn_hilo != nullptr && warp == 0) {
    // lanes 0-3 pre, 4-7 post, 16-31 comb[i][j] with i = (lane-16)/4, j = lane%4
    const int idx = lane < 8 ? lane : (lane >= 16 ? 8 + lane - 16 : -1);
    const float r = rsqrtf(ssx / (float)(HC * D) + p.norm_eps);
    // projection m = hi[m] + lo[m] = column m + column 24 + m
    const float hi_lo0 = __shfl_sync(0xffffffffu, r0, idx < 0 ? 0 : idx);          // hi rows 0..23 live in r0
    const int lo_col = 24 + (idx < 0 ? 0 : idx);                                    // 24..47
    const float lo_a = __shfl_sync(0xffffffffu, r0, lo_col & 31);
    const float lo_b = __shfl_sync(0xffffffffu, r1, lo_col & 31);
    const float lo = lo_col < 32 ? lo_a : lo_b;
    float v = 0.f;
    if (idx >= 0) v = (hi_lo0 + lo) * r * p.scale[idx < HC ? 0 : (idx < 2 * HC ? 1 : 2)] + p.base[idx];
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
  if (!do_norm) return;
  // RMSNorm of the collapse + MXFP8: lane owns 8 consecutive columns of each
  // 256-column chunk; 4 lanes cover one 32-column scale block.
  const float rr = rsqrtf(ssc / (float)D + p.norm_eps);
#pragma unroll
  for (int i = 0; i < kFinMaxIt; ++i) {
    const int d0 = warp * 256 + i * 1024 + lane * 8;
    if (d0 >= D) break;
    const uint4 raw = craw[i];
    const uint4 wr = wraw[i];
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
  if ((p.yperm != nullptr || p.tp_mode >= 2) && p.topk > kMaxCombine) return cudaErrorInvalidValue;
  if (p.D % kSlice) return cudaErrorInvalidValue;
  const int ns = hc_num_slices(p.D);
  const size_t smem = (size_t)(kNMix + kTokTile) * kRowE * 2;
  static_assert((size_t)8 * kTokTile * kNMix * 4 <= (size_t)kNMix * kRowE * 2, "sRed must fit in sFn");
  static std::atomic<uint64_t> smem_set{0};
  {
    const cudaError_t e = smem_attr_once(hc_post_kernel, (int)smem, smem_set);
    if (e != cudaSuccess) return e;
  }
  dim3 g(ns, (p.T + kTokTile - 1) / kTokTile);
  launch_pdl(hc_post_kernel, g, 256, smem, st, p, ns);
  return cudaGetLastError();
}

cudaError_t hc_finish(const HcParams& p, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  if (p.D % 256 || p.D > 1024 * kFinMaxIt) return cudaErrorInvalidValue;
  launch_pdl(hc_finish_kernel, p.T, 128, 0, st, p, hc_num_slices(p.D));
  return cudaGetLastError();
}

}  // namespace dsv4
