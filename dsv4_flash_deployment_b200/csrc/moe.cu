// MoE routing, dispatch planning and token permutation.
//
// router_topk: scores = sqrt(softplus(logit)) (V4 family) or sigmoid(logit);
//   experts = top-k of (score + bias) (ties -> lower expert id); weights =
//   score / sum(score) * route_scale (reference.py:355-382).  One warp per token.
// router_small: the gate GEMV and the top-k in one launch for decode-sized T.
// moe_plan: per-expert counts -> 128-row-aligned segments of the permuted
//   activation buffer (tiles under 128 rows get a 128-row slot each, seg_rows)
//   activation buffer -> GEMM tile lists for W13 and W2 (device-built, so the
//   whole MoE block replays inside a CUDA graph) -> permuted row of every
//   (token, slot) and its routing weight.
// moe_scatter: copies MXFP8 token rows and their scale bytes into permuted order.
#include "common.cuh"
#include "kernels.h"
#include "moe_route.cuh"

namespace dsv4 {

// One warp per token (route_token in moe_route.cuh); lane k < topk writes the k-th pick.
template <int kMaxPer>
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, int T, int E,
                                                          const float* __restrict__ bias, int topk, int score_func,
                                                          float route_scale, int* ids, float* wts) {
  pdl_entry();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  int my_id;
  float my_w;
  route_token<kMaxPer>(logits + (size_t)warp * E, E, bias, topk, score_func, route_scale, lane, my_id, my_w);
  if (lane < topk) {
    ids[(size_t)warp * topk + lane] = my_id;
    wts[(size_t)warp * topk + lane] = my_w;
  }
}

// Small-T router (decode steps): logits = u . gate_w^T on CUDA cores (fp32
// accumulation of the bf16 products), two warps per expert for every token, 4
// experts per CTA; the last CTA to finish (device counter; nothing waits) copies
// each token's logits to shared memory with L2 loads and runs its top-k
// (route_token), then re-arms the counter.  Replaces a split-K tensor-core GEMM
// plus a separate top-k launch where the gate matrix is a few MB.
constexpr int kRouterSmallChunks = 12;   // 16-byte pieces per lane: two warps per row, D <= 6144

template <int kMaxPer>
__global__ void __launch_bounds__(256) router_small_kernel(RouterSmallParams p) {
  pdl_entry();
  __shared__ float s_log[kRouterSmallMaxT][512];
  __shared__ float s_half[8][kRouterSmallMaxT];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 4 + (warp >> 1), half = warp & 1;   // two warps per gate row
  float acc[kRouterSmallMaxT];
#pragma unroll
  for (int t = 0; t < kRouterSmallMaxT; ++t) acc[t] = 0.f;
  if (e < p.E) {
    const __nv_bfloat16* wr = p.w + (size_t)e * p.D;
    // every 16-byte piece of this lane's share of the gate row is requested before
    // any is used (one DRAM round trip, not one per piece)
    uint4 wv[kRouterSmallChunks];
#pragma unroll
    for (int c = 0; c < kRouterSmallChunks; ++c) {
      const int d = lane * 8 + (2 * c + half) * 256;
      wv[c] = d < p.D ? *reinterpret_cast<const uint4*>(wr + d) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int t = 0; t < kRouterSmallMaxT; ++t) {
      if (t >= p.T) break;
      uint4 uv[kRouterSmallChunks];
#pragma unroll
      for (int c = 0; c < kRouterSmallChunks; ++c) {
        const int d = lane * 8 + (2 * c + half) * 256;
        uv[c] = d < p.D ? *reinterpret_cast<const uint4*>(p.u + (size_t)t * p.D + d) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int c = 0; c < kRouterSmallChunks; ++c) {
        const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv[c]);
        const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv[c]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 a = __bfloat1622float2(w2[i]), b = __bfloat1622float2(u2[i]);
          acc[t] += a.x * b.x + a.y * b.y;
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kRouterSmallMaxT; ++t) {
    const float v = warp_sum(acc[t]);
    if (lane == 0) s_half[warp][t] = v;
  }
  __syncthreads();
  if (half == 0 && lane < p.T && e < p.E)
    p.logits[(size_t)lane * p.E + e] = s_half[warp][lane] + s_half[warp + 1][lane];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(p.counter, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < p.T * p.E; i += blockDim.x) s_log[i / p.E][i % p.E] = __ldcg(p.logits + i);
  __syncthreads();
  if (warp < p.T) {
    int my_id;
    float my_w;
    route_token<kMaxPer>(s_log[warp], p.E, p.bias, p.topk, p.score_func, p.route_scale, lane, my_id, my_w);
    if (lane < p.topk) {
      p.ids[(size_t)warp * p.topk + lane] = my_id;
      p.wts[(size_t)warp * p.topk + lane] = my_w;
    }
  }
  if (threadIdx.x == 0) *p.counter = 0;
}

cudaError_t router_small(const RouterSmallParams& p, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  if (p.T > kRouterSmallMaxT || p.E > 512 || p.topk > 16 || p.topk > p.E || p.D % 256 ||
      p.D > 512 * kRouterSmallChunks || p.counter == nullptr)
    return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)((p.E + 3) / 4);
  const int per = (p.E + 31) / 32;
  if (per <= 2) launch_pdl(router_small_kernel<2>, grid, 256, 0, st, p);
  else if (per <= 4) launch_pdl(router_small_kernel<4>, grid, 256, 0, st, p);
  else if (per <= 8) launch_pdl(router_small_kernel<8>, grid, 256, 0, st, p);
  else if (per <= 12) launch_pdl(router_small_kernel<12>, grid, 256, 0, st, p);
  else launch_pdl(router_small_kernel<16>, grid, 256, 0, st, p);
  return cudaGetLastError();
}

cudaError_t router_topk(const float* logits, int T, int E, const float* bias, int topk, int score_func,
                        float route_scale, int* ids, float* wts, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (E > 512 || topk > 16 || topk > E) return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)((T * 32 + 255) / 256);
  const int per = (E + 31) / 32;
#define DSV4_ROUTER(P) \
  launch_pdl(router_topk_kernel<P>, grid, 256, 0, st, logits, T, E, bias, topk, score_func, route_scale, ids, wts)
  if (per <= 2) DSV4_ROUTER(2);
  else if (per <= 4) DSV4_ROUTER(4);
  else if (per <= 8) DSV4_ROUTER(8);
  else if (per <= 12) DSV4_ROUTER(12);
  else DSV4_ROUTER(16);
#undef DSV4_ROUTER
  return cudaGetLastError();
}

// Single CTA of 1024 threads: counts, scan, tiles, positions.
__global__ void __launch_bounds__(1024) moe_plan_kernel(MoePlanParams p) {
  pdl_entry();
  extern __shared__ int sh[];
  int* cnt = sh;                        // [E_local]
  int* start = sh + p.E_local;          // [E_local + 1]
  int* toff = sh + 2 * p.E_local + 1;   // [E_local + 1] row-tile offsets
  __shared__ int s_ok;
  const int n = p.T * p.topk;
  const int mt13 = p.m13 / 128, mt2 = p.m2 / 128;
  for (int e = threadIdx.x; e < p.E_local; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  // entries to visit: all n, or the valid prefix of each receive segment
  const int n_seg = p.seg_cnt ? n / p.seg_cap : 1;
  const int seg_len = p.seg_cnt ? p.seg_cap : n;
  for (int sg = 0; sg < n_seg; ++sg) {
    const int c = p.seg_cnt ? min(p.seg_cnt[sg], p.seg_cap) : n;
    for (int j = threadIdx.x; j < c; j += blockDim.x) {
      const int i = sg * seg_len + j;
      const int e = p.ids[i] - p.e_begin;
      if (e >= 0 && e < p.E_local) p.rank[i] = atomicAdd(&cnt[e], 1);
    }
  }
  __syncthreads();
  {
    // exclusive scans of the 128-aligned row counts and the row-tile counts,
    // one expert per thread (E_local <= 1024): warp scans, then warp totals
    __shared__ int s_wrows[32], s_wtiles[32];
    const int e = threadIdx.x;
    const int lane = e & 31, w = e >> 5;
    const int c = e < p.E_local ? cnt[e] : 0;
    const int rows = seg_rows(c, p.tile_rows);
    const int tl = (c + p.tile_rows - 1) / p.tile_rows;
    int ir = rows, it = tl;   // inclusive within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, ir, o), b = __shfl_up_sync(0xffffffffu, it, o);
      if (lane >= o) {
        ir += a;
        it += b;
      }
    }
    if (lane == 31) {
      s_wrows[w] = ir;
      s_wtiles[w] = it;
    }
    __syncthreads();
    if (w == 0) {
      const int nw = (int)(blockDim.x >> 5);
      int vr = lane < nw ? s_wrows[lane] : 0, vt = lane < nw ? s_wtiles[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, vr, o), b = __shfl_up_sync(0xffffffffu, vt, o);
        if (lane >= o) {
          vr += a;
          vt += b;
        }
      }
      s_wrows[lane] = vr;   // inclusive totals through warp `lane`
      s_wtiles[lane] = vt;
    }
    __syncthreads();
    const int base_r = w > 0 ? s_wrows[w - 1] : 0, base_t = w > 0 ? s_wtiles[w - 1] : 0;
    if (e < p.E_local) {
      start[e] = base_r + ir - rows;
      toff[e] = base_t + it - tl;
    }
    if (e == p.E_local - 1) {
      const int acc = base_r + ir, tacc = base_t + it;
      start[p.E_local] = acc;
      toff[p.E_local] = tacc;
      const int st = (p.shared_rows + p.tile_rows - 1) / p.tile_rows;   // shared expert row tiles
      const bool ok = acc <= p.cap_rows && (tacc + st) * mt13 <= p.max_tiles13 && (tacc + st) * mt2 <= p.max_tiles2 &&
                      (p.shared_rows == 0 || acc <= p.shared_row0);
      if (!ok) report_error(p.err, ERR_CAPACITY, KID_MOE, 1);
      s_ok = ok;
      *p.n_tiles13 = ok ? (tacc + st) * mt13 : 0;  // run nothing rather than overrun the buffers
      *p.n_tiles2 = ok ? (tacc + st) * mt2 : 0;
    }
  }
  __syncthreads();
  const bool ok = s_ok;
  for (int e = threadIdx.x; e < p.E_local; e += blockDim.x) {
    p.counts[e] = cnt[e];
    p.seg_start[e] = start[e];
    if (!ok) continue;
    const int c = cnt[e];
    int rt = toff[e];
    for (int r0 = 0; r0 < c; r0 += p.tile_rows, ++rt) {
      const int valid = min(p.tile_rows, c - r0);
      const int b0 = start[e] + seg_tile_row(r0, p.tile_rows);
      for (int mt = 0; mt < mt13; ++mt)
        p.tiles13[(size_t)rt * mt13 + mt] = make_int4(e * p.m13 + mt * 128, b0, valid, mt * 128);
      for (int mt = 0; mt < mt2; ++mt)
        p.tiles2[(size_t)rt * mt2 + mt] = make_int4(e * p.m2 + mt * 128, b0, valid, mt * 128);
    }
  }
  if (ok && p.shared_rows > 0) {
    // the shared expert: row tiles after the routed ones, weights from the second operand
    const int st = (p.shared_rows + p.tile_rows - 1) / p.tile_rows, t0 = toff[p.E_local];
    for (int i = threadIdx.x; i < st * mt13; i += blockDim.x) {
      const int j = i / mt13, mt = i % mt13;
      p.tiles13[(size_t)(t0 + j) * mt13 + mt] = make_int4(kTileA2 | (mt * 128), p.shared_row0 + j * p.tile_rows,
                                                          min(p.tile_rows, p.shared_rows - j * p.tile_rows), mt * 128);
    }
    for (int i = threadIdx.x; i < st * mt2; i += blockDim.x) {
      const int j = i / mt2, mt = i % mt2;
      p.tiles2[(size_t)(t0 + j) * mt2 + mt] = make_int4(kTileA2 | (mt * 128), p.shared_row0 + j * p.tile_rows,
                                                        min(p.tile_rows, p.shared_rows - j * p.tile_rows), mt * 128);
    }
    for (int t = threadIdx.x; t < p.shared_rows; t += blockDim.x) {
#ifdef DSV4_DEBUG_BOUNDS
      if (p.shared_row0 + t >= p.rs_rows) {
        dbg_bad(BS_MOE_ROW);
        break;
      }
#endif
      p.row_scale[p.shared_row0 + t] = 1.f;
    }
  }
  for (int sg = 0; sg < n_seg; ++sg) {
    const int c = p.seg_cnt ? min(p.seg_cnt[sg], p.seg_cap) : n;
    for (int j = threadIdx.x; j < c; j += blockDim.x) {
      const int i = sg * seg_len + j;
      const int e = p.ids[i] - p.e_begin;
      if (ok && e >= 0 && e < p.E_local) {
        const int row = start[e] + seg_row(p.rank[i], p.tile_rows);
        p.pos[i] = row;
#ifdef DSV4_DEBUG_BOUNDS
        if (row < 0 || row >= p.rs_rows) {
          dbg_bad(BS_MOE_ROW);
          p.pos[i] = -1;
          continue;
        }
#endif
        p.row_scale[row] = p.wts[i];
      } else {
        p.pos[i] = -1;
      }
    }
  }
}

cudaError_t moe_plan(const MoePlanParams& p, cudaStream_t st) {
  if (p.E_local < 1 || p.E_local > 1024) return cudaErrorInvalidValue;
  if (p.tile_rows != 32 && p.tile_rows != 64 && p.tile_rows != 128 && p.tile_rows != 256) return cudaErrorInvalidValue;
  if (p.seg_cnt && (p.seg_cap < 1 || (p.T * p.topk) % p.seg_cap)) return cudaErrorInvalidValue;
  if (p.shared_rows < 0 || (p.shared_rows > 0 && (p.tile_rows < 128 || p.shared_row0 % 256)))
    return cudaErrorInvalidValue;
  const int smem = (3 * p.E_local + 2) * 4;
  launch_pdl(moe_plan_kernel, 1, 1024, smem, st, p);
  return cudaGetLastError();
}

// One warp per (token, slot): 16-byte copies of the e4m3 row, then scale bytes;
// with a shared segment, the warps of slot 0 also copy the token to its row there.
__global__ void moe_scatter_kernel(const uint8_t* __restrict__ xq, const uint8_t* __restrict__ xsf, int T, int D,
                                   int topk, const int* __restrict__ pos, uint8_t* pq, uint8_t* psf, int shared_row0,
                                   int pq_rows) {
  pdl_entry();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= T * topk) return;
  const int t = w / topk;
  const uint4* src = reinterpret_cast<const uint4*>(xq + (size_t)t * D);
  const int kt = D / 128;
  const int rows[2] = {pos[w], (shared_row0 >= 0 && w % topk == 0) ? shared_row0 + t : -1};
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int row = rows[c];
    if (row < 0) continue;
#ifdef DSV4_DEBUG_BOUNDS
    if (row >= pq_rows) {
      dbg_bad(BS_MOE_ROW);
      continue;
    }
#endif
    uint4* dst = reinterpret_cast<uint4*>(pq + (size_t)row * D);
    for (int i = lane; i < D / 16; i += 32) dst[i] = src[i];
    for (int b = lane; b < D / 32; b += 32) psf[sf_chunk_offset(row, b, kt)] = xsf[sf_chunk_offset(t, b, kt)];
  }
}

cudaError_t moe_scatter(const uint8_t* xq, const uint8_t* xsf, int T, int D, int topk, const int* pos, uint8_t* pq,
                        uint8_t* psf, int shared_row0, int pq_rows, cudaStream_t st) {
  const long long warps = (long long)T * topk;
  if (warps == 0) return cudaSuccess;
  launch_pdl(moe_scatter_kernel, (unsigned)((warps * 32 + 255) / 256), 256, 0, st, xq, xsf, T, D, topk, pos, pq, psf,
             shared_row0, pq_rows);
  return cudaGetLastError();
}

}  // namespace dsv4
