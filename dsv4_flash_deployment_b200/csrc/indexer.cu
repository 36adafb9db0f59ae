// Lightning-indexer scoring and top-k selection (reference.py:605-702).
//
// For query token t with causal compressed length clen:
//   raw[h, j]  = bf16(q[h] . k[j])                  (fp32 dot of bf16 values)
//   score[j]   = bf16( sum_h bf16(relu(raw[h, j]) * w[h]) )
// optional level-1 candidate mask (V4.1): layer 20 keeps the top cand_topk
// blocks of cand_block entries by block max (the block holding the newest
// entry is always kept); later indexers mask scores outside those blocks.
// Output: the top-k entries sorted by index ascending (ties broken toward the
// lower index); when clen <= topk every entry is selected, as top_k of a
// shorter list returns all of it.
//
// Two kernels:
//   idx_score   one CTA per (token, 64 compressed rows): the head x row dot
//               products on tensor cores (mma.sync m16n8k16, bf16 in, fp32
//               accumulate), then per row the head sum in fixed order h = 0..H-1
//               with the bf16 rounding points above; writes order-preserving keys
//   idx_select  one CTA per token: candidate-block mask (level 1), 4-pass radix
//               select and ordered compaction on the keys in shared memory
// Spreading the scoring over the compressed rows keeps long contexts (9K
// tokens = 2304 entries at ratio 4) from serializing on one CTA per token.
#include <cuda_fp4.h>

#include "common.cuh"
#include "kernels.h"
#include "mma_sync.cuh"

namespace dsv4 {

DSV4_DEV uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Returns the k-th largest key (1-based k) among keys[0..n) and the number of
// keys strictly greater than it.
DSV4_DEV void radix_select(const uint32_t* keys, int n, int k, uint32_t* hist, uint32_t& kth, int& n_greater) {
  __shared__ uint32_t s_prefix, s_mask, s_k;
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_k = k;
  }
  __syncthreads();
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t pre = s_prefix, msk = s_mask;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t key = keys[i];
      if ((key & msk) == pre) atomicAdd(&hist[(key >> shift) & 0xFF], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t need = s_k;
      int b = 255;
      for (; b > 0; --b) {
        if (hist[b] >= need) break;
        need -= hist[b];
      }
      s_prefix = pre | ((uint32_t)b << shift);
      s_mask = msk | (0xFFu << shift);
      s_k = need;
    }
    __syncthreads();
  }
  kth = s_prefix;
  // count strictly greater
  __shared__ int s_gt;
  if (threadIdx.x == 0) s_gt = 0;
  __syncthreads();
  int local = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) local += keys[i] > kth;
  atomicAdd(&s_gt, local);
  __syncthreads();
  n_greater = s_gt;
}

// Writes, in index order, every j with keys[j] > kth, plus the first (k - n_gt)
// indices with keys[j] == kth.  Block-wide ordered compaction, chunk by chunk.
DSV4_DEV int ordered_select(const uint32_t* keys, int n, uint32_t kth, int n_eq_take, int* out) {
  __shared__ int s_base, s_eq_base;
  __shared__ int s_warp[8], s_warp_eq[8];
  if (threadIdx.x == 0) {
    s_base = 0;
    s_eq_base = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int i = c0 + threadIdx.x;
    const uint32_t key = i < n ? keys[i] : 0u;
    const bool gt = i < n && key > kth;
    const bool eq = i < n && key == kth;
    const unsigned mg = __ballot_sync(0xffffffffu, gt), me = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) {
      s_warp[warp] = __popc(mg);
      s_warp_eq[warp] = __popc(me);
    }
    __syncthreads();
    int wo = 0, weo = 0;
    for (int w = 0; w < warp; ++w) {
      wo += s_warp[w];
      weo += s_warp_eq[w];
    }
    const int below = __popc(mg & ((1u << lane) - 1)), below_eq = __popc(me & ((1u << lane) - 1));
    const int eq_rank = s_eq_base + weo + below_eq;
    // selected entries before this one = gt so far + min(eq so far, n_eq_take)
    int tot_gt = 0, tot_eq = 0;
    for (int w = 0; w < 8; ++w) {
      tot_gt += s_warp[w];
      tot_eq += s_warp_eq[w];
    }
    if (gt || (eq && eq_rank < n_eq_take)) {
      const int gt_before = s_base + wo + below;  // gt entries strictly before i (global)
      const int eq_before = min(eq_rank, n_eq_take);
      out[gt_before + eq_before] = i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      s_base += tot_gt;
      s_eq_base += tot_eq;
    }
    __syncthreads();
  }
  return s_base + min(s_eq_base, n_eq_take);
}

constexpr int kIdxRows = 64;            // compressed rows per scoring CTA
constexpr int kIdxDh = 128;             // indexer head dim (both model families)
constexpr int kIdxPad = kIdxDh + 8;     // smem row stride (bf16) against bank conflicts
constexpr int kIk4 = ik4_bytes(kIdxDh);  // 68-byte key records (4-byte aligned)
constexpr int kIdxMaxHeads = 64;

DSV4_DEV float bf16r(float x) { return __bfloat162float(__float2bfloat16(x)); }

__global__ void __launch_bounds__(128) idx_score_kernel(IdxParams p, uint32_t* keys, int keys_ld) {
  pdl_entry();
  __shared__ __align__(16) __nv_bfloat16 sQ[kIdxMaxHeads * kIdxPad];
  __shared__ __align__(16) __nv_bfloat16 sK[kIdxRows * kIdxPad];
  __shared__ __nv_bfloat16 sS[kIdxMaxHeads * (kIdxRows + 2)];   // terms are bf16 values: exact
  __shared__ float sw[kIdxMaxHeads];
  const int t = blockIdx.x, r0 = blockIdx.y * kIdxRows;
  const int clen = p.clen[t];
  if (r0 >= clen) return;
  if (clen <= p.topk && p.cand_mode != 1) return;   // every entry is selected: no scores needed
  const int H = p.n_heads, Hp = (H + 15) & ~15;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int c = tid; c < Hp * (kIdxDh / 8); c += 128) {
    const int h = c / (kIdxDh / 8), ch = c % (kIdxDh / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h < H) v = *reinterpret_cast<const uint4*>(p.q + ((size_t)t * H + h) * kIdxDh + ch * 8);
    *reinterpret_cast<uint4*>(sQ + h * kIdxPad + ch * 8) = v;
  }
  if (tid < kIdxMaxHeads) sw[tid] = tid < H ? p.w[(size_t)t * H + tid] : 0.f;
  const int slot = p.slot[t];
  const bool use_alt = p.kcache_alt != nullptr && ((p.pos[t] + 1) % p.own_r) != 0 &&
                       p.chunk_start[t] == p.last_pos[t];
  const uint8_t* kc = use_alt ? p.kcache_alt : p.kcache;
  const KvPages kpg = use_alt ? p.alt_pages : p.pages;
  const int kmax = use_alt ? p.alt_max_c : p.max_c;
  // keys are IK4 records: 8 columns = one 4-byte word of e2m1 codes; the scale is
  // the ue8m0 byte of their 32-column block.  Decoded exactly to bf16.
  for (int c = tid; c < kIdxRows * (kIdxDh / 8); c += 128) {
    const int r = c / (kIdxDh / 8), ch = c % (kIdxDh / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r0 + r < clen) {
      const uint8_t* rec = kc + kv_row(kpg, slot, r0 + r, kmax) * kIk4;
      const uint32_t codes = *reinterpret_cast<const uint32_t*>(rec + 4 * ch);
      const uint32_t e = rec[kIdxDh / 2 + (ch >> 2)];
      const float sc = e ? __uint_as_float(e << 23) : 0.f;
      uint32_t* v32 = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {   // two e2m1 codes per hardware conversion (exact in f16)
        const __half2_raw hr =
            __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)((codes >> (8 * i)) & 0xFF), __NV_E2M1);
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
        v32[i] = pack_bf16(f.x * sc, f.y * sc);
      }
    }
    *reinterpret_cast<uint4*>(sK + r * kIdxPad + ch * 8) = v;
  }
  __syncthreads();
  // raw[h, j] = q_h . k_j : warp w takes rows 16w..16w+15, all head tiles
  const int n0 = warp * 16, g = lane >> 2, cq = lane & 3;
  const uint32_t ba = smem_u32(sK + (n0 + (lane & 7) + 8 * (lane >> 4)) * kIdxPad + 8 * ((lane >> 3) & 1));
  for (int mt = 0; mt < Hp / 16; ++mt) {
    float acc[2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[a][e] = 0.f;
    const uint32_t qa = smem_u32(sQ + (mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * kIdxPad + 8 * (lane >> 4));
#pragma unroll
    for (int k0 = 0; k0 < kIdxDh; k0 += 16) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      ldsm_x4(qa + k0 * 2, a0, a1, a2, a3);
      ldsm_x4(ba + k0 * 2, b0, b1, b2, b3);
      mma16816(acc[0], a0, a1, a2, a3, b0, b1);
      mma16816(acc[1], a0, a1, a2, a3, b2, b3);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = mt * 16 + g + 8 * (e >> 1);
        const int col = n0 + nt * 8 + 2 * cq + (e & 1);
        sS[h * (kIdxRows + 2) + col] = __float2bfloat16(fmaxf(bf16r(acc[nt][e]), 0.f) * sw[h]);
      }
  }
  __syncthreads();
  if (tid < kIdxRows && r0 + tid < clen) {
    float sum = 0.f;
    for (int h = 0; h < H; ++h) sum += __bfloat162float(sS[h * (kIdxRows + 2) + tid]);
    float sc = bf16r(sum);
    const int j = r0 + tid;
    if (p.cand_mode == 2 && !p.cand[(size_t)t * (p.max_c / p.cand_block) + j / p.cand_block]) sc = -INFINITY;
    keys[(size_t)t * keys_ld + j] = order_key(sc);
  }
}

__global__ void __launch_bounds__(256) idx_select_kernel(IdxParams p, const uint32_t* keys_in, int keys_ld) {
  pdl_entry();
  extern __shared__ uint8_t smem[];
  const int t = blockIdx.x;
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem);
  uint32_t* keys = hist + 256;
  const int clen = p.clen[t];
  const int k = p.topk;
  if (clen <= k) {
    for (int j = threadIdx.x; j < k; j += blockDim.x) p.out_idx[(size_t)t * k + j] = j < clen ? j : -1;
    if (threadIdx.x == 0) p.out_cnt[t] = clen;
    if (p.cand_mode != 1) return;
  }
  for (int j = threadIdx.x; j < clen; j += blockDim.x) keys[j] = keys_in[(size_t)t * keys_ld + j];
  __syncthreads();
  if (p.cand_mode == 1) {
    // block maxima (newest block forced in), top cand_topk blocks -> mask
    const int nb = (clen + p.cand_block - 1) / p.cand_block;
    uint32_t* bkeys = keys + clen;
    const int last = (clen - 1) / p.cand_block;
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
      uint32_t m = 0;
      for (int j = b * p.cand_block; j < min(clen, (b + 1) * p.cand_block); ++j) m = max(m, keys[j]);
      bkeys[b] = (b == last) ? order_key(INFINITY) : m;
    }
    __syncthreads();
    uint8_t* cand = p.cand + (size_t)t * (p.max_c / p.cand_block);
    if (nb <= p.cand_topk) {
      for (int b = threadIdx.x; b < p.max_c / p.cand_block; b += blockDim.x)
        cand[b] = (b < nb) && bkeys[b] > order_key(-INFINITY);
    } else {
      uint32_t kth;
      int ngt;
      radix_select(bkeys, nb, p.cand_topk, hist, kth, ngt);
      // ties at the threshold: keep lower block ids
      __shared__ int s_eq;
      if (threadIdx.x == 0) {
        s_eq = 0;
        for (int b = 0; b < nb; ++b) {
          const bool keep = bkeys[b] > kth || (bkeys[b] == kth && s_eq < p.cand_topk - ngt && (++s_eq, true));
          cand[b] = keep && bkeys[b] > order_key(-INFINITY);
        }
      }
      __syncthreads();
      for (int b = nb + threadIdx.x; b < p.max_c / p.cand_block; b += blockDim.x) cand[b] = 0;
    }
    __syncthreads();
    if (clen <= k) return;
  }
  uint32_t kth;
  int ngt;
  radix_select(keys, clen, k, hist, kth, ngt);
  const int cnt = ordered_select(keys, clen, kth, k - ngt, p.out_idx + (size_t)t * k);
  for (int j = cnt + threadIdx.x; j < k; j += blockDim.x) p.out_idx[(size_t)t * k + j] = -1;
  if (threadIdx.x == 0) p.out_cnt[t] = cnt;
}

cudaError_t indexer_topk(const IdxParams& p, uint32_t* keys, int keys_ld, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  if (p.head_dim != kIdxDh || p.n_heads > kIdxMaxHeads || keys_ld < p.max_c) return cudaErrorInvalidValue;
  dim3 g(p.T, (p.max_c + kIdxRows - 1) / kIdxRows);
  launch_pdl(idx_score_kernel, g, 128, 0, st, p, keys, keys_ld);
  const size_t smem = 256 * 4 + (size_t)(p.max_c + p.max_c / max(1, p.cand_block) + 1) * 4;
  // dynamic + the kernel's static shared memory must stay under the 227 KB opt-in limit
  if (smem > 220 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    // the limit is raised to the largest size this binding accepts, once per device
    static std::atomic<uint64_t> smem_set{0};
    const cudaError_t e = smem_attr_once(idx_select_kernel, 220 * 1024, smem_set);
    if (e != cudaSuccess) return e;
  }
  launch_pdl(idx_select_kernel, p.T, 256, smem, st, p, keys, keys_ld);
  return cudaGetLastError();
}

}  // namespace dsv4
