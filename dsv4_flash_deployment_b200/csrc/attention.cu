// Sparse multi-query attention over gathered latent rows (decode + prefill).
//
// Per query token t at position p (reference.py:172-235, _attention_step
// :704-838): q [H, Dh] gets (optional per-head RMSNorm, V4-Flash) + RoPE on the
// last 64 dims; the attended row set is the sliding window (positions
// max(0, p-W+1)..p) plus the selected compressed rows (indexer top-k list, or
// every compressed entry for dense layers).  K and V are the same latent row.
// Scores in fp32, online softmax over blocks of 64 rows with P rounded to bf16
// before PV, and exp(sink - max) added to the denominator.  The output gets the
// inverse RoPE on the last 64 dims and is written bf16.
//
// Window rows of positions at or after the token's chunk start come from this
// step's kv buffer (prefill chunks), earlier ones from the per-sequence ring.
//
// The caches hold quantized row records (kernels.h): window rows (the ring and
// this step's rows) as KV8 (e4m3 + ue8m0 per 32, 528 bytes), compressed rows as
// KV4 (packed e2m1 + e4m3 per 16, 288 bytes).  Both decode exactly to the bf16
// values of the reference's round trips.
//
// One CTA (8 warps) per (token, split).  A block's raw records are gathered with
// cp.async into double-buffered shared memory, then decoded into one bf16 tile;
// QK^T and PV use mma.sync m16n8k16 bf16 with fp32 accumulators (PV accumulators
// stay in registers, 64 dims per warp).
// With splits > 1 the partial (acc, max, sum) go to a workspace and
// attn_combine merges them (C = 1 decode spreads a token over many SMs).
#include <cuda_fp4.h>

#include "common.cuh"
#include "kernels.h"
#include "mma_sync.cuh"

namespace dsv4 {

namespace {
constexpr int kH = 64;
constexpr int kDh = 512;
constexpr int kBlk = 64;
constexpr int kPadE = 8;                 // row padding (bf16 elements) to spread banks
constexpr int kRowE = kDh + kPadE;       // 520
constexpr int kPPad = kBlk + 8;          // P row stride (bf16)

constexpr int kRec8 = kv8_bytes(kDh);   // 528
constexpr int kRec4 = kv4_bytes(kDh);   // 288
constexpr int kRecChunks = kRec8 / 16;  // 16-byte pieces of the widest record

constexpr size_t kSmemQ = (size_t)kH * kRowE * 2;
constexpr size_t kSmemKV = (size_t)kBlk * kRowE * 2;     // one decoded block
constexpr size_t kSmemRaw = (size_t)kBlk * kRec8;        // one block of raw records (x2)
constexpr size_t kSmemP = (size_t)kH * kPPad * 2;
constexpr size_t kSmemRows = (size_t)kAttnMaxRows * 8;
constexpr size_t kSmemStats = (size_t)kH * 4 * 7;  // max, sum, corr, 2x partial max, 2x partial sum
constexpr size_t kSmemTotal = kSmemQ + kSmemKV + 2 * kSmemRaw + kSmemP + kSmemRows + kSmemStats;
static_assert(kRec8 % 16 == 0 && kRec4 % 16 == 0, "records must be whole 16-byte pieces");
static_assert(kSmemTotal <= 227 * 1024, "attention shared memory exceeds the per-CTA limit");

// Eight columns [8c, 8c + 8) of a KV8 record -> bf16: two e4m3 codes per
// hardware conversion to f16 (exact), then the power-of-two scale in fp32.
DSV4_DEV uint4 decode8_kv8(const uint8_t* rec, int c) {
  const uint2 codes = *reinterpret_cast<const uint2*>(rec + 8 * c);
  const uint32_t e = rec[kDh + (c >> 2)];
  const float sc = e ? __uint_as_float(e << 23) : 0.f;
  uint4 o;
  uint32_t* o32 = reinterpret_cast<uint32_t*>(&o);
  const uint32_t w[2] = {codes.x, codes.y};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i >> 1] >> (16 * (i & 1))), __NV_E4M3);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    o32[i] = pack_bf16(f.x * sc, f.y * sc);
  }
  return o;
}

// Eight columns [8c, 8c + 8) of a KV4 record -> bf16: two e2m1 codes per
// hardware conversion to f16, times the e4m3 scale in f16 (e2m1 x e4m3 lies in
// [2^-10, 2688] with at most 6 significant bits: exact in f16 and in bf16).
DSV4_DEV uint4 decode8_kv4(const uint8_t* rec, int c) {
  const uint32_t codes = *reinterpret_cast<const uint32_t*>(rec + 4 * c);
  const __half_raw sr = __nv_cvt_fp8_to_halfraw(rec[kDh / 2 + (c >> 1)], __NV_E4M3);
  const __half2 s2 = __half2half2(*reinterpret_cast<const __half*>(&sr));
  uint4 o;
  uint32_t* o32 = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2_raw hr = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)((codes >> (8 * i)) & 0xFF), __NV_E2M1);
    const float2 f = __half22float2(__hmul2(*reinterpret_cast<const __half2*>(&hr), s2));
    o32[i] = pack_bf16(f.x, f.y);
  }
  return o;
}
}  // namespace

__global__ void __launch_bounds__(256, 1) attn_kernel(AttnParams p) {
  pdl_entry();
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sKV = reinterpret_cast<__nv_bfloat16*>(smem + kSmemQ);
  uint8_t* sRaw = smem + kSmemQ + kSmemKV;
  __nv_bfloat16* sP = reinterpret_cast<__nv_bfloat16*>(smem + kSmemQ + kSmemKV + 2 * kSmemRaw);
  const uint8_t** sRows = reinterpret_cast<const uint8_t**>(smem + kSmemQ + kSmemKV + 2 * kSmemRaw + kSmemP);
  float* sMax = reinterpret_cast<float*>(smem + kSmemQ + kSmemKV + 2 * kSmemRaw + kSmemP + kSmemRows);
  float* sSum = sMax + kH;
  float* sCorr = sSum + kH;
  float* sPMax = sCorr + kH;   // [kH][2]
  float* sPSum = sPMax + 2 * kH;

  const int t = blockIdx.x;
  const int split = blockIdx.y;
  const int nsplit = gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos = p.pos[t];
  const int slot = p.slot[t];
  const int rope_pos = p.rope_pos ? p.rope_pos[t] : pos;

  // ---------------- row list: window (KV8), then compressed entries (KV4, valid ones first)
  const int we = p.win_end ? p.win_end[t] : pos;
  const int n_win = min(we + 1, p.win_len > 0 ? p.win_len : p.W);
  const int n_comp = p.comp != nullptr ? min(p.comp_cnt[t], kAttnMaxRows - n_win) : 0;
  {
    const int cs = p.chunk_start[t];
    for (int j = tid; j < n_win + n_comp; j += blockDim.x) {
      const uint8_t* r;
      if (j < n_win) {
        const int pp = we - n_win + 1 + j;
        if (pp >= cs)
          r = p.kv_step + (size_t)(p.step_row0[t] + (pp - cs)) * kRec8;
        else
          r = p.ring + ((size_t)slot * p.W + (pp % p.W)) * kRec8;
      } else {
        const int jj = j - n_win;
        const int ci = p.comp_idx != nullptr ? p.comp_idx[(size_t)t * p.comp_k + jj] : jj;
        r = p.comp + kv_row(p.comp_pages, slot, ci, p.max_c) * kRec4;
      }
      sRows[j] = r;
    }
  }
  // ---------------- Q: optional head norm, RoPE, into smem
  for (int h = warp; h < kH; h += 8) {
    if (h >= p.n_heads) {   // padding rows of the head tile
      *reinterpret_cast<uint4*>(sQ + (size_t)h * kRowE + lane * 16) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sQ + (size_t)h * kRowE + lane * 16 + 8) = make_uint4(0, 0, 0, 0);
      continue;
    }
    const __nv_bfloat16* qg = p.q + (size_t)t * p.q_stride + (size_t)h * kDh;
    float v[16];
    {
      uint4 raw[2];
      raw[0] = *reinterpret_cast<const uint4*>(qg + lane * 16);
      raw[1] = *reinterpret_cast<const uint4*>(qg + lane * 16 + 8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
    if (p.q_head_norm) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) ss += v[i] * v[i];
      ss = warp_sum(ss);
      const float r = rsqrtf(ss / (float)kDh + p.norm_eps);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = __bfloat162float(__float2bfloat16(v[i] * r));
    }
    if (lane * 16 >= kDh - 64) {  // rope dims 448..511, pairs (2i, 2i+1)
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const int pi = (lane * 16 + i - (kDh - 64)) >> 1;
        const float c = p.rope_cos[(size_t)rope_pos * 32 + pi], s = p.rope_sin[(size_t)rope_pos * 32 + pi];
        const float e = v[i], o = v[i + 1];
        v[i] = e * c - o * s;
        v[i + 1] = e * s + o * c;
      }
    }
    __nv_bfloat16* qs = sQ + (size_t)h * kRowE + lane * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) qs[i] = __float2bfloat16(v[i]);
  }
  if (tid < kH) {
    sMax[tid] = -1e30f;
    sSum[tid] = 0.f;
  }
  __syncthreads();
  const int n_rows = n_win + n_comp;
  const int n_blocks = (n_rows + kBlk - 1) / kBlk;
  const int bps = (n_blocks + nsplit - 1) / nsplit;
  const int b_begin = split * bps;
  const int b_end = min(n_blocks, b_begin + bps);

  // raw records of block b -> sRaw[buf] (rows past the end are zero-filled, which
  // decodes to zeros; the unused tail of a KV4 row is not copied)
  auto load_block = [&](int b, int buf) {
    uint8_t* dst = sRaw + (size_t)buf * kSmemRaw;
    for (int c = tid; c < kBlk * kRecChunks; c += 256) {
      const int r = c / kRecChunks, ch = c % kRecChunks;
      const int gr = b * kBlk + r;
      const bool ok = gr < n_rows;
      if (ok && gr >= n_win && ch * 16 >= kRec4) continue;
      const uint8_t* src = ok ? sRows[gr] + ch * 16 : reinterpret_cast<const uint8_t*>(p.q);
      cp_async16(dst + (size_t)r * kRec8 + ch * 16, src, ok);
    }
    cp_async_commit();
  };
  // sRaw[buf] -> the bf16 tile: thread -> 8-column chunk (tid % 64) of rows tid / 64 + 4i
  auto decode_block = [&](int b, int buf) {
    const uint8_t* raw = sRaw + (size_t)buf * kSmemRaw;
    const int c = tid & 63;
#pragma unroll 4
    for (int r = tid >> 6; r < kBlk; r += 4) {
      const int gr = b * kBlk + r;
      const uint8_t* rec = raw + (size_t)r * kRec8;
      const uint4 v = (gr >= n_win && gr < n_rows) ? decode8_kv4(rec, c) : decode8_kv8(rec, c);
      *reinterpret_cast<uint4*>(sKV + (size_t)r * kRowE + 8 * c) = v;
    }
  };

  float acc[4][8][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[i][j][k] = 0.f;

  const int g = lane >> 2, cq = lane & 3;
  if (b_begin < b_end) load_block(b_begin, 0);
  for (int b = b_begin; b < b_end; ++b) {
    const int buf = (b - b_begin) & 1;
    if (b + 1 < b_end) {
      load_block(b + 1, buf ^ 1);
      cp_async_wait1();
    } else {
      cp_async_wait0();
    }
    __syncthreads();
    decode_block(b, buf);
    __syncthreads();
    const __nv_bfloat16* kv = sKV;
    // ---- S = Q K^T : warp -> heads (warp%4)*16, rows (warp/4)*32
    {
      const int h0 = (warp & 3) * 16, n0 = (warp >> 2) * 32;
      float s[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) s[i][k] = 0.f;
      const uint32_t qa = smem_u32(sQ + (size_t)(h0 + (lane & 7) + 8 * ((lane >> 3) & 1)) * kRowE + 8 * (lane >> 4));
#pragma unroll 4
      for (int k0 = 0; k0 < kDh; k0 += 16) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(qa + k0 * 2, a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < 4; nt += 2) {
          uint32_t b0, b1, b2, b3;
          const uint32_t ba =
              smem_u32(kv + (size_t)(n0 + nt * 8 + (lane & 7) + 8 * (lane >> 4)) * kRowE + k0 + 8 * ((lane >> 3) & 1));
          ldsm_x4(ba, b0, b1, b2, b3);
          mma16816(s[nt], a0, a1, a2, a3, b0, b1);
          mma16816(s[nt + 1], a0, a1, a2, a3, b2, b3);
        }
      }
      // ---- online softmax from registers (each head's 64 columns span 2 warps)
      const int valid = min(kBlk, n_rows - b * kBlk);
      float pm[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int col = n0 + nt * 8 + 2 * cq;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int cc = col + (e & 1);
          s[nt][e] = cc < valid ? s[nt][e] * p.scale : -INFINITY;
          pm[e >> 1] = fmaxf(pm[e >> 1], s[nt][e]);
        }
      }
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        pm[hf] = fmaxf(pm[hf], __shfl_xor_sync(0xffffffffu, pm[hf], 1));
        pm[hf] = fmaxf(pm[hf], __shfl_xor_sync(0xffffffffu, pm[hf], 2));
      }
      if (cq == 0) {
        sPMax[(h0 + g) * 2 + (warp >> 2)] = pm[0];
        sPMax[(h0 + g + 8) * 2 + (warp >> 2)] = pm[1];
      }
      __syncthreads();
      float nm[2], ps[2] = {0.f, 0.f};
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int h = h0 + g + 8 * hf;
        nm[hf] = fmaxf(sMax[h], fmaxf(sPMax[h * 2], sPMax[h * 2 + 1]));
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int col = n0 + nt * 8 + 2 * cq;
        const float p0 = expf(s[nt][0] - nm[0]), p1 = expf(s[nt][1] - nm[0]);
        const float p2 = expf(s[nt][2] - nm[1]), p3 = expf(s[nt][3] - nm[1]);
        ps[0] += p0 + p1;
        ps[1] += p2 + p3;
        *reinterpret_cast<uint32_t*>(sP + (h0 + g) * kPPad + col) = pack_bf16(p0, p1);
        *reinterpret_cast<uint32_t*>(sP + (h0 + g + 8) * kPPad + col) = pack_bf16(p2, p3);
      }
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        ps[hf] += __shfl_xor_sync(0xffffffffu, ps[hf], 1);
        ps[hf] += __shfl_xor_sync(0xffffffffu, ps[hf], 2);
      }
      if (cq == 0) {
        sPSum[(h0 + g) * 2 + (warp >> 2)] = ps[0];
        sPSum[(h0 + g + 8) * 2 + (warp >> 2)] = ps[1];
      }
    }
    __syncthreads();
    if (tid < kH) {
      const float om = sMax[tid];
      const float nmx = fmaxf(om, fmaxf(sPMax[tid * 2], sPMax[tid * 2 + 1]));
      const float corr = expf(om - nmx);
      sCorr[tid] = corr;
      sSum[tid] = sSum[tid] * corr + sPSum[tid * 2] + sPSum[tid * 2 + 1];
      sMax[tid] = nmx;
    }
    __syncthreads();
    // ---- O += P V : warp -> dims 64*warp.., all heads
    {
      const int d0 = warp * 64;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const float c0 = sCorr[mt * 16 + g], c1 = sCorr[mt * 16 + g + 8];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          acc[mt][nt][0] *= c0;
          acc[mt][nt][1] *= c0;
          acc[mt][nt][2] *= c1;
          acc[mt][nt][3] *= c1;
        }
      }
#pragma unroll
      for (int k0 = 0; k0 < kBlk; k0 += 16) {
        uint32_t bfr[8][2];
#pragma unroll
        for (int nt = 0; nt < 8; nt += 2) {
          const uint32_t va =
              smem_u32(kv + (size_t)(k0 + (lane & 7) + 8 * ((lane >> 3) & 1)) * kRowE + d0 + nt * 8 + 8 * (lane >> 4));
          ldsm_x4_t(va, bfr[nt][0], bfr[nt][1], bfr[nt + 1][0], bfr[nt + 1][1]);
        }
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          uint32_t a0, a1, a2, a3;
          const uint32_t pa =
              smem_u32(sP + (size_t)(mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * kPPad + k0 + 8 * (lane >> 4));
          ldsm_x4(pa, a0, a1, a2, a3);
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) mma16816(acc[mt][nt], a0, a1, a2, a3, bfr[nt][0], bfr[nt][1]);
        }
      }
    }
    __syncthreads();
  }

  // ---------------- epilogue
  const int d0 = warp * 64;
  if (nsplit == 1) {
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int h = mt * 16 + g + 8 * half;
        if (h >= p.n_heads) continue;
        const float den = sSum[h] + expf(p.sink[h] - sMax[h]);
        const float inv = 1.f / den;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int d = d0 + nt * 8 + 2 * cq;
          float e = acc[mt][nt][2 * half] * inv, o = acc[mt][nt][2 * half + 1] * inv;
          // output rounds to bf16 before the inverse rotation, as the reference does
          e = __bfloat162float(__float2bfloat16(e));
          o = __bfloat162float(__float2bfloat16(o));
          if (d >= kDh - 64) {
            const int pi = (d - (kDh - 64)) >> 1;
            const float c = p.rope_cos[(size_t)rope_pos * 32 + pi], s = -p.rope_sin[(size_t)rope_pos * 32 + pi];
            const float ne = e * c - o * s, no = e * s + o * c;
            e = ne;
            o = no;
          }
          *reinterpret_cast<uint32_t*>(p.out + (size_t)t * p.out_stride + (size_t)h * kDh + d) = pack_bf16(e, o);
        }
      }
    }
  } else {
    float* ws = p.workspace + ((size_t)t * nsplit + split) * kH * (kDh + 2);
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int h = mt * 16 + g + 8 * half;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int d = d0 + nt * 8 + 2 * cq;
          ws[(size_t)h * (kDh + 2) + d] = acc[mt][nt][2 * half];
          ws[(size_t)h * (kDh + 2) + d + 1] = acc[mt][nt][2 * half + 1];
        }
      }
    }
    if (tid < kH) {
      ws[(size_t)tid * (kDh + 2) + kDh] = sMax[tid];
      ws[(size_t)tid * (kDh + 2) + kDh + 1] = sSum[tid];
    }
  }
}

// Merge split partials: one CTA per (token, head), thread -> dim pair.  The
// per-split rescale factors exp(m_s - m) and the denominator are formed once
// in shared memory; each thread then issues nsplit independent float2 loads.
constexpr int kMaxSplits = 32;
__global__ void __launch_bounds__(256) attn_combine_kernel(AttnParams p, int nsplit) {
  pdl_entry();
  const int t = blockIdx.x, h = blockIdx.y;
  __shared__ float sF[kMaxSplits];
  __shared__ float sInv;
  const float* base = p.workspace + (size_t)t * nsplit * kH * (kDh + 2) + (size_t)h * (kDh + 2);
  const size_t sstride = (size_t)kH * (kDh + 2);
  if (threadIdx.x < 32) {
    const int s = threadIdx.x;
    const float ms = s < nsplit ? base[s * sstride + kDh] : -1e30f;
    float m = ms;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float f = s < nsplit ? expf(ms - m) : 0.f;
    float den = s < nsplit ? base[s * sstride + kDh + 1] * f : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    if (s < nsplit) sF[s] = f;
    if (s == 0) sInv = 1.f / (den + expf(p.sink[h] - m));
  }
  __syncthreads();
  const int rope_pos = p.rope_pos ? p.rope_pos[t] : p.pos[t];
  const float inv = sInv;
  for (int d = 2 * threadIdx.x; d < kDh; d += 2 * blockDim.x) {
    float num0 = 0.f, num1 = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float2 w = *reinterpret_cast<const float2*>(base + s * sstride + d);
      num0 += w.x * sF[s];
      num1 += w.y * sF[s];
    }
    float e0 = __bfloat162float(__float2bfloat16(num0 * inv));
    float o0 = __bfloat162float(__float2bfloat16(num1 * inv));
    if (d >= kDh - 64) {
      const int pi = (d - (kDh - 64)) >> 1;
      const float c = p.rope_cos[(size_t)rope_pos * 32 + pi], sn = -p.rope_sin[(size_t)rope_pos * 32 + pi];
      const float ne = e0 * c - o0 * sn, no = e0 * sn + o0 * c;
      e0 = ne;
      o0 = no;
    }
    *reinterpret_cast<uint32_t*>(p.out + (size_t)t * p.out_stride + (size_t)h * kDh + d) = pack_bf16(e0, o0);
  }
}

size_t attn_smem_bytes() { return kSmemTotal; }

cudaError_t attention(const AttnParams& p, int nsplit, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  if (p.n_heads < 1 || p.n_heads > kH) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> smem_set{0};
  {
    const cudaError_t e = smem_attr_once(attn_kernel, (int)kSmemTotal, smem_set);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(p.T, nsplit);
  launch_pdl(attn_kernel, grid, 256, kSmemTotal, st, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || nsplit == 1) return e;
  if (nsplit > kMaxSplits) return cudaErrorInvalidValue;
  launch_pdl(attn_combine_kernel, dim3(p.T, p.n_heads), 256, 0, st, p, nsplit);
  return cudaGetLastError();
}

}  // namespace dsv4
