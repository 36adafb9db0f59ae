// KV compressor: softmax-gated pooling of r (or 2r, overlapped) token
// projections into one compressed latent row, then RMSNorm, RoPE at the group
// start, e2m1 codes with e4m3 scales per 16 stored as a KV4 record (kernels.h)
// into the sequence's compressed cache; optionally the indexer key of the same
// entry (latent @ wk -> RMSNorm -> RoPE -> e2m1 with ue8m0 scales per 32, an
// IK4 record).  Reference:
// _compressor_step (reference.py:547-603), _indexer_step k path (:621-640),
// latent store (:792-807).
//
// One CTA per compressed entry closed in this step.  Source positions come from
// this step's projection rows when they belong to the step, otherwise from the
// per-sequence ring of the most recent (overlap * r) projections.
#include "common.cuh"
#include "kernels.h"

namespace dsv4 {

template <int NT>
DSV4_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = threadIdx.x < NT / 32 ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) red[NT / 32] = s;
  }
  __syncthreads();
  return red[NT / 32];
}

// 512 threads.  Pooling: 128 dim-quads (float4 loads) x 4 slot lanes, each lane an
// independent online softmax over every 4th slot, merged through shared
// memory.  Then thread d owns latent dim d (dh == 512).
__global__ void __launch_bounds__(512) compress_pool_kernel(CompParams p) {
  pdl_entry();
  __shared__ float red[32];
  __shared__ __nv_bfloat16 lat[512];
  __shared__ float kbuf[256];
  __shared__ float4 sm_m[4][128], sm_s[4][128], sm_a[4][128];
  const int gi = blockIdx.x;
  if (gi >= *p.n_groups_dev) return;
  const int slot = p.g_slot[gi], g = p.g_index[gi], cs = p.g_chunk_start[gi], row0 = p.g_row0[gi];
  const int d = threadIdx.x;
  const int r = p.r, co = p.co, dh = p.dh;
  const int width = 2 * co * dh;
  const int depth = co * r;
  {
    const int q4 = (threadIdx.x & 127) * 4, lane4 = threadIdx.x >> 7;
    float m[4], ss[4], ac[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) m[k] = -INFINITY, ss[k] = 0.f, ac[k] = 0.f;
    const int first = g * r - (co - 1) * r;
#pragma unroll 4
    for (int pp = first + lane4; pp < (g + 1) * r; pp += 4) {
      if (pp < 0) continue;
      const int half = (pp < g * r) ? 0 : (co - 1);
      const float* src = (pp >= cs) ? p.proj + (size_t)(row0 + pp - cs) * width
                                    : p.ring + ((size_t)slot * depth + (pp % depth)) * width;
      const float4 kv = *reinterpret_cast<const float4*>(src + half * dh + q4);
      float4 sc = *reinterpret_cast<const float4*>(src + co * dh + half * dh + q4);
      if (p.ape) {
        const float4 a = *reinterpret_cast<const float4*>(p.ape + (size_t)(pp % r) * co * dh + half * dh + q4);
        sc.x += a.x, sc.y += a.y, sc.z += a.z, sc.w += a.w;
      }
      const float scv[4] = {sc.x, sc.y, sc.z, sc.w}, kvv[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float nm = fmaxf(m[k], scv[k]);
        const float corr = expf(m[k] - nm);
        const float e = expf(scv[k] - nm);
        ss[k] = ss[k] * corr + e;
        ac[k] = ac[k] * corr + e * kvv[k];
        m[k] = nm;
      }
    }
    sm_m[lane4][threadIdx.x & 127] = make_float4(m[0], m[1], m[2], m[3]);
    sm_s[lane4][threadIdx.x & 127] = make_float4(ss[0], ss[1], ss[2], ss[3]);
    sm_a[lane4][threadIdx.x & 127] = make_float4(ac[0], ac[1], ac[2], ac[3]);
  }
  __syncthreads();
  float acc = 0.f, ssum = 0.f;
  {
    const int q = d >> 2, k = d & 3;
    float mj[4], M = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mj[j] = reinterpret_cast<const float*>(&sm_m[j][q])[k];
      M = fmaxf(M, mj[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (mj[j] == -INFINITY) continue;   // lane saw no slot
      const float w = expf(mj[j] - M);
      ssum += reinterpret_cast<const float*>(&sm_s[j][q])[k] * w;
      acc += reinterpret_cast<const float*>(&sm_a[j][q])[k] * w;
    }
  }
  const float pooled = __bfloat162float(__float2bfloat16(acc / ssum));
  const float ss = block_sum<512>(pooled * pooled, red);
  const float rr = rsqrtf(ss / (float)dh + p.eps);
  const float y = __bfloat162float(__float2bfloat16(pooled * rr * __bfloat162float(p.norm_w[d])));
  lat[d] = __float2bfloat16(y);
  // RoPE at the group start position, pairs (2i, 2i+1) in the last 64 dims
  const int gp = g * r;
  __syncthreads();
  float z = y;
  if (d >= dh - 64) {
    const int pi = (d - (dh - 64)) >> 1;
    const float c = p.rope_cos[(size_t)gp * 32 + pi], s = p.rope_sin[(size_t)gp * 32 + pi];
    const float e = __bfloat162float(lat[d & ~1]), o = __bfloat162float(lat[d | 1]);
    z = (d & 1) ? (e * s + o * c) : (e * c - o * s);
    z = __bfloat162float(__float2bfloat16(z));
  }
  // e2m1 with an e4m3 scale per 16 (16 consecutive dims = half a warp), stored as
  // a KV4 record: packed codes (even dim in the low nibble), then the scale bytes
  {
    float amax = fabsf(z);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = fmaxf(amax, 6.f * 0.001953125f);
    const uint8_t sb = f32_to_e4m3(amax / 6.f);
    const uint32_t code = e2m1_code(z, e4m3_to_f32(sb));
    const uint32_t hi = __shfl_down_sync(0xffffffffu, code, 1);
    uint8_t* rec = p.comp_out + kv_row(p.pages, slot, g, p.max_c) * kv4_bytes(dh);
    if ((d & 1) == 0) rec[d >> 1] = (uint8_t)(code | (hi << 4));
    if ((d & 15) == 0) rec[dh / 2 + (d >> 4)] = sb;
  }
  if (p.wk == nullptr) return;
  // ---- indexer key: k = bf16(latent @ wk^T) -> RMSNorm -> RoPE -> e2m1 (ue8m0 / 32)
  const int kd = p.idx_dim;
  {
    // warp-cooperative GEMV: warp w computes outputs w, w+16, ...; lanes split the 512 inputs
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float lv[16];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 raw = *reinterpret_cast<const uint4*>(lat + c * 256 + lane * 8);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) lv[c * 8 + e] = __bfloat162float(b[e]);
    }
    for (int o = warp; o < kd; o += 16) {
      const __nv_bfloat16* wr = p.wk + (size_t)o * dh;
      float a = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint4 raw = *reinterpret_cast<const uint4*>(wr + c * 256 + lane * 8);
        const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int e = 0; e < 8; ++e) a += lv[c * 8 + e] * __bfloat162float(b[e]);
      }
      a = warp_sum(a);
      if (lane == 0) kbuf[o] = __bfloat162float(__float2bfloat16(a));
    }
  }
  __syncthreads();
  const float kv = d < kd ? kbuf[d] : 0.f;
  const float kss = block_sum<512>(kv * kv, red);
  if (d >= kd) return;  // whole warps exit (kd is a multiple of 32)
  const float kr = rsqrtf(kss / (float)kd + p.eps);
  float kn = __bfloat162float(__float2bfloat16(kv * kr * __bfloat162float(p.k_norm_w[d])));
  {
    const float other = __shfl_xor_sync(0xffffffffu, kn, 1);
    if (d >= kd - 64) {
      const int pi = (d - (kd - 64)) >> 1;
      const float c = p.rope_cos[(size_t)gp * 32 + pi], s = p.rope_sin[(size_t)gp * 32 + pi];
      kn = (d & 1) ? (other * s + kn * c) : (kn * c - other * s);
      kn = __bfloat162float(__float2bfloat16(kn));
    }
  }
  // IK4 record: packed e2m1 codes, then the ue8m0 exponent of each 32 dims (one warp)
  const float amax = fmaxf(warp_max(fabsf(kn)), 6.f * 1.1754943508222875e-38f);
  const uint32_t e = pow2_ceil_exp(amax, 1.f / 6.f);
  const uint32_t code = e2m1_code(kn, exp_to_f32(e));
  const uint32_t hi = __shfl_down_sync(0xffffffffu, code, 1);
  uint8_t* rec = p.idx_out + kv_row(p.pages, slot, g, p.max_c) * ik4_bytes(kd);
  if ((d & 1) == 0) rec[d >> 1] = (uint8_t)(code | (hi << 4));
  if ((d & 31) == 0) rec[kd / 2 + (d >> 5)] = (uint8_t)e;
}

cudaError_t compress_pool(const CompParams& p, cudaStream_t st) {
  if (p.n_groups == 0) return cudaSuccess;
  if (p.dh != 512 || (p.wk && (p.idx_dim % 32 || p.idx_dim > 256))) return cudaErrorInvalidValue;
  launch_pdl(compress_pool_kernel, p.n_groups, 512, 0, st, p);
  return cudaGetLastError();
}

template <typename T>
__global__ void ring_update_kernel(T* ring, int depth, int width, const T* src, int T_, const int* slot,
                                   const int* pos, const int* last_pos) {
  pdl_entry();
  const int t = blockIdx.x;
  if (t >= T_) return;
  const int ps = pos[t];
  // rows past last_pos are not committed (rejected draft tokens of a verify step);
  // rows more than depth before it are overwritten later in the same step
  if (ps > last_pos[t] || ps <= last_pos[t] - depth) return;
  T* dst = ring + ((size_t)slot[t] * depth + (ps % depth)) * width;
  const T* s = src + (size_t)t * width;
  for (int i = threadIdx.x; i < width; i += blockDim.x) dst[i] = s[i];
}

cudaError_t ring_update_f32(float* ring, int depth, int width, const float* src, int T, const int* slot,
                            const int* pos, const int* last_pos, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  launch_pdl(ring_update_kernel<float>, T, 256, 0, st, ring, depth, width, src, T, slot, pos, last_pos);
  return cudaGetLastError();
}

cudaError_t ring_update_bf16(__nv_bfloat16* ring, int depth, int width, const __nv_bfloat16* src, int T,
                             const int* slot, const int* pos, const int* last_pos, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  launch_pdl(ring_update_kernel<__nv_bfloat16>, T, 256, 0, st, ring, depth, width, src, T, slot, pos, last_pos);
  return cudaGetLastError();
}

// Byte rows (KV8 records): 16-byte vectors, width a multiple of 16.
__global__ void ring_update_rec_kernel(uint8_t* ring, int depth, int width, const uint8_t* src, int T_,
                                       const int* slot, const int* pos, const int* last_pos) {
  pdl_entry();
  const int t = blockIdx.x;
  if (t >= T_) return;
  const int ps = pos[t];
  if (ps > last_pos[t] || ps <= last_pos[t] - depth) return;
  uint4* dst = reinterpret_cast<uint4*>(ring + ((size_t)slot[t] * depth + (ps % depth)) * width);
  const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)t * width);
  for (int i = threadIdx.x; i < width / 16; i += blockDim.x) dst[i] = s[i];
}

cudaError_t ring_update_rec(uint8_t* ring, int depth, int width, const uint8_t* src, int T, const int* slot,
                            const int* pos, const int* last_pos, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (width % 16) return cudaErrorInvalidValue;
  launch_pdl(ring_update_rec_kernel, T, 64, 0, st, ring, depth, width, src, T, slot, pos, last_pos);
  return cudaGetLastError();
}

}  // namespace dsv4
