// Engram sublayer on the device (V4.1 layers 1 and 14).
//
//   engram_hash    per (token, Engram layer): n-gram row ids from this step's
//                  tokens and a per-slot ring of the last N-1 compressed ids
//                  (the int64 hashing contract of ref/engram.py and
//                  csrc/host/engram.cpp: wrapping products, rolling XOR,
//                  floor-mod by per-(order, head) primes, row offsets)
//   engram_ring    stores each chunk's last N-1 compressed ids into the ring
//   engram_gather  reads the rows straight from the pinned host tables
//                  (zero-copy over PCIe/C2C, 16 bytes per thread) into the
//                  MXFP8 A operand of the wkv GEMM: e4m3 values + ue8m0 scales
//                  in the tensor-core scale-chunk layout; ids outside a table
//                  give zero rows (reference.py:272-319 masks them)
//   engram_gate    after the wkv GEMM: per stream s, dot = <h_s * (q_w*k_w)_s,
//                  key_s> * rsqrt(ms(h_s)) * rsqrt(ms(key_s)) / sqrt(D),
//                  g = sigmoid(signed_sqrt(dot)), h_s += g * value
#include "common.cuh"
#include "kernels.h"

namespace dsv4 {

DSV4_DEV int64_t floor_mod64(int64_t a, int64_t m) {
  const int64_t r = a % m;
  return r < 0 ? r + m : r;
}

__global__ void engram_hash_kernel(EngramParams p) {
  pdl_entry();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.T * p.nl) return;
  const int t = i / p.nl, l = i % p.nl;
  const int N = p.N, H = p.H, cols = (N - 1) * H;
  const int pos = p.pos[t], cs = p.chunk_start[t], row0 = p.step_row0[t], slot = p.slot[t];
  int64_t tok[8];
  bool blocked = false;
  for (int s = 0; s < N; ++s) {
    const int q = pos - s;
    int64_t c = p.pad;
    if (q >= 0 && !blocked) {
      c = q >= cs ? p.token_map[p.ids[row0 + (q - cs)]] : p.ring[(size_t)slot * (N - 1) + q % (N - 1)];
    }
    blocked = blocked || q < 0 || c == -1;
    tok[s] = blocked ? p.pad : c;
  }
  const int64_t* m = p.mult + (size_t)l * N;
  uint64_t roll = (uint64_t)tok[0] * (uint64_t)m[0];
  int64_t* o = p.rows + ((size_t)t * p.nl + l) * cols;
  for (int k = 1; k < N; ++k) {
    roll ^= (uint64_t)tok[k] * (uint64_t)m[k];
    for (int h = 0; h < H; ++h) {
      const int c = (k - 1) * H + h;
      o[c] = floor_mod64((int64_t)roll, p.primes[((size_t)l * (N - 1) + (k - 1)) * H + h]) +
             p.offsets[(size_t)l * cols + c];
    }
  }
}

__global__ void engram_ring_kernel(EngramParams p) {
  pdl_entry();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.T) return;
  const int pos = p.pos[t];
  if (pos > p.last_pos[t] || pos <= p.last_pos[t] - (p.N - 1)) return;
  p.ring[(size_t)p.slot[t] * (p.N - 1) + pos % (p.N - 1)] = p.token_map[p.ids[t]];
}

// one thread per 16 bytes of a gathered row; threads with c < hd/32 also move one scale byte
__global__ void engram_gather_kernel(EngramParams p) {
  pdl_entry();
  const int per_row = p.hd / 16;
  const int cols = (p.N - 1) * p.H;
  const long long total = (long long)p.T * p.nl * cols * per_row;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int c = (int)(i % per_row);
  const long long r = i / per_row;            // (t, l, col)
  const int col = (int)(r % cols);
  const int l = (int)((r / cols) % p.nl);
  const int t = (int)(r / ((long long)cols * p.nl));
  const int64_t id = p.rows[r];
  const bool ok = id >= 0 && id < p.n_emb[l];
  const int K = cols * p.hd;
  uint8_t* aq = p.a_q + (size_t)l * p.a_stride_q + (size_t)t * K + (size_t)col * p.hd;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (ok) v = reinterpret_cast<const uint4*>(p.table[l] + (size_t)id * p.hd)[c];
  reinterpret_cast<uint4*>(aq)[c] = v;
  if (c < p.hd / 32) {
    const uint8_t s = ok ? p.table_sf[l][(size_t)id * (p.hd / 32) + c] : (uint8_t)127;
    p.a_sf[(size_t)l * p.a_stride_sf + sf_chunk_offset(t, col * (p.hd / 32) + c, K / 128)] = s;
  }
}

cudaError_t engram_prepare(const EngramParams& p, int mode, cudaStream_t st) {
  // mode: bit 0 hash, bit 1 ring update, bit 2 gather
  if (p.T == 0) return cudaSuccess;
  if (p.N < 2 || p.N > 8 || p.nl > kEngramMaxLayers || p.hd % 32 || ((p.N - 1) * p.H * p.hd) % 128)
    return cudaErrorInvalidValue;
  if (mode & 1) launch_pdl(engram_hash_kernel, (p.T * p.nl + 127) / 128, 128, 0, st, p);
  if (mode & 2) launch_pdl(engram_ring_kernel, (p.T + 127) / 128, 128, 0, st, p);
  if (mode & 4) {
    const long long total = (long long)p.T * p.nl * (p.N - 1) * p.H * (p.hd / 16);
    launch_pdl(engram_gather_kernel, (unsigned)((total + 255) / 256), 256, 0, st, p);
  }
  return cudaGetLastError();
}

__global__ void __launch_bounds__(128) engram_gate_kernel(__nv_bfloat16* X, const __nv_bfloat16* __restrict__ kv,
                                                          const float* __restrict__ wgt, int D, int hc, float eps) {
  pdl_entry();
  const int t = blockIdx.x;
  const int s = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (s >= hc) return;
  __nv_bfloat16* h = X + ((size_t)t * hc + s) * D;
  const __nv_bfloat16* key = kv + (size_t)t * (hc + 1) * D + (size_t)s * D;
  const __nv_bfloat16* val = kv + (size_t)t * (hc + 1) * D + (size_t)hc * D;
  const float* w = wgt + (size_t)s * D;
  float hh = 0.f, kk = 0.f, hwk = 0.f;
  for (int d = lane * 8; d < D; d += 256) {
    const uint4 hv = *reinterpret_cast<const uint4*>(h + d);
    const uint4 kv4 = *reinterpret_cast<const uint4*>(key + d);
    const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&hv);
    const __nv_bfloat16* kb = reinterpret_cast<const __nv_bfloat16*>(&kv4);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a = __bfloat162float(hb[j]), b = __bfloat162float(kb[j]);
      hh += a * a;
      kk += b * b;
      hwk += a * w[d + j] * b;
    }
  }
  hh = warp_sum(hh);
  kk = warp_sum(kk);
  hwk = warp_sum(hwk);
  const float rstd = rsqrtf(hh / D + eps) * rsqrtf(kk / D + eps);
  const float dot = hwk * rstd * rsqrtf((float)D);
  const float sq = sqrtf(fmaxf(fabsf(dot), 1e-6f));
  const float g = 1.f / (1.f + expf(-copysignf(sq, dot)));
  for (int d = lane * 8; d < D; d += 256) {
    uint4 hv = *reinterpret_cast<const uint4*>(h + d);
    const uint4 vv = *reinterpret_cast<const uint4*>(val + d);
    __nv_bfloat16* hb = reinterpret_cast<__nv_bfloat16*>(&hv);
    const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(&vv);
#pragma unroll
    for (int j = 0; j < 8; ++j) hb[j] = __float2bfloat16(__bfloat162float(hb[j]) + g * __bfloat162float(vb[j]));
    *reinterpret_cast<uint4*>(h + d) = hv;
  }
}

cudaError_t engram_gate(__nv_bfloat16* X, const __nv_bfloat16* kv, const float* wgt, int T, int D, int hc, float eps,
                        cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (D % 256 || hc > 4) return cudaErrorInvalidValue;
  launch_pdl(engram_gate_kernel, T, 128, 0, st, X, kv, wgt, D, hc, eps);
  return cudaGetLastError();
}

}  // namespace dsv4
