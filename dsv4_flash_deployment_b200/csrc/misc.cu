// Small fused kernels: embedding lookup into the residual streams, row argmax.
#include "common.cuh"
#include "kernels.h"

namespace dsv4 {

// X[t, i, :] = table[ids[t], :] for every stream i (reference.py:909-911).
__global__ void embed_streams_kernel(const __nv_bfloat16* __restrict__ table, const int* __restrict__ ids, int D,
                                     int hc, __nv_bfloat16* X) {
  const int t = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)ids[t] * D);
  for (int i = threadIdx.x; i < D / 8; i += blockDim.x) {
    const uint4 v = src[i];
    for (int s = 0; s < hc; ++s) reinterpret_cast<uint4*>(X + ((size_t)t * hc + s) * D)[i] = v;
  }
}

cudaError_t embed_streams(const __nv_bfloat16* table, const int* ids, int T, int D, int hc, __nv_bfloat16* X,
                          cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  embed_streams_kernel<<<T, 256, 0, st>>>(table, ids, D, hc, X);
  return cudaGetLastError();
}

// out[t] = argmax_v logits[t, v] (first index on ties).
__global__ void __launch_bounds__(512) argmax_kernel(const float* __restrict__ logits, int V, int ld, int* out) {
  const int t = blockIdx.x;
  const float* row = logits + (size_t)t * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float x = row[v];
    if (x > bv) {
      bv = x;
      bi = v;
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
  __shared__ float sv[16];
  __shared__ int si[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
        bv = sv[w];
        bi = si[w];
      }
    out[t] = bi;
  }
}

cudaError_t argmax_rows(const float* logits, int T, int V, int ld, int* out, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  argmax_kernel<<<T, 512, 0, st>>>(logits, V, ld, out);
  return cudaGetLastError();
}

}  // namespace dsv4

namespace dsv4 {

// One DSpark Markov-head step per sequence j (reference.py:1216-1247):
//   i >= 0: tok = argmax_v(logits[(j*blk + i), v] + mlog[j, v]), toks[i+1][j] = tok
//   i <  0: tok = toks[0][j] (the root)      (toks rows are ts apart)
// then emb[j, :] = memb[tok, :] (the next step's rank-R input).
__global__ void __launch_bounds__(512) markov_step_kernel(const float* __restrict__ logits, int ld, int blk, int i,
                                                          const float* __restrict__ mlog, int mld, int V, int n,
                                                          int* toks, int ts, const __nv_bfloat16* __restrict__ memb,
                                                          int R, __nv_bfloat16* emb) {
  const int j = blockIdx.x;
  __shared__ int s_tok;
  if (i >= 0) {
    const float* row = logits + (size_t)(j * blk + i) * ld;
    const float* add = mlog + (size_t)j * mld;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      const float x = row[v] + add[v];
      if (x > bv) {
        bv = x;
        bi = v;
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
    __shared__ float sv[16];
    __shared__ int si[16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
      sv[warp] = bv;
      si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
          bv = sv[w];
          bi = si[w];
        }
      toks[(size_t)(i + 1) * ts + j] = bi;
      s_tok = bi;
    }
  } else if (threadIdx.x == 0) {
    s_tok = toks[j];
  }
  __syncthreads();
  const int tok = s_tok;
  for (int r = threadIdx.x; r < R; r += blockDim.x) emb[(size_t)j * R + r] = memb[(size_t)tok * R + r];
}

cudaError_t markov_step(const float* logits, int ld, int blk, int i, const float* mlog, int mld, int V, int n,
                        int* toks, int ts, const __nv_bfloat16* memb, int R, __nv_bfloat16* emb, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  markov_step_kernel<<<n, 512, 0, st>>>(logits, ld, blk, i, mlog, mld, V, n, toks, ts, memb, R, emb);
  return cudaGetLastError();
}

}  // namespace dsv4
