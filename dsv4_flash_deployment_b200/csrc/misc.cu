// Small fused kernels: embedding lookup into the residual streams, row argmax.
#include "common.cuh"
#include "kernels.h"
#include "peer.cuh"

#include <algorithm>
#include <cstdlib>

namespace dsv4 {

std::vector<DbgSetter>& dbg_registry() {
  static std::vector<DbgSetter> reg;
  return reg;
}

int dbg_bounds_attach(uint32_t* err) {
  int n = 0;
  for (DbgSetter f : dbg_registry()) {
    const cudaError_t e = f(err);
    if (e != cudaSuccess) return -(int)e;
    ++n;
  }
  return n;
}

int dbg_bounds_units() { return (int)dbg_registry().size(); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("DSV4_PDL");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

// PDL probe: a one-CTA kernel that runs for `ns` nanoseconds (bounded by the
// clock, nothing else), then a dependent grid whose CTAs stamp %globaltimer on
// entry (before griddepcontrol.wait) and after it.  With programmatic launch the
// dependent's entry stamps precede the first kernel's end stamp.
__global__ void pdl_probe_first(unsigned long long* stamps, unsigned long long ns) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < ns) {
  }
  stamps[0] = globaltimer_ns();
}

__global__ void pdl_probe_second(unsigned long long* stamps) {
  pdl_trigger();
  const uint64_t t_in = globaltimer_ns();
  pdl_wait();
  const uint64_t t_out = globaltimer_ns();
  if (threadIdx.x == 0) {
    stamps[1 + 2 * blockIdx.x] = t_in;
    stamps[2 + 2 * blockIdx.x] = t_out;
  }
}

cudaError_t pdl_probe(unsigned long long* stamps, int ctas, unsigned long long ns, cudaStream_t st) {
  if (ns > 1000000ull) return cudaErrorInvalidValue;   // at most 1 ms of spinning
  cudaError_t e = launch_pdl(pdl_probe_first, 1, 32, 0, st, stamps, ns);
  if (e != cudaSuccess) return e;
  return launch_pdl(pdl_probe_second, ctas, 32, 0, st, stamps);
}

// Device timestamp ring: one thread stores %globaltimer into ring[slot] after
// the previous kernel on the stream has completed (griddepcontrol.wait waits for
// the whole preceding grid and its memory operations).  Launched between op
// groups of a captured step, the differences of consecutive slots are the
// device time each group took inside a graph replay, on every rank at once.
__global__ void ts_mark_kernel(unsigned long long* ring, int slot) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) ring[slot] = globaltimer_ns();
}

cudaError_t ts_mark(unsigned long long* ring, int slot, cudaStream_t st) {
  launch_pdl(ts_mark_kernel, 1, 32, 0, st, ring, slot);
  return cudaGetLastError();
}

// X[t, i, :] = table[ids[t], :] for every stream i (reference.py:909-911).
__global__ void embed_streams_kernel(const __nv_bfloat16* __restrict__ table, const int* __restrict__ ids, int D,
                                     int hc, __nv_bfloat16* X) {
  pdl_entry();
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
  launch_pdl(embed_streams_kernel, T, 256, 0, st, table, ids, D, hc, X);
  return cudaGetLastError();
}

// out[t] = argmax_v logits[t, v] (first index on ties).
//
// Grid (S, T): CTA s of row t scans columns [s*chunk, (s+1)*chunk) with
// float4 loads (4 in flight per thread), writes its (value, index) to ws, and
// the last CTA of the row to arrive (counter per row, reset by that CTA)
// merges the S partials in order.  S spreads a few rows over many SMs: a
// 129K-entry row read by one CTA is latency-bound.
DSV4_DEV void better(float& bv, int& bi, float ov, int oi) {
  if (ov > bv || (ov == bv && oi < bi)) {
    bv = ov;
    bi = oi;
  }
}

__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ logits, int V, int ld, int* out,
                                                     float* ws_v, int* ws_i, int* counters, float* out_val,
                                                     int idx_base) {
  pdl_entry();
  const int t = blockIdx.y, s = blockIdx.x, S = gridDim.x;
  const float* row = logits + (size_t)t * ld;
  const int chunk = ((V + S - 1) / S + 3) & ~3;
  const int v0 = s * chunk, v1 = min(V, v0 + chunk);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const bool vec = (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  if (vec) {
    const int n4 = (v1 - v0) >> 2;
    const float4* r4 = reinterpret_cast<const float4*>(row + v0);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
      const float4 x = r4[i];
      const int v = v0 + 4 * i;
      better(bv, bi, x.x, v);
      better(bv, bi, x.y, v + 1);
      better(bv, bi, x.z, v + 2);
      better(bv, bi, x.w, v + 3);
    }
    for (int v = v0 + 4 * n4 + threadIdx.x; v < v1; v += blockDim.x) better(bv, bi, row[v], v);
  } else {
    for (int v = v0 + threadIdx.x; v < v1; v += blockDim.x) better(bv, bi, row[v], v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  __shared__ float sv[8];
  __shared__ int si[8];
  __shared__ bool s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) better(bv, bi, sv[w], si[w]);
    if (S == 1) {
      out[t] = bi + idx_base;
      if (out_val) out_val[t] = bv;
    } else {
      ws_v[(size_t)t * S + s] = bv;
      ws_i[(size_t)t * S + s] = bi;
      __threadfence();
      s_last = atomicAdd(&counters[t], 1) == S - 1;
    }
  }
  if (S == 1) return;
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  float fv = -INFINITY;
  int fi = 0x7fffffff;
  for (int k = 0; k < S; ++k) better(fv, fi, __ldcg(ws_v + (size_t)t * S + k), __ldcg(ws_i + (size_t)t * S + k));
  out[t] = fi + idx_base;
  if (out_val) out_val[t] = fv;
  counters[t] = 0;
}

int argmax_splits(int T) { return T >= 148 ? 1 : std::min(32, 296 / std::max(T, 1)); }

cudaError_t argmax_rows(const float* logits, int T, int V, int ld, int* out, float* ws_v, int* ws_i, int* counters,
                        float* out_val, int idx_base, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const int S = (ws_v && ws_i && counters) ? argmax_splits(T) : 1;
  launch_pdl(argmax_kernel, dim3(S, T), 256, 0, st, logits, V, ld, out, ws_v, ws_i, counters, out_val, idx_base);
  return cudaGetLastError();
}

// Vocab-parallel head: every rank holds (value, global index) of its shard's
// best entry per row in symmetric memory.  One CTA publishes this rank's pairs,
// waits (bounded) for every rank's, and keeps the best (the lower index on
// ties, as a single argmax over the whole vocabulary would).  Every rank gets
// the same ids.
__global__ void __launch_bounds__(256) tp_argmax_merge_kernel(PeerSync s, const float* const* peer_val,
                                                              const int* const* peer_idx, int T, int* out,
                                                              uint32_t* err) {
  pdl_entry();
  peer_publish_cta(s);
  peer_wait(s, err, KID_COMM);
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < s.world; ++r) better(bv, bi, peer_val[r][t], peer_idx[r][t]);
    out[t] = bi;
  }
}

cudaError_t tp_argmax_merge(const PeerSync& s, const float* const* peer_val, const int* const* peer_idx, int T,
                            int* out, uint32_t* err, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  launch_pdl(tp_argmax_merge_kernel, 1, 256, 0, st, s, peer_val, peer_idx, T, out, err);
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
  pdl_entry();
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
  launch_pdl(markov_step_kernel, n, 512, 0, st, logits, ld, blk, i, mlog, mld, V, n, toks, ts, memb, R, emb);
  return cudaGetLastError();
}

}  // namespace dsv4
