// Expert-parallel dispatch / combine packing.
//
// Transport record of one (token, expert) pair: [e4m3 row D bytes | ue8m0
// scales D/32 bytes | local expert id int32 | routing weight f32], padded to
// 16 bytes.  The source rank packs every pair into the per-destination region
// of its send buffer (fixed capacity per peer, so the exchange needs no host
// synchronization and replays inside a CUDA graph); the destination unpacks
// records into the permuted expert buffer; expert outputs travel back in
// bf16 rows, and the source combines them through the (peer * cap + slot)
// position of each pair (the mHC boundary kernel reads them directly).
//
// The same packers feed the NCCL all-to-all baseline and the NVLink
// peer-store exchange (records written straight into the owner's receive
// buffer).
#include "common.cuh"
#include "kernels.h"
#include "moe_route.cuh"
#include "peer.cuh"

#include <algorithm>

namespace dsv4 {

// Grid of the packing / unpacking kernels: two CTAs of 256 threads per SM, each
// striding over the valid records (the buffers are sized for the worst case,
// so one thread per capacity slot would launch mostly idle CTAs and make the
// completion counter of the publishing kernels a long chain of atomics).
constexpr long long kEpGrid = 296;

// ------------------------------------------------------------ peer signals
// NVLink transport: after the last CTA of a packing kernel has finished its
// peer stores, it publishes (for the dispatch) this rank's record counts into
// every peer's count array, then release-stores the step's epoch into slot
// [phase * world + my_rank] of every peer's signal array.  The consumer side
// (ep_wait_kernel) acquire-loads its own signal slots until every peer has
// reached the epoch, bounded by kWaitLimitNs.  Epochs advance once per call
// on every rank (all ranks run the same sequence of MoE layers), so no reset
// is needed between CUDA-graph replays.
// Called by every CTA at its end (all threads).  The last CTA publishes.
DSV4_DEV void grid_publish(const EpSync& s, const int* cnt, int world, int my_rank, int cap) {
  __syncthreads();
  if (threadIdx.x != 0 || s.done == nullptr) return;
  __threadfence_system();
  const int prev = atomicAdd(s.done, 1);
  if (prev != (int)gridDim.x - 1) return;
  *s.done = 0;
  const uint32_t ep = *s.epoch + 1u;
  *s.epoch = ep;
  if (s.peer_cnt) {
    for (int p = 0; p < world; ++p) {
      const int c = atomicAdd(const_cast<int*>(cnt) + p, 0);
      s.peer_cnt[p][my_rank] = c < cap ? c : cap;
    }
  }
  __threadfence_system();
  for (int p = 0; p < world; ++p) st_release_sys(s.peer_sig[p] + s.phase * world + my_rank, ep);
}

__global__ void ep_wait_kernel(const uint32_t* sig, int world, int phase, const uint32_t* epoch, uint32_t* err) {
  pdl_entry();
  const int p = threadIdx.x;
  if (p >= world) return;
  const uint32_t want = *epoch;
  const uint32_t* slot = sig + phase * world + p;
  if ((int)(ld_acquire_sys(slot) - want) >= 0) return;
  const uint64_t t0 = globaltimer_ns();
  while ((int)(ld_acquire_sys(slot) - want) < 0) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      report_error(err, ERR_PEER_TIMEOUT, KID_COMM, (uint32_t)(phase * 16 + p));
      return;
    }
  }
}

cudaError_t ep_wait(const uint32_t* sig, int world, int phase, const uint32_t* epoch, uint32_t* err,
                    cudaStream_t st) {
  launch_pdl(ep_wait_kernel, 1, 32, 0, st, sig, world, phase, epoch, err);
  return cudaGetLastError();
}

__global__ void ep_pack_kernel(const int* __restrict__ ids, const float* __restrict__ wts, int T, int topk,
                               const uint8_t* __restrict__ xq, const uint8_t* __restrict__ xsf, int D, int e_local,
                               int world, int cap, int rec, uint8_t* __restrict__ send, int* cnt, int* pos_back,
                               uint8_t* const* peer_recv, int my_rank, uint32_t* err, EpSync sync) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const int n_warps = (int)(gridDim.x * blockDim.x) >> 5;
  for (int w = (int)(blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < T * topk; w += n_warps) {
    const int t = w / topk;
    const int e = ids[w];
    const int dest = e / e_local;
    int slot = 0;
    if (lane == 0) slot = atomicAdd(&cnt[dest], 1);
    slot = __shfl_sync(0xffffffffu, slot, 0);
    if (slot >= cap) {
      if (lane == 0) {
        pos_back[w] = -1;
        report_error(err, ERR_CAPACITY, KID_MOE, 2);
      }
    } else {
      // direct peer store (NVLink) when the peer's receive buffer is mapped, else the local send buffer
      uint8_t* dst = peer_recv ? peer_recv[dest] + ((size_t)my_rank * cap + slot) * rec
                               : send + ((size_t)dest * cap + slot) * rec;
      const uint4* src = reinterpret_cast<const uint4*>(xq + (size_t)t * D);
      for (int i = lane; i < D / 16; i += 32) reinterpret_cast<uint4*>(dst)[i] = src[i];
      const int kt = D / 128;
      for (int b = lane; b < D / 32; b += 32) dst[D + b] = xsf[sf_chunk_offset(t, b, kt)];
      if (lane == 0) {
        *reinterpret_cast<int*>(dst + D + D / 32) = e - dest * e_local;
        *reinterpret_cast<float*>(dst + D + D / 32 + 4) = wts[w];
        pos_back[w] = dest * cap + slot;
      }
    }
  }
  grid_publish(sync, cnt, world, my_rank, cap);
}

cudaError_t ep_pack(const int* ids, const float* wts, int T, int topk, const uint8_t* xq, const uint8_t* xsf, int D,
                    int e_local, int world, int cap, int rec, uint8_t* send, int* cnt, int* pos_back,
                    uint8_t* const* peer_recv, int my_rank, uint32_t* err, const EpSync& sync, cudaStream_t st) {
  const long long warps = (long long)T * topk;
  if (warps == 0 && sync.done == nullptr) return cudaSuccess;
  const unsigned grid = (unsigned)std::min<long long>(kEpGrid, std::max(1LL, (warps * 32 + 255) / 256));
  launch_pdl(ep_pack_kernel, grid, 256, 0, st, ids, wts, T, topk, xq, xsf, D, e_local, world, cap, rec, send, cnt, pos_back,
                                       peer_recv, my_rank, err, sync);
  return cudaGetLastError();
}

// recv [world * cap] records with per-peer counts -> ids/wts of the valid slots
// (slot p * cap + j, j < cnt[p]); the other slots are never read (moe_plan and
// the unpack/combine kernels below visit valid slots only).
__global__ void ep_unpack_meta_kernel(const uint8_t* __restrict__ recv, const int* __restrict__ cnt, int world,
                                      int cap, int rec, int D, int* ids, float* wts) {
  pdl_entry();
  const int n_thr = (int)(gridDim.x * blockDim.x);
  for (int p = 0; p < world; ++p) {
    const int c = min(cnt[p], cap);
    for (int j = (int)(blockIdx.x * blockDim.x + threadIdx.x); j < c; j += n_thr) {
      const size_t i = (size_t)p * cap + j;
      const uint8_t* r = recv + i * rec;
      ids[i] = *reinterpret_cast<const int*>(r + D + D / 32);
      wts[i] = *reinterpret_cast<const float*>(r + D + D / 32 + 4);
    }
  }
}

cudaError_t ep_unpack_meta(const uint8_t* recv, const int* cnt, int world, int cap, int rec, int D, int* ids,
                           float* wts, cudaStream_t st) {
  const long long n = (long long)world * cap;
  const unsigned grid = (unsigned)std::min<long long>(kEpGrid, std::max(1LL, (n + 255) / 256));
  launch_pdl(ep_unpack_meta_kernel, grid, 256, 0, st, recv, cnt, world, cap, rec, D, ids, wts);
  return cudaGetLastError();
}

// Received records -> permuted expert rows (e4m3 + scale chunks), one warp per record.
__global__ void ep_unpack_rows_kernel(const uint8_t* __restrict__ recv, const int* __restrict__ cnt, int world,
                                      int cap, int rec, int D, const int* __restrict__ pos, uint8_t* pq,
                                      uint8_t* psf) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const int n_warps = (int)(gridDim.x * blockDim.x) >> 5;
  const int kt = D / 128;
  for (int p = 0; p < world; ++p) {
    const int c = min(cnt[p], cap);
    for (int j = (int)(blockIdx.x * blockDim.x + threadIdx.x) >> 5; j < c; j += n_warps) {
      const size_t w = (size_t)p * cap + j;
      const int row = pos[w];
      if (row < 0) continue;
      const uint8_t* r = recv + w * rec;
      uint4* dst = reinterpret_cast<uint4*>(pq + (size_t)row * D);
      for (int i = lane; i < D / 16; i += 32) dst[i] = reinterpret_cast<const uint4*>(r)[i];
      for (int b = lane; b < D / 32; b += 32) psf[sf_chunk_offset(row, b, kt)] = r[D + b];
    }
  }
}

cudaError_t ep_unpack_rows(const uint8_t* recv, const int* cnt, int world, int cap, int rec, int D, const int* pos,
                           uint8_t* pq, uint8_t* psf, cudaStream_t st) {
  if (world * cap == 0) return cudaSuccess;
  const unsigned grid = (unsigned)std::min<long long>(kEpGrid, std::max(1LL, ((long long)world * cap * 32 + 255) / 256));
  launch_pdl(ep_unpack_rows_kernel, grid, 256, 0, st, recv, cnt, world, cap, rec, D, pos, pq, psf);
  return cudaGetLastError();
}

// Expert outputs back to record order: back[i] = yperm[pos[i]] (bf16 rows), or
// written straight into the source rank's return buffer over NVLink.
__global__ void ep_combine_pack_kernel(const __nv_bfloat16* __restrict__ yperm, const int* __restrict__ pos,
                                       const int* __restrict__ cnt, int D, int cap, __nv_bfloat16* back,
                                       __nv_bfloat16* const* peer_back, int my_rank, int world, EpSync sync) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const int n_warps = (int)(gridDim.x * blockDim.x) >> 5;
  for (int src_rank = 0; src_rank < world; ++src_rank) {
    const int c = min(cnt[src_rank], cap);
    for (int j = (int)(blockIdx.x * blockDim.x + threadIdx.x) >> 5; j < c; j += n_warps) {
      const size_t w = (size_t)src_rank * cap + j;
      const int row = pos[w];
      if (row < 0) continue;
      __nv_bfloat16* dst = peer_back ? peer_back[src_rank] + ((size_t)my_rank * cap + j) * D : back + w * D;
      const uint4* s = reinterpret_cast<const uint4*>(yperm + (size_t)row * D);
      for (int i = lane; i < D / 8; i += 32) reinterpret_cast<uint4*>(dst)[i] = s[i];
    }
  }
  grid_publish(sync, nullptr, world, my_rank, cap);
}

cudaError_t ep_combine_pack(const __nv_bfloat16* yperm, const int* pos, const int* cnt, int D, int cap,
                            __nv_bfloat16* back, __nv_bfloat16* const* peer_back, int my_rank, int world,
                            const EpSync& sync, cudaStream_t st) {
  const long long n = (long long)world * cap;
  if (n == 0 && sync.done == nullptr) return cudaSuccess;
  const unsigned grid = (unsigned)std::min<long long>(kEpGrid, std::max(1LL, (n * 32 + 255) / 256));
  launch_pdl(ep_combine_pack_kernel, grid, 256, 0, st, yperm, pos, cnt, D, cap, back, peer_back, my_rank, world, sync);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- fused path
// Expert-parallel MoE in three kernels per layer instead of a pack / exchange /
// unpack / plan / combine chain:
//
//   ep_dispatch  router top-k of each token (one warp per token), then each
//                routed pair claims a row of its expert on the owning rank with
//                a system-scope atomic on the owner's per-expert counter and
//                stores the token's MXFP8 row, its scale words, the routing
//                weight and the pair's origin straight into the owner's expert
//                rows (symmetric memory, NVLink stores); the last CTA publishes
//                phase 0.  Expert e of a rank owns rows [e * cap_e, (e+1) * cap_e)
//                (cap_e >= every token of every rank), so no prefix sum over
//                sources is needed and no row is ever copied twice.
//   ep_plan      one CTA: bounded wait until every rank has published phase 0,
//                the W13 / W2 tile lists from the per-expert counts, counters
//                back to zero for the next layer.
//   grouped W13 (SwiGLU epilogue, the routing weight folded in) and grouped W2
//                whose epilogue stores each output row into the source rank's
//                return buffer at the pair's index and publishes phase 1; the
//                next mHC boundary kernel waits for phase 1 and sums the pairs.
//
// Counter reuse: a rank reaches the next layer's dispatch only after every
// owner's W2 of this layer has published, and every owner's ep_plan (which
// zeroed the counters) precedes its W2 in stream order.
// One CTA (8 warps) per token: warp 0 routes the token and claims the k rows on
// their owners; then warp j stores pair j (and j + 8) -- the NVLink row stores
// of a token run in parallel, and every SM is busy at decode-sized token counts.
constexpr int kDispatchMaxD = 8192;   // hidden sizes the dispatch stages in shared memory

template <int kMaxPer>
__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpDispatchParams p) {
  pdl_entry();
  __shared__ int s_owner[16], s_row[16];
  __shared__ float s_w[16];
  __shared__ uint4 s_xrow[kDispatchMaxD / 16];
  __shared__ uint32_t s_sfw[kDispatchMaxD / 128];
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = p.D;
  const int kt = D / 128;
  if (t < p.T) {
    if (warp == 0) {
      int id;
      float w;
      route_token<kMaxPer>(p.logits + (size_t)t * p.E, p.E, p.bias, p.topk, p.score_func, p.route_scale, lane, id,
                           w);
      if (lane < p.topk) {
        if (p.ids) {
          p.ids[(size_t)t * p.topk + lane] = id;
          p.wts[(size_t)t * p.topk + lane] = w;
        }
        const int owner = id / p.e_local;
        const int le = id - owner * p.e_local;
        const int slot = atomicAdd_system(p.peer_cnt[owner] + le, 1);
        int row = -1;
        if (slot < seg_pairs(p.cap_e, p.tile_rows)) {
          row = le * p.cap_e + seg_row(slot, p.tile_rows);
        } else {
          report_error(p.err, ERR_CAPACITY, KID_MOE, 3);
        }
#ifdef DSV4_DEBUG_BOUNDS
        if (owner < 0 || owner >= p.world || (row >= 0 && row >= p.rows)) {
          dbg_bad(BS_EP_OWNER);
          row = -1;
        }
        if (t * p.topk + lane >= p.ret_rows) {
          dbg_bad(BS_EP_RET);
          row = -1;
        }
#endif
        s_owner[lane] = owner;
        s_row[lane] = row;
        s_w[lane] = w;
      }
    }
    // the token's row (D bytes) and its scale words (one 4-byte word per 128
    // columns in the chunk layout) are staged in shared memory once, with every
    // load in flight together, while warp 0 routes; then each warp streams its
    // pairs out of shared memory
    const int nvec = D / 16;
    const int m_src = t & 127;
    const uint4* src = reinterpret_cast<const uint4*>(p.xq + (size_t)t * D);
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) s_xrow[i] = src[i];
    for (int b = threadIdx.x; b < kt; b += blockDim.x)
      s_sfw[b] = *reinterpret_cast<const uint32_t*>(p.xsf + ((size_t)(t >> 7) * kt + b) * 512 + (m_src & 31) * 16 +
                                                    (m_src >> 5) * 4);
    __syncthreads();
    for (int j = warp; j < p.topk; j += 8) {
      const int o = s_owner[j], r = s_row[j];
      if (r < 0) continue;
      uint4* dst = reinterpret_cast<uint4*>(p.peer_x[o] + (size_t)r * D);
      for (int i = lane; i < nvec; i += 32) dst[i] = s_xrow[i];
      const int m = r & 127;
      for (int b = lane; b < kt; b += 32)
        *reinterpret_cast<uint32_t*>(p.peer_xsf[o] + ((size_t)(r >> 7) * kt + b) * 512 + (m & 31) * 16 +
                                     (m >> 5) * 4) = s_sfw[b];
      if (lane == 0) {
        p.peer_rscale[o][r] = s_w[j];
        p.peer_meta[o][r] = (p.rank << 24) | (t * p.topk + j);
      }
    }
    if (p.shared_row0 >= 0 && warp == p.topk % 8) {
      // the shared expert's input: this token's row in this rank's own segment (its
      // row weight 1 and return destination are constant, set at allocation)
      const int r = p.shared_row0 + t;
      uint4* dst = reinterpret_cast<uint4*>(p.peer_x[p.rank] + (size_t)r * D);
      for (int i = lane; i < nvec; i += 32) dst[i] = s_xrow[i];
      const int m = r & 127;
      for (int b = lane; b < kt; b += 32)
        *reinterpret_cast<uint32_t*>(p.peer_xsf[p.rank] + ((size_t)(r >> 7) * kt + b) * 512 + (m & 31) * 16 +
                                     (m >> 5) * 4) = s_sfw[b];
    }
  }
  peer_publish_grid(p.pub);
}

cudaError_t ep_dispatch(const EpDispatchParams& p, cudaStream_t st) {
  if (p.E > 512 || p.topk > 16 || p.topk > p.E || p.D % 128 || p.D < 128 || p.D > kDispatchMaxD)
    return cudaErrorInvalidValue;
  if ((long long)p.T * p.topk >= (1 << 24) || p.world > 127 || p.e_local < 1) return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)std::max(1, p.T);   // every rank publishes, even with T = 0
  const int per = (p.E + 31) / 32;
#define DSV4_DISPATCH(P) launch_pdl(ep_dispatch_kernel<P>, grid, 256, 0, st, p)
  if (per <= 2) DSV4_DISPATCH(2);
  else if (per <= 4) DSV4_DISPATCH(4);
  else if (per <= 8) DSV4_DISPATCH(8);
  else if (per <= 12) DSV4_DISPATCH(12);
  else DSV4_DISPATCH(16);
#undef DSV4_DISPATCH
  return cudaGetLastError();
}

// One CTA of 1024 threads (one expert per thread, e_local <= 1024).
__global__ void __launch_bounds__(1024) ep_plan_kernel(EpPlanParams p) {
  pdl_entry();
  peer_wait(p.wait, p.err, KID_COMM);
  __shared__ int s_wt[32];
  __shared__ int s_ok;
  const int e = threadIdx.x;
  const int lane = e & 31, w = e >> 5;
  int c = 0;
  if (e < p.e_local) {
    c = p.cnt[e];
    // dispatch reported an overflow; pairs past the segment were not written
    c = min(c, seg_pairs(p.cap_e, p.tile_rows));
    p.cnt[e] = 0;                   // re-armed for the next layer (see the counter-reuse note above)
  }
  const int tl = (c + p.tile_rows - 1) / p.tile_rows;
  int it = tl;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int b = __shfl_up_sync(0xffffffffu, it, o);
    if (lane >= o) it += b;
  }
  if (lane == 31) s_wt[w] = it;
  __syncthreads();
  if (w == 0) {
    const int nw = (int)(blockDim.x >> 5);
    int vt = lane < nw ? s_wt[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int b = __shfl_up_sync(0xffffffffu, vt, o);
      if (lane >= o) vt += b;
    }
    s_wt[lane] = vt;
  }
  __syncthreads();
  const int toff = (w > 0 ? s_wt[w - 1] : 0) + it - tl;
  const int mt13 = p.m13 / 128, mt2 = p.m2 / 128;
  const int st = (p.shared_rows + p.tile_rows - 1) / p.tile_rows;   // shared expert row tiles
  if (e == 0) {
    const int total = s_wt[31] + st;
    const bool ok = total * mt13 <= p.max_tiles13 && total * mt2 <= p.max_tiles2;
    if (!ok) report_error(p.err, ERR_CAPACITY, KID_MOE, 4);
    s_ok = ok;
    *p.n_tiles13 = ok ? total * mt13 : 0;
    *p.n_tiles2 = ok ? total * mt2 : 0;
  }
  __syncthreads();
  if (!s_ok) return;
  if (st > 0) {
    // the shared expert: row tiles after the routed ones, weights from the GEMMs' second operand
    const int t0 = s_wt[31];
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
  }
  if (e >= p.e_local) return;
  int rt = toff;
  for (int r0 = 0; r0 < c; r0 += p.tile_rows, ++rt) {
    const int valid = min(p.tile_rows, c - r0);
    const int b0 = e * p.cap_e + seg_tile_row(r0, p.tile_rows);
    for (int mt = 0; mt < mt13; ++mt)
      p.tiles13[(size_t)rt * mt13 + mt] = make_int4(e * p.m13 + mt * 128, b0, valid, mt * 128);
    for (int mt = 0; mt < mt2; ++mt)
      p.tiles2[(size_t)rt * mt2 + mt] = make_int4(e * p.m2 + mt * 128, b0, valid, mt * 128);
  }
}

cudaError_t ep_plan(const EpPlanParams& p, cudaStream_t st) {
  if (p.e_local < 1 || p.e_local > 1024 || p.cap_e % 256 || p.m13 % 128 || p.m2 % 128 ||
      (p.tile_rows != 32 && p.tile_rows != 64 && p.tile_rows != 128 && p.tile_rows != 256))
    return cudaErrorInvalidValue;
  if (p.shared_rows < 0 || (p.shared_rows > 0 && (p.tile_rows < 128 || p.shared_row0 < p.e_local * p.cap_e ||
                                                  p.shared_row0 % 256)))
    return cudaErrorInvalidValue;
  launch_pdl(ep_plan_kernel, 1, 1024, 0, st, p);
  return cudaGetLastError();
}

}  // namespace dsv4
