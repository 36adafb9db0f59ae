// tcgen05 GEMM for sm_100a: D[m, n] = sum_k A[m, k] * B[n, k].
//
// Orientation ("swap-AB"): A is the weight ([out_features, K], K-major), B is
// the activation ([tokens, K], K-major).  The 128-row MMA M side covers output
// features and tokens ride on the N side (16..256), which is what decode-sized
// token counts need.  The result tile D[128 x BN] lives in TMEM and is written
// transposed, out[token][feature].
//
// Kinds:
//   KIND_BF16   tcgen05.mma kind::f16, bf16 x bf16 -> fp32.
//   KIND_MX8    kind::mxf8f6f4.block_scale, e4m3 x e4m3 with ue8m0 scales per
//               32 K-elements on both operands (MXFP8), fp32 accumulate.
//   KIND_MX4A   same with the A operand e2m1 (MXFP4 weights, unpacked to one byte
//               per element in smem by TMA's 16U4_ALIGN16B type; the TMA
//               transaction count is the packed size, half the smem footprint).
// Block scales arrive in the 512-byte "chunk" layout (common.cuh), one chunk per
// (128-row tile, 128-column k tile), moved by a 1-D bulk copy into shared
// memory and by tcgen05.cp into TMEM next to the accumulator.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer (one elected lane), warps 2..5 = epilogue (each reads the TMEM lane
// quadrant it is allowed to access).  The kernel is persistent over a tile list
// (dense: computed; grouped/MoE: device tile records), with optional split-K.
// Split-K reduces deterministically (fixed summation order over splits), either
// through a global workspace by the last-arriving CTA, or -- the default for
// dense GEMMs -- inside a thread-block cluster: the S splits of a tile are one
// cluster, each parks its fp32 partial tile in its own (now idle) pipeline
// shared memory, and after a cluster barrier CTA r reduces column chunks
// r, r+S, ... by reading all S partials over distributed shared memory.
//
// Epilogues: bf16 store, fp32 store, and SwiGLU-requant for expert W13 tiles
// whose rows are [64 gate rows; 64 up rows]: h = silu(min(g, L)) * clip(u, L) *
// row_weight, rounded to bf16 and re-quantized to MXFP8 (e4m3 + ue8m0 per 32)
// for the W2 GEMM, so the intermediate never leaves the chip in high precision.
#include <atomic>

#include "common.cuh"
#include "gemm.h"
#include "peer.cuh"

namespace dsv4 {

template <int BN, int BM = 128>
struct GemmSmem {
  static constexpr int kA = BM * 128;                 // 16 KB per 128 weight rows
  static constexpr int kB = BN * 128;
  static constexpr int kSfaChunks = BM / 128;         // 128-row halves of the weight tile
  static constexpr int kSfbChunks = (BN + 127) / 128;
  static constexpr int kSf = 512 * (kSfaChunks + kSfbChunks);
  static constexpr int kStages = BM == 256 ? (BN >= 128 ? 4 : 5)
                                           : (BN >= 256 ? 4 : (BN >= 128 ? 6 : (BN >= 64 ? 8 : 9)));
  static constexpr int kStage = kA + kB + kSf;
  static constexpr int kXbuf = 4 * 32 * 32 * 4;        // SwiGLU exchange (4 warps x 32 cols x 32 lanes)
  static constexpr int kBarriers = 256;
  static constexpr int kRetPtrs = 32 * 8;              // return-row destinations of one 32-token chunk
  static constexpr int kTotal = 1024 + kStages * kStage + kXbuf + kBarriers + kRetPtrs;
  static_assert(kTotal <= 227 * 1024, "GEMM shared memory exceeds the per-CTA limit");
  static_assert(8 * (2 * kStages + 2 * 2 + 1) + 16 <= kBarriers, "barrier region too small");
  // TMEM: NUM_ACC accumulator buffers (double-buffered when they fit, so the
  // epilogue of one tile overlaps the mainloop of the next), then per-stage
  // scale-factor columns.
  static constexpr int kNumAcc = (BM == 128 && BN <= 128) ? 2 : 1;
  static constexpr int kAccColsHalf = BN < 32 ? 32 : BN;     // one 128-row half of the tile
  static constexpr int kAccCols = kAccColsHalf * kSfaChunks;
  static constexpr int kSfCols = 4 * (kSfaChunks + kSfbChunks);
  static constexpr int kColsNeeded = kNumAcc * kAccCols + kStages * kSfCols;
  static constexpr int kTmemCols = kColsNeeded <= 32 ? 32 : kColsNeeded <= 64 ? 64 : kColsNeeded <= 128 ? 128
                                 : kColsNeeded <= 256 ? 256 : 512;
  static_assert(kColsNeeded <= 512, "TMEM columns exceed one SM's 512");
  static_assert(BM == 128 || BM == 256, "weight tile rows");
};

DSV4_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16(x)); }

struct TileCoord {
  int a_row0, b_row0, b_valid, out_col0, k_begin, k_end, split, tile, n_eff;
  bool a2;     // grouped: the tile reads the second weight operand
  int k_rot;   // the k loop starts at k_begin + k_rot and wraps (0: plain order; a
               // rotated start per tile was measured and gave no gain)
};

// k tile of step i of a tile's mainloop.
DSV4_DEV int k_of(const TileCoord& t, int i) {
  const int nk = t.k_end - t.k_begin;
  int k = i + t.k_rot;
  if (k >= nk) k -= nk;
  return t.k_begin + k;
}

// Per-tile MMA width: the smallest of 32/64/128/256 covering the valid rows.
// Tiles start on 128-row boundaries of the activation buffer (256 for n_eff
// 256), so scale-factor chunks are always used unshifted: the tensor core wants
// scale-factor TMEM addresses on a 4-column boundary.
DSV4_DEV int n_eff_for(int valid) { return valid <= 32 ? 32 : valid <= 64 ? 64 : valid <= 128 ? 128 : 256; }
DSV4_DEV int bmap_index(int n_eff) { return n_eff == 32 ? 0 : n_eff == 64 ? 1 : n_eff == 128 ? 2 : 3; }

// Accumulator columns [c0, c0 + kCols) of this warp's TMEM lane quadrant.  A
// split whose k range is empty (more splits than k tiles allow) issued no MMA,
// so its accumulator holds stale data: it contributes zeros instead.
template <int kCols>
DSV4_DEV void load_acc(uint32_t d_tmem, int q, int c0, uint32_t (&r)[32], bool kempty) {
  if (kempty) {
#pragma unroll
    for (int j = 0; j < 32; ++j) r[j] = 0u;
    return;
  }
  if constexpr (kCols == 32) tmem_ld_32x32b_x32(d_tmem + ((uint32_t)(32 * q) << 16) + c0, r);
  else tmem_ld_32x32b_x16(d_tmem + ((uint32_t)(32 * q) << 16) + c0, *reinterpret_cast<uint32_t(*)[16]>(r));
  tmem_ld_wait();
}

template <bool GROUPED, int BN, int BM = 128>
DSV4_DEV bool get_work(const GemmParams& p, int w, TileCoord& t) {
  const int n_units = (GROUPED ? __ldg(p.n_tiles_ptr) : p.n_tiles) * p.splits;
  if (w >= n_units) return false;
  const int tile = w / p.splits;
  const int split = w % p.splits;
  if (GROUPED) {
    const int4 r = p.tiles[tile];
    t.a2 = (r.x & kTileA2) != 0;
    t.a_row0 = r.x & ~kTileA2;
    t.b_row0 = r.y;
    t.b_valid = r.z;
    t.out_col0 = r.w;
    t.n_eff = min(BN, n_eff_for(r.z));
#ifdef DSV4_DEBUG_BOUNDS
    if (r.x < 0 || t.a_row0 + BM > (t.a2 ? p.M2 : p.M) || (t.a2 && p.sfa2 == nullptr) || r.y < 0 ||
        r.y + t.n_eff > p.N || r.z < 0) {
      dbg_bad(BS_GEMM_TILE);
      return false;   // the rest of this CTA's work list is dropped
    }
#endif
  } else {
    const int m_tiles = p.M / BM;
    const int mt = tile % m_tiles, nt = tile / m_tiles;
    t.a_row0 = mt * BM;
    t.a2 = false;
    t.b_row0 = nt * BN;
    t.b_valid = min(BN, p.N - t.b_row0);
    t.out_col0 = mt * BM;
    t.n_eff = BN;
  }
  const int per = (p.k_tiles + p.splits - 1) / p.splits;
  t.k_begin = split * per;
  t.k_end = min(p.k_tiles, t.k_begin + per);
  t.split = split;
  t.tile = tile;
  t.k_rot = 0;
  return true;
}

template <int KIND, int BN, int EPI, bool GROUPED, int BM = 128>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ AMaps tma_a, const __grid_constant__ BMaps tma_b, GemmParams p) {
  using L = GemmSmem<BN, BM>;
  constexpr bool MX = KIND != KIND_BF16;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + S * L::kA;
  uint8_t* sSF = sB + S * L::kB;
  float* xbuf = reinterpret_cast<float*>(sSF + S * L::kSf);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(xbuf) + L::kXbuf);
  uint8_t** ret_rows = reinterpret_cast<uint8_t**>(reinterpret_cast<uint8_t*>(bars) + L::kBarriers);
  constexpr int NA = L::kNumAcc;
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* acc_full = bars + 2 * S;
  uint64_t* acc_empty = bars + 2 * S + NA;
  uint64_t* drain = bars + 2 * S + 2 * NA;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 2 * NA + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = const_cast<int*>(abort_flag) + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool csplit = p.cluster_split != 0 && p.splits > 1;
  int csyncs = 0;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NA; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a.m[0]);
    if (GROUPED && p.sfa2 != nullptr) tma_prefetch_desc(&tma_a.m[1]);
    tma_prefetch_desc(&tma_b.m[0]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // grouped GEMMs read their tile list from the previous kernel (moe_plan); in
  // dense GEMMs only the producer runs ahead (weight prefetch below)
  if (GROUPED || warp != 0) pdl_wait();

  constexpr int kBkElems = KIND == KIND_BF16 ? 64 : 128;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    TileCoord t;
    constexpr uint32_t kATx = KIND == KIND_MX4A ? L::kA / 2 : L::kA;
    // dense GEMMs: the weight tiles (A + their scales) of the first stages do not
    // depend on the previous kernel, so they stream in while it finishes
    int pre = 0;
    if constexpr (!GROUPED) {
      if (get_work<GROUPED, BN, BM>(p, blockIdx.x, t)) {
        pre = min(S, t.k_end - t.k_begin);
        if (lane == 0) {
          const int sfb_chunks = t.n_eff > 128 ? 2 : 1;
          const uint32_t tx = kATx + t.n_eff * 128 + (MX ? 512 * (L::kSfaChunks + sfb_chunks) : 0);
          for (int i = 0; i < pre; ++i) {
            const int kt = k_of(t, i);
            mbar_arrive_expect_tx(&full[i], tx);
            tma_load_2d(sA + i * L::kA, &tma_a.m[0], &full[i], kt * kBkElems, t.a_row0);
            if constexpr (MX)
              for (int h = 0; h < L::kSfaChunks; ++h)
                bulk_load(sSF + i * L::kSf + 512 * h, p.sfa + ((size_t)((t.a_row0 >> 7) + h) * p.sfa_ktiles + kt) * 512,
                          512, &full[i]);
          }
        }
        __syncwarp();
      }
      pdl_wait();
    }
    bool first = true;
    for (int w = blockIdx.x; get_work<GROUPED, BN, BM>(p, w, t); w += gridDim.x, first = false) {
      const int sfb_chunks = t.n_eff > 128 ? 2 : 1;
      const uint32_t txa = (KIND == KIND_MX4A && t.a2 && p.a2_e4m3) ? (uint32_t)L::kA : kATx;
      const uint32_t tx = txa + t.n_eff * 128 + (MX ? 512 * (L::kSfaChunks + sfb_chunks) : 0);
      const CUtensorMap* bmap = GROUPED ? &tma_b.m[bmap_index(t.n_eff)] : &tma_b.m[0];
      const int b_kofs = p.group_k * (t.a_row0 / p.group_rows);
      const CUtensorMap* amap = t.a2 ? &tma_a.m[1] : &tma_a.m[0];
      const uint8_t* sfa = t.a2 ? p.sfa2 : p.sfa;
      for (int i = 0; i < t.k_end - t.k_begin; ++i) {
        const int kt = k_of(t, i);
        const bool prefetched = first && i < pre;   // fresh stage: its A half is already in flight
        if (!prefetched && !mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.err, KID_GEMM, 1)) goto done;
        if (lane == 0) {
          if (!prefetched) {
            mbar_arrive_expect_tx(&full[stage], tx);
            tma_load_2d(sA + stage * L::kA, amap, &full[stage], kt * kBkElems, t.a_row0);
          }
          tma_load_2d(sB + stage * L::kB, bmap, &full[stage], b_kofs + kt * kBkElems, t.b_row0);
          if constexpr (MX) {
            uint8_t* sf = sSF + stage * L::kSf;
            if (!prefetched)
              for (int h = 0; h < L::kSfaChunks; ++h)
                bulk_load(sf + 512 * h, sfa + ((size_t)((t.a_row0 >> 7) + h) * p.sfa_ktiles + kt) * 512, 512,
                          &full[stage]);
            for (int c = 0; c < sfb_chunks; ++c)
              bulk_load(sf + 512 * (L::kSfaChunks + c),
                        p.sfb + ((size_t)((t.b_row0 >> 7) + c) * p.sfb_ktiles + kt + b_kofs / 128) * 512, 512,
                        &full[stage]);
          }
        }
        __syncwarp();
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    TileCoord t;
    for (int w = blockIdx.x; get_work<GROUPED, BN, BM>(p, w, t); w += gridDim.x) {
      const uint32_t afmt = (KIND == KIND_MX4A && !(t.a2 && p.a2_e4m3)) ? 5 : 0;   // e2m1 or e4m3 weights
      const uint32_t idesc = MX ? idesc_mx(128, t.n_eff, afmt, 0) : idesc_bf16(128, t.n_eff);
      const int sfb_chunks = t.n_eff > 128 ? 2 : 1;
      const uint32_t d_tmem = tmem + acc * L::kAccCols;
      if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, p.err, KID_GEMM, 2)) goto done;
      tc_fence_after();
      for (int i = 0; i < t.k_end - t.k_begin; ++i) {
        if (!mbar_wait(&full[stage], phase, abort_flag, p.err, KID_GEMM, 3)) goto done;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a0 = smem_u32(sA + stage * L::kA);
          const uint32_t b0 = smem_u32(sB + stage * L::kB);
          uint32_t sfa_t = 0, sfb_t = 0;
          if constexpr (MX) {
            const uint32_t sf0 = smem_u32(sSF + stage * L::kSf);
            const uint32_t col = tmem + NA * L::kAccCols + stage * L::kSfCols;
            for (int h = 0; h < L::kSfaChunks; ++h)
              utccp_32x128b_x4(col + 4 * h, umma_sdesc(sf0 + 512 * h, 16, 128, kLayoutNone));
            for (int c = 0; c < sfb_chunks; ++c)
              utccp_32x128b_x4(col + 4 * (L::kSfaChunks + c),
                               umma_sdesc(sf0 + 512 * (L::kSfaChunks + c), 16, 128, kLayoutNone));
            sfa_t = col;
            sfb_t = col + 4 * L::kSfaChunks;
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bd = sdesc_kmajor_sw128(b0 + kk * 32);
            const uint32_t accum = (i > 0 || kk > 0) ? 1u : 0u;
            // 256-row weight tiles: two M=128 MMAs (rows 0-127, 128-255) share the token tile
#pragma unroll
            for (int h = 0; h < L::kSfaChunks; ++h) {
              const uint64_t ad = sdesc_kmajor_sw128(a0 + h * 128 * 128 + kk * 32);
              if constexpr (MX)
                umma_mx(d_tmem + h * L::kAccColsHalf, ad, bd, idesc_mx_sf(idesc, kk), sfa_t + 4 * h, sfb_t, accum);
              else
                umma_bf16(d_tmem + h * L::kAccColsHalf, ad, bd, idesc, accum);
            }
          }
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (lane == 0) umma_commit(&acc_full[acc]);
      __syncwarp();
      if (++acc == NA) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = 32 * q + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    TileCoord t;
    for (int w = blockIdx.x; get_work<GROUPED, BN, BM>(p, w, t); w += gridDim.x) {
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, p.err, KID_GEMM, 4)) goto done;
      tc_fence_after();
      // 256-row weight tiles: the two 128-row halves (TMEM columns BN apart) are
      // finished one after the other; the accumulator is released after the last
      bool tile_done = false;
      for (int hh = 0; hh < L::kSfaChunks && !tile_done; ++hh) {
      const bool last_h = hh == L::kSfaChunks - 1;
      TileCoord th = t;
      th.out_col0 += 128 * hh;
      const uint32_t d_tmem = tmem + acc * L::kAccCols + hh * L::kAccColsHalf;
      const bool kempty = t.k_end <= t.k_begin;
      const bool split = p.splits > 1;
      constexpr int kCols = BN < 32 ? BN : 32;
      constexpr int kPS = BN + 4;   // padded row stride of a parked partial tile (floats)
      float* ws_tile = split && !csplit ? p.workspace + (size_t)th.tile * p.splits * 128 * BN : nullptr;
      int c_begin = 0, c_step = kCols;
      if (csplit) {
        // park this split's partial (row-major, 16-byte stores) in the idle stage buffers
        float* part = reinterpret_cast<float*>(smem);
        for (int c0 = 0; c0 < th.n_eff; c0 += kCols) {
          uint32_t r[32];
          load_acc<kCols>(d_tmem, q, c0, r, kempty);
          float4* dst = reinterpret_cast<float4*>(part + (size_t)row * kPS + c0);
#pragma unroll
          for (int j = 0; j < kCols / 4; ++j)
            dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                 __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && last_h) mbar_arrive(&acc_empty[acc]);
        cluster_sync_all();   // every split's partial is parked
        ++csyncs;
        c_begin = kCols * (int)cluster_ctarank();
        c_step = kCols * p.splits;
        const int nv_tile = min(th.n_eff, th.b_valid);
        // the column-chunk reduction below gives each CTA of the cluster one 32-column
        // chunk; with fewer valid chunks than splits (decode) spread the work instead
        const bool spread = (nv_tile + kCols - 1) / kCols < p.splits && (EPI != EPI_SWIGLU || nv_tile <= 8);
        if (EPI != EPI_SWIGLU && spread) {
          // Spread (row, 4-token group) items of the valid token columns over every
          // CTA of the cluster: each item sums its S partials (independent DSMEM
          // loads, fixed order s = 0..S-1) and stores 4 outputs.  Decode tiles hold
          // one or a few valid tokens, so this reads a small part of each partial.
          const int nv = min(th.n_eff, th.b_valid);
          const int items = 128 * ((nv + 3) >> 2);
          const int etid = threadIdx.x - 64;
          constexpr int kEl = EPI == EPI_F32 ? 4 : 2;
          for (int it = (int)cluster_ctarank() * 128 + etid; it < items; it += p.splits * 128) {
            const int r = it & 127, c4 = it >> 7;
            const uint32_t local = smem_u32(part + (size_t)r * kPS + 4 * c4);
            float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
            for (int sp = 0; sp < p.splits; ++sp) {
              const float4 x = dsmem_ld_f4(dsmem_map(local, (uint32_t)sp));
              acc4.x += x.x, acc4.y += x.y, acc4.z += x.z, acc4.w += x.w;
            }
            const int m = th.out_col0 + r;
            if (m >= p.m_valid) continue;
            const float vals[4] = {acc4.x, acc4.y, acc4.z, acc4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int n = 4 * c4 + j;
              if (n >= nv) break;
              float x = vals[j];
              if (p.row_scale) x *= __ldg(p.row_scale + th.b_row0 + n);
              uint8_t* dst = reinterpret_cast<uint8_t*>(p.out) + ((size_t)(th.b_row0 + n) * p.ldo + m) * kEl;
              if constexpr (EPI == EPI_F32)
                *reinterpret_cast<float*>(dst) = x;
              else
                *reinterpret_cast<__nv_bfloat16*>(dst) = __float2bfloat16(x);
            }
          }
          c_begin = th.n_eff;   // nothing left for the column-chunk loop below
        } else if (EPI == EPI_SWIGLU && spread) {
          // SwiGLU: a warp item is (token n, 32-block ib of the tile's 64 intermediate
          // indices); lane l sums gate row 32*ib + l and up row 64 + 32*ib + l over
          // the splits (fixed order), then the same SwiGLU / clamp / row scale /
          // MXFP8 requant as the column-chunk epilogue below (one scale per 32 indices).
          const int nv = min(th.n_eff, th.b_valid);
          const int n_items = 2 * nv;
          const int gw = (int)cluster_ctarank() * 4 + (warp - 2);
          const float lim = p.swiglu_limit;
          for (int it = gw; it < n_items; it += 4 * p.splits) {
            const int n = it >> 1, ib = it & 1;
            const int i_local = 32 * ib + lane;
            const uint32_t lg = smem_u32(part + (size_t)i_local * kPS + n);
            const uint32_t lu = smem_u32(part + (size_t)(64 + i_local) * kPS + n);
            float gsum = 0.f, usum = 0.f;
#pragma unroll 8
            for (int sp = 0; sp < p.splits; ++sp) {
              gsum += dsmem_ld_f32(dsmem_map(lg, (uint32_t)sp));
              usum += dsmem_ld_f32(dsmem_map(lu, (uint32_t)sp));
            }
            float gv = bf16_round(gsum), u = bf16_round(usum);
            if (lim > 0.f) {
              u = fminf(fmaxf(u, -lim), lim);
              gv = fminf(gv, lim);
            }
            float h = gv / (1.f + expf(-gv)) * u;
            const int brow = th.b_row0 + n;
            if (p.row_scale) h *= __ldg(p.row_scale + brow);
            h = bf16_round(h);
            const float amax = fmaxf(warp_max(fabsf(h)), 1e-4f);
            const uint32_t e = pow2_ceil_exp(amax, 1.f / 448.f);
            const float qv = fminf(fmaxf(h / exp_to_f32(e), -448.f), 448.f);
            const int i_global = (th.out_col0 >> 1) + i_local;
            p.hq[(size_t)brow * p.ldh + i_global] = f32_to_e4m3(qv);
            if (lane == 0) p.hsf[sf_chunk_offset(brow, i_global >> 5, p.h_ktiles)] = (uint8_t)e;
          }
          c_begin = th.n_eff;
        }
      } else if (split) {
        // Publish this split's partial tile, then let the last arrival reduce.
        for (int c0 = 0; c0 < th.n_eff; c0 += kCols) {
          uint32_t r[32];
          load_acc<kCols>(d_tmem, q, c0, r, kempty);
          // row-major partial tile: each thread stores whole 16-byte column groups of its row
          float4* dst = reinterpret_cast<float4*>(ws_tile + (size_t)th.split * 128 * BN + (size_t)row * BN + c0);
#pragma unroll
          for (int j = 0; j < kCols / 4; ++j)
            dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                 __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && last_h) mbar_arrive(&acc_empty[acc]);
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          const int prev = atomicAdd(&p.tile_counters[th.tile], 1);
          *last_flag = (prev == p.splits - 1);
          if (prev == p.splits - 1) p.tile_counters[th.tile] = 0;  // re-arm for the next launch
          __threadfence();
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (!*last_flag) {
          tile_done = true;   // another split reduces this tile
          continue;
        }
        __threadfence();
      }
      for (int c0 = c_begin; c0 < th.n_eff; c0 += c_step) {
        float v[32];
        if (csplit) {
          // fixed summation order s = 0..splits-1 over the cluster's parked partials
#pragma unroll
          for (int j = 0; j < kCols; ++j) v[j] = 0.f;
          const uint32_t local = smem_u32(reinterpret_cast<float*>(smem) + (size_t)row * kPS + c0);
          for (int s = 0; s < p.splits; ++s) {
            const uint32_t ra = dsmem_map(local, (uint32_t)s);
            float4 x[kCols / 4];
#pragma unroll
            for (int j = 0; j < kCols / 4; ++j) x[j] = dsmem_ld_f4(ra + 16 * j);
#pragma unroll
            for (int j = 0; j < kCols / 4; ++j)
              v[4 * j] += x[j].x, v[4 * j + 1] += x[j].y, v[4 * j + 2] += x[j].z, v[4 * j + 3] += x[j].w;
          }
        } else if (split) {
          // fixed summation order s = 0..splits-1 (deterministic); two splits' loads in flight
#pragma unroll
          for (int j = 0; j < kCols; ++j) v[j] = 0.f;
          int s = 0;
          for (; s + 1 < p.splits; s += 2) {
            const float4* a = reinterpret_cast<const float4*>(ws_tile + (size_t)s * 128 * BN + (size_t)row * BN + c0);
            const float4* b = reinterpret_cast<const float4*>(ws_tile + (size_t)(s + 1) * 128 * BN +
                                                              (size_t)row * BN + c0);
            float4 x[kCols / 4], y[kCols / 4];
#pragma unroll
            for (int j = 0; j < kCols / 4; ++j) x[j] = __ldcg(a + j);
#pragma unroll
            for (int j = 0; j < kCols / 4; ++j) y[j] = __ldcg(b + j);
#pragma unroll
            for (int j = 0; j < kCols / 4; ++j) {
              v[4 * j] += x[j].x, v[4 * j + 1] += x[j].y, v[4 * j + 2] += x[j].z, v[4 * j + 3] += x[j].w;
              v[4 * j] += y[j].x, v[4 * j + 1] += y[j].y, v[4 * j + 2] += y[j].z, v[4 * j + 3] += y[j].w;
            }
          }
          if (s < p.splits) {
            const float4* a = reinterpret_cast<const float4*>(ws_tile + (size_t)s * 128 * BN + (size_t)row * BN + c0);
#pragma unroll
            for (int j = 0; j < kCols / 4; ++j) {
              const float4 x = __ldcg(a + j);
              v[4 * j] += x.x, v[4 * j + 1] += x.y, v[4 * j + 2] += x.z, v[4 * j + 3] += x.w;
            }
          }
        } else {
          uint32_t r[32];
          load_acc<kCols>(d_tmem, q, c0, r, kempty);
#pragma unroll
          for (int j = 0; j < kCols; ++j) v[j] = __uint_as_float(r[j]);
        }
        if constexpr (EPI == EPI_SWIGLU) {
          // rows 0..63 gate, 64..127 up (same 64 intermediate indices).  Every warp
          // stages its 32 columns, then warp w finishes row group (w & 1) for the
          // column half (w >> 1): all four warps share the SwiGLU/requant work.
#pragma unroll
          for (int j = 0; j < kCols; ++j) xbuf[(q * 32 + j) * 32 + lane] = v[j];
          asm volatile("bar.sync 1, 128;" ::: "memory");
          {
            const int g = q & 1, half = q >> 1;
            const int i_local = 32 * g + lane;
            const int i_global = (th.out_col0 >> 1) + i_local;  // out_col0 = 128 * m-tile
            const int kblk = i_global >> 5;
            const float lim = p.swiglu_limit;
            const int j0 = half * (kCols / 2);
#pragma unroll 4
            for (int jj = 0; jj < kCols / 2; ++jj) {
              const int j = j0 + jj;
              const int n = c0 + j;
              float gv = bf16_round(xbuf[(g * 32 + j) * 32 + lane]);
              float u = bf16_round(xbuf[((2 + g) * 32 + j) * 32 + lane]);
              if (lim > 0.f) {
                u = fminf(fmaxf(u, -lim), lim);
                gv = fminf(gv, lim);
              }
              float h = gv / (1.f + expf(-gv)) * u;
              const int brow = th.b_row0 + n;
              if (p.row_scale && n < th.b_valid) h *= __ldg(p.row_scale + brow);
              h = bf16_round(h);
              const float amax = fmaxf(warp_max(fabsf(h)), 1e-4f);
              const uint32_t e = pow2_ceil_exp(amax, 1.f / 448.f);
              const float qv = fminf(fmaxf(h / exp_to_f32(e), -448.f), 448.f);
              if (n < th.b_valid) {
                p.hq[(size_t)brow * p.ldh + i_global] = f32_to_e4m3(qv);
                if (lane == 0) p.hsf[sf_chunk_offset(brow, kblk, p.h_ktiles)] = (uint8_t)e;
              }
            }
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        } else {
          // Stage the 32 x 128 chunk in shared memory as [token][feature] and store
          // whole 256-byte (bf16) / 512-byte (fp32) token rows with 16-byte writes.
          constexpr int kEl = EPI == EPI_F32 ? 4 : 2;
          uint8_t* stage = reinterpret_cast<uint8_t*>(xbuf);   // 32 x 128 x 4 B = 16 KB
          if (GROUPED && p.ret_meta != nullptr && row < kCols && c0 + row < th.b_valid) {
            // destination row of each token of the chunk, resolved once (its load
            // overlaps the staging below instead of sitting in front of every store)
            int mt = __ldg(p.ret_meta + th.b_row0 + c0 + row);
#ifdef DSV4_DEBUG_BOUNDS
            if ((mt >> 24) < 0 || (mt >> 24) >= p.ret_world) {
              dbg_bad(BS_GEMM_RET);
              mt = 0;
            }
#endif
            ret_rows[row] = reinterpret_cast<uint8_t*>(p.ret_peer[mt >> 24]) + (size_t)(mt & 0xffffff) * p.ldo * kEl;
          }
#pragma unroll
          for (int j = 0; j < kCols; ++j) {
            float x = v[j];
            if (p.row_scale && c0 + j < th.b_valid) x *= __ldg(p.row_scale + th.b_row0 + c0 + j);
            if constexpr (EPI == EPI_F32)
              reinterpret_cast<float*>(stage)[j * 128 + row] = x;
            else
              reinterpret_cast<__nv_bfloat16*>(stage)[j * 128 + row] = __float2bfloat16(x);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          constexpr int kVecPerRow = 128 * kEl / 16;   // 16 (bf16) or 32 (fp32) vectors per token row
          const int tid = threadIdx.x - 64;
          const bool full_m = th.out_col0 + 128 <= p.m_valid && (p.ldo * kEl) % 16 == 0;
          for (int e = tid; e < kCols * kVecPerRow; e += 128) {
            const int j = e / kVecPerRow, vi = e % kVecPerRow;
            if (c0 + j >= th.b_valid) continue;
            const size_t orow = (size_t)(th.b_row0 + c0 + j) * p.ldo;
            const uint4 val = reinterpret_cast<const uint4*>(stage + (size_t)j * 128 * kEl)[vi];
            if (GROUPED && p.ret_meta != nullptr) {
              // expert-parallel return: straight into the source rank's buffer (NVLink)
              reinterpret_cast<uint4*>(ret_rows[j] + (size_t)th.out_col0 * kEl)[vi] = val;
            } else if (full_m) {
              reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.out) + (orow + th.out_col0) * kEl)[vi] = val;
            } else {
              const int m0 = th.out_col0 + vi * (16 / kEl);
              const uint8_t* src = reinterpret_cast<const uint8_t*>(&val);
              for (int b = 0; b < 16 / kEl; ++b)
                if (m0 + b < p.m_valid)
                  memcpy(reinterpret_cast<uint8_t*>(p.out) + (orow + m0 + b) * kEl, src + b * kEl, kEl);
            }
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
      }
      if (csplit) {
        cluster_sync_all();   // the cluster has finished reading this CTA's partial
        ++csyncs;
      }
      if (!split) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && last_h) mbar_arrive(&acc_empty[acc]);
      }
      }   // halves
      if (++acc == NA) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
done:
  __syncwarp();
  // cluster split: every thread takes part in exactly two cluster barriers (the
  // epilogue's, or here for the producer/MMA warps and after an abort), so no
  // CTA of the cluster can be left waiting
  if (csplit)
    while (csyncs < 2 * L::kSfaChunks) {
      cluster_sync_all();
      ++csyncs;
    }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (*abort_flag) {
      // Make sure no tensor-core op still reads TMEM before releasing it.
      if (lane == 0) umma_commit(drain);
      __syncwarp();
      mbar_wait(drain, 0, nullptr, p.err, KID_GEMM, 5);
    }
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
  peer_publish_grid(p.pub);
}

// ------------------------------------------------------------------- host
template <int KIND, int BN, int EPI, bool GROUPED, int BM = 128>
static cudaError_t launch_one(const AMaps& ta, const BMaps& tb, const GemmParams& p, int grid,
                              cudaStream_t st) {
  using L = GemmSmem<BN, BM>;
  auto k = gemm_kernel<KIND, BN, EPI, GROUPED, BM>;
  // the shared-memory attribute is a per-device setting of the function: set it
  // once on every device this instantiation launches on
  static std::atomic<uint64_t> configured{0};
  {
    const cudaError_t e = smem_attr_once(k, L::kTotal, configured);
    if (e != cudaSuccess) return e;
  }
  if (p.cluster_split && p.splits > 1) {
    // one CTA per (tile, split); the splits of a tile are one cluster
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(192);
    cfg.dynamicSmemBytes = L::kTotal;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, k, ta, tb, p);
  }
  return launch_pdl(k, grid, 192, L::kTotal, st, ta, tb, p);
}

template <int KIND, int EPI, bool GROUPED>
static cudaError_t dispatch_bn(int bn, int bm, const AMaps& ta, const BMaps& tb, const GemmParams& p, int grid,
                               cudaStream_t st) {
  if constexpr (KIND != KIND_BF16 && !GROUPED && EPI != EPI_SWIGLU) {
    if (bm == 256) {
      switch (bn) {
        case 64: return launch_one<KIND, 64, EPI, GROUPED, 256>(ta, tb, p, grid, st);
        case 128: return launch_one<KIND, 128, EPI, GROUPED, 256>(ta, tb, p, grid, st);
        default: return cudaErrorInvalidValue;
      }
    }
  }
  if (bm != 128) return cudaErrorInvalidValue;
  switch (bn) {
    case 32: return launch_one<KIND, 32, EPI, GROUPED>(ta, tb, p, grid, st);
    case 64: return launch_one<KIND, 64, EPI, GROUPED>(ta, tb, p, grid, st);
    case 128: return launch_one<KIND, 128, EPI, GROUPED>(ta, tb, p, grid, st);
    case 256: return launch_one<KIND, 256, EPI, GROUPED>(ta, tb, p, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

// How many clusters of `splits` CTAs of this kernel can be resident at once
// (clusters live inside one GPC, so this is below SMs / splits).  Cached.
template <int KIND, int BN, int EPI, int BM = 128>
static int cluster_cap(int splits) {
  // per device: the answer depends on the GPU's SM and GPC layout
  constexpr int kDevs = 64;
  static std::atomic<int> cache[kDevs][9] = {};
  if (splits < 2 || splits > 8) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
    (void)cudaGetLastError();
    return 0;
  }
  const int c = dev < kDevs ? cache[dev][splits].load(std::memory_order_relaxed) : 0;
  if (c) return c;
  using L = GemmSmem<BN, BM>;
  auto k = gemm_kernel<KIND, BN, EPI, false, BM>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)splits);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = L::kTotal;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  if (dev < kDevs) cache[dev][splits].store(n, std::memory_order_relaxed);
  return n;
}

template <int KIND, int EPI>
static int cap_bn(int bn, int splits, int bm) {
  if constexpr (KIND != KIND_BF16 && EPI != EPI_SWIGLU) {
    if (bm == 256) {
      switch (bn) {
        case 64: return cluster_cap<KIND, 64, EPI, 256>(splits);
        case 128: return cluster_cap<KIND, 128, EPI, 256>(splits);
        default: return 0;
      }
    }
  }
  if (bm != 128) return 0;
  switch (bn) {
    case 32: return cluster_cap<KIND, 32, EPI>(splits);
    case 64: return cluster_cap<KIND, 64, EPI>(splits);
    case 128: return cluster_cap<KIND, 128, EPI>(splits);
    case 256: return cluster_cap<KIND, 256, EPI>(splits);
    default: return 0;
  }
}

int gemm_max_clusters(int kind, int epi, int bn, int splits, int bm) {
  if (kind == KIND_BF16) {
    if (epi == EPI_BF16) return cap_bn<KIND_BF16, EPI_BF16>(bn, splits, bm);
    if (epi == EPI_F32) return cap_bn<KIND_BF16, EPI_F32>(bn, splits, bm);
    return 0;
  }
  if (kind == KIND_MX8) {
    if (epi == EPI_BF16) return cap_bn<KIND_MX8, EPI_BF16>(bn, splits, bm);
    if (epi == EPI_F32) return cap_bn<KIND_MX8, EPI_F32>(bn, splits, bm);
    if (epi == EPI_SWIGLU) return cap_bn<KIND_MX8, EPI_SWIGLU>(bn, splits, bm);
  }
  if (kind == KIND_MX4A) {
    if (epi == EPI_BF16) return cap_bn<KIND_MX4A, EPI_BF16>(bn, splits, bm);
    if (epi == EPI_F32) return cap_bn<KIND_MX4A, EPI_F32>(bn, splits, bm);
    if (epi == EPI_SWIGLU) return cap_bn<KIND_MX4A, EPI_SWIGLU>(bn, splits, bm);
  }
  return 0;
}

int gemm_smem_bytes(int bn) {
  switch (bn) {
    case 32: return GemmSmem<32>::kTotal;
    case 64: return GemmSmem<64>::kTotal;
    case 128: return GemmSmem<128>::kTotal;
    case 256: return GemmSmem<256>::kTotal;
    default: return -1;
  }
}

cudaError_t gemm_launch(int kind, int epi, bool grouped, int bn, int bm, const AMaps& ta, const BMaps& tb,
                        const GemmParams& p, int grid, cudaStream_t st) {
  if (kind == KIND_BF16) {
    if (grouped) return cudaErrorInvalidValue;
    if (epi == EPI_BF16) return dispatch_bn<KIND_BF16, EPI_BF16, false>(bn, bm, ta, tb, p, grid, st);
    if (epi == EPI_F32) return dispatch_bn<KIND_BF16, EPI_F32, false>(bn, bm, ta, tb, p, grid, st);
    return cudaErrorInvalidValue;
  }
#define DSV4_MX(KD)                                                                                  \
  if (kind == KD) {                                                                                  \
    if (!grouped) {                                                                                  \
      if (epi == EPI_BF16) return dispatch_bn<KD, EPI_BF16, false>(bn, bm, ta, tb, p, grid, st);         \
      if (epi == EPI_F32) return dispatch_bn<KD, EPI_F32, false>(bn, bm, ta, tb, p, grid, st);           \
      if (epi == EPI_SWIGLU) return dispatch_bn<KD, EPI_SWIGLU, false>(bn, bm, ta, tb, p, grid, st);     \
    } else {                                                                                         \
      if (epi == EPI_BF16) return dispatch_bn<KD, EPI_BF16, true>(bn, bm, ta, tb, p, grid, st);          \
      if (epi == EPI_F32) return dispatch_bn<KD, EPI_F32, true>(bn, bm, ta, tb, p, grid, st);            \
      if (epi == EPI_SWIGLU) return dispatch_bn<KD, EPI_SWIGLU, true>(bn, bm, ta, tb, p, grid, st);      \
    }                                                                                                \
    return cudaErrorInvalidValue;                                                                    \
  }
  DSV4_MX(KIND_MX8)
  DSV4_MX(KIND_MX4A)
#undef DSV4_MX
  return cudaErrorInvalidValue;
}

}  // namespace dsv4
