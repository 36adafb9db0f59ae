// Host-visible interface of the tcgen05 GEMM (gemm.cu).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "peer.h"

namespace dsv4 {

enum GemmKind { KIND_BF16 = 0, KIND_MX8 = 1, KIND_MX4A = 2 };
enum EpiKind { EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU = 2 };

struct GemmParams {
  int M;         // dense: A rows (multiple of 128)
  int N;         // dense: B rows (tokens)
  int k_tiles;   // K / 128 bytes
  int n_tiles;   // dense tile count
  int splits;    // split-K factor (1 = none)
  const uint8_t* sfa;  // A scale chunks [M/128][sfa_ktiles][512]
  int sfa_ktiles;
  const uint8_t* sfb;  // B scale chunks [rows/128][sfb_ktiles][512]
  int sfb_ktiles;
  const int4* tiles;   // grouped: {a_row0, b_row0, b_valid, out_col0}; a_row0 with
                       // kTileA2 set reads the second weight operand (AMaps::m[1], sfa2)
  const int* n_tiles_ptr;
  // batched dense mode: A rows group_rows apart read B columns group_k apart
  int group_rows;
  int group_k;
  void* out;           // out[b_row][out_col0 + m]
  int ldo;
  int m_valid;
  const float* row_scale;  // optional per-B-row multiplier
  // SwiGLU epilogue output (MXFP8 for the next GEMM)
  uint8_t* hq;
  int ldh;
  uint8_t* hsf;
  int h_ktiles;
  float swiglu_limit;
  // split-K: either partial tiles in a global workspace reduced by the last
  // arriving CTA (workspace + tile_counters), or cluster_split: the splits of a
  // tile form one thread-block cluster and reduce through distributed shared memory
  float* workspace;
  int* tile_counters;
  int cluster_split;
  // optional: after the last CTA has stored its tiles, publish the phase to every
  // peer (tensor-parallel partial sums read by the next kernel over NVLink)
  PeerSync pub;
  // optional (grouped, bf16 output): output row b goes to row (ret_meta[b] &
  // 0xffffff) of rank (ret_meta[b] >> 24)'s return buffer ret_peer[rank] (row
  // stride ldo) instead of out -- the expert-parallel combine stores each expert
  // row straight into the source rank's memory over NVLink
  // grouped: second weight operand (the shared expert riding in the routed experts'
  // tile list): scale chunks [M2/128][sfa_ktiles][512]
  const uint8_t* sfa2;
  int M2;
  int a2_e4m3;         // KIND_MX4A: the second operand is e4m3 (MXFP8), not e2m1 -- both sit
                       // one byte per element in shared memory; only the TMA byte count and
                       // the A format of the instruction descriptor differ
  const int* ret_meta;
  __nv_bfloat16* const* ret_peer;
  int ret_world;       // entries of ret_peer (checked in the debug-bounds build)
  uint32_t* err;
};

// Activation tensor maps with box heights 32/64/128/256 rows (grouped GEMMs
// pick one per tile); dense GEMMs use m[0] with box height BN.
struct BMaps {
  CUtensorMap m[4];
};
// Weight tensor maps: m[0] the GEMM's weights; m[1] (grouped GEMMs, optional)
// a second weight matrix of the same K for tiles flagged with kTileA2.
struct AMaps {
  CUtensorMap m[2];
};

int gemm_smem_bytes(int bn);
// bm: weight rows per tile, 128, or 256 (two 128-row MMAs sharing the token tile;
// dense MXFP8/MXFP4 GEMMs with bf16/fp32 outputs and 64/128-token tiles only)
int gemm_max_clusters(int kind, int epi, int bn, int splits, int bm);   // resident clusters of `splits` CTAs
cudaError_t gemm_launch(int kind, int epi, bool grouped, int bn, int bm, const AMaps& ta, const BMaps& tb,
                        const GemmParams& p, int grid, cudaStream_t st);

// 2-D tensor map over a row-major [rows, cols] matrix of 1-byte (e4m3), 2-byte
// (bf16) or packed 4-bit (e2m1, TMA type 16U4_ALIGN16B: unpacked to one byte per element in smem, the operand form of kind::mxf8f6f4)
// elements; box = {128 bytes of K, box_rows}, 128B swizzle.
enum TmaElem { TMA_U8 = 0, TMA_BF16 = 1, TMA_E2M1 = 2 };
bool make_tma_2d(CUtensorMap* map, const void* base, int elem, uint64_t rows, uint64_t cols, uint32_t box_rows);

}  // namespace dsv4
