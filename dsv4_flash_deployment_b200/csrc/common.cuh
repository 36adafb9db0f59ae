// Shared device helpers for the sm_100a kernels of this engine.
//
// * PTX wrappers: mbarrier, TMA tile loads (plain, each CTA loads its own tiles),
//   1-D bulk copies, tcgen05 (alloc / mma / commit / cp / ld / fences).
// * Bounded waits: every spin in this code base is limited by wall time read
//   from %globaltimer.  On expiry the waiting thread records an error code in a
//   device error word (host reads it and raises) and the kernel unwinds: no
//   wait may hang a GPU.
// * Descriptor builders for the 5th-generation tensor core (UMMA shared-memory
//   matrix descriptors and instruction descriptors).  Field positions follow the
//   public sm_100 descriptor definitions (CUTLASS cute/arch/mma_sm100_desc.hpp).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>
#include <vector>

#include "kernels.h"

#define DSV4_DEV __device__ __forceinline__

namespace dsv4 {


// ------------------------------------------------------------------ errors
// Error word layout: bits [0,8) code, [8,16) kernel id, [16,32) detail.
enum ErrCode : uint32_t {
  ERR_NONE = 0,
  ERR_WAIT_TIMEOUT = 1,
  ERR_PEER_TIMEOUT = 2,
  ERR_BAD_ARG = 3,
  ERR_CAPACITY = 4,
};

enum KernelId : uint32_t {
  KID_GEMM = 1,
  KID_ATTN = 2,
  KID_MOE = 3,
  KID_COMM = 4,
  KID_MEGA = 5,
  KID_BOUNDS = 6,   // debug-bounds build: an index check failed (detail = site)
};

DSV4_DEV void report_error(uint32_t* err, uint32_t code, uint32_t kid, uint32_t detail) {
  if (err) atomicCAS(err, 0u, code | (kid << 8) | (detail << 16));
}

// ------------------------------------------------------------ debug bounds
// Compiled with -DDSV4_DEBUG_BOUNDS (the separate debug extension, built when
// DSV4_DEBUG_BOUNDS=1), cache gathers and writes check their indices: a bad
// one is recorded as ERR_BAD_ARG / KID_BOUNDS in the device error word and the
// access goes to row 0 of the same buffer instead, so the kernel completes and
// the host raises on its next check.  Every translation unit has its own copy
// of the error-word pointer; dbg_bounds_attach() (misc.cu) sets all of them
// for the current device.  In the default build all of this compiles away.
enum BoundsSite : uint32_t {
  BS_KV_ENTRY = 1,      // compressed entry index outside [0, max_c) or a negative slot
  BS_KV_UNMAPPED = 2,   // paged cache: the entry's block is not mapped (table entry < 0)
  BS_EP_OWNER = 3,      // expert-parallel dispatch: owner rank or expert row out of range
  BS_EP_RET = 4,        // expert-parallel dispatch: return row index out of range
  BS_GEMM_TILE = 5,     // grouped GEMM tile outside the A or B operand rows
  BS_GEMM_RET = 6,      // grouped GEMM return row: source rank out of range
  BS_MOE_ROW = 7,       // MoE plan / scatter: a permuted row outside the permuted buffers
};

using DbgSetter = cudaError_t (*)(uint32_t*);
std::vector<DbgSetter>& dbg_registry();   // misc.cu

#ifdef DSV4_DEBUG_BOUNDS
static __device__ uint32_t* dsv4_dbg_err;

DSV4_DEV void dbg_bad(uint32_t site) { report_error(dsv4_dbg_err, ERR_BAD_ARG, KID_BOUNDS, site); }

namespace {
cudaError_t dbg_set_this_unit(uint32_t* p) { return cudaMemcpyToSymbol(dsv4_dbg_err, &p, sizeof(p)); }
struct DbgRegistrar {
  DbgRegistrar() { dbg_registry().push_back(&dbg_set_this_unit); }
};
DbgRegistrar dbg_registrar_instance;
}  // namespace
#endif

// Row of compressed entry ci of sequence slot `slot` in a (paged or contiguous) cache.
DSV4_DEV size_t kv_row(const KvPages& pg, int slot, int ci, int max_c) {
#ifdef DSV4_DEBUG_BOUNDS
  if (ci < 0 || ci >= max_c || slot < 0) {
    dbg_bad(BS_KV_ENTRY);
    return 0;
  }
#endif
  if (pg.table == nullptr) return (size_t)slot * max_c + ci;
  const int blk = pg.table[(size_t)slot * pg.ld + (ci >> pg.shift)];
#ifdef DSV4_DEBUG_BOUNDS
  if (blk < 0) {
    dbg_bad(BS_KV_UNMAPPED);
    return 0;
  }
#endif
  return ((size_t)blk << pg.shift) + (ci & ((1 << pg.shift) - 1));
}

DSV4_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Default limit for any device-side wait (2 s).  A healthy pipeline waits
// microseconds; only a bug or a dead peer reaches this.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// ------------------------------------------- programmatic dependent launch
// Every kernel of this library is launched with programmatic stream
// serialization (launch_pdl) and begins with pdl_entry(): it lets the next
// kernel of the stream be scheduled right away (its CTAs take free SM slots
// and run their own preamble, e.g. a GEMM's weight prefetch) and then waits
// until the previous kernel has completed and its writes are visible.  Nothing
// that depends on, or overwrites, another kernel's data may run before
// pdl_wait().  Without the launch attribute both are no-ops.
DSV4_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
DSV4_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
DSV4_DEV void pdl_entry() {
  pdl_trigger();
  pdl_wait();
}

// DSV4_PDL=0 in the environment turns the launch attribute off (A/B timing).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

DSV4_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
DSV4_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

DSV4_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

DSV4_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

DSV4_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

DSV4_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  ``abort`` is a CTA-shared flag: once any
// role gives up, every other waiter in the CTA gives up too.
DSV4_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint32_t* err,
                        uint32_t kid, uint32_t detail) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort && *abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      if (abort) *abort = 1;
      report_error(err, ERR_WAIT_TIMEOUT, kid, detail);
      return false;
    }
  }
}

// ---------------------------------------------------------------- clusters
// Thread-block cluster barrier (every thread of every CTA of the cluster) and
// distributed shared memory reads.
DSV4_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

DSV4_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA ``rank`` of this cluster.
DSV4_DEV uint32_t dsmem_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

DSV4_DEV float4 dsmem_ld_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

DSV4_DEV float dsmem_ld_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// --------------------------------------------------------------------- TMA
DSV4_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

DSV4_DEV void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// 1-D bulk global->shared copy; both addresses 16-byte aligned, bytes % 16 == 0.
DSV4_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

DSV4_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ----------------------------------------------------------------- tcgen05
DSV4_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
DSV4_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;"); }
DSV4_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
DSV4_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DSV4_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

DSV4_DEV void umma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

DSV4_DEV void umma_mx(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa, uint32_t sfb, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}

DSV4_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Copy a 32-row x 16-byte shared-memory block to TMEM lanes 0..31 of the given
// columns, replicated into all four lane quadrants.
DSV4_DEV void utccp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread.
DSV4_DEV void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

DSV4_DEV void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

DSV4_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------- descriptors
// UMMA shared-memory matrix descriptor (sm_100 "version 1").
DSV4_DEV uint64_t umma_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}
constexpr uint32_t kLayoutSw128 = 2;
constexpr uint32_t kLayoutNone = 0;

// K-major operand tile, 128-byte rows, 128B swizzle, 8-row groups 1024 B apart.
DSV4_DEV uint64_t sdesc_kmajor_sw128(uint32_t saddr) { return umma_sdesc(saddr, 16, 1024, kLayoutSw128); }

// Instruction descriptor, kind::f16 with bf16 inputs and fp32 accumulate.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t m, uint32_t n) {
  return (1u << 4)            // D format f32
         | (1u << 7)          // A bf16
         | (1u << 10)         // B bf16
         | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Instruction descriptor, kind::mxf8f6f4 with ue8m0 block scales.
// fmt: 0 = e4m3, 5 = e2m1.  sf_id selects the scale byte (k-block) in the TMEM word.
__host__ __device__ constexpr uint32_t idesc_mx(uint32_t m, uint32_t n, uint32_t afmt, uint32_t bfmt) {
  return (afmt << 7) | (bfmt << 10) | ((n >> 3) << 17) | (1u << 23) | ((m >> 4) << 24);
}
DSV4_DEV uint32_t idesc_mx_sf(uint32_t base, uint32_t sf_id) { return base | (sf_id << 29) | (sf_id << 4); }

// ------------------------------------------------------------------ numerics
// 2^ceil(log2(amax * inv_max)) as a biased exponent byte, from IEEE bits.
DSV4_DEV uint32_t pow2_ceil_exp(float amax, float inv_max) {
  float prod = amax * inv_max;
  uint32_t bits = __float_as_uint(prod);
  int e = (int)((bits >> 23) & 0xFF) + ((bits & 0x7FFFFF) != 0 ? 1 : 0);
  e = e < 0 ? 0 : (e > 254 ? 254 : e);
  return (uint32_t)e;
}
DSV4_DEV float exp_to_f32(uint32_t e) { return __uint_as_float(e << 23); }

DSV4_DEV uint8_t f32_to_e4m3(float v) {
  __nv_fp8_e4m3 q(v);  // round-to-nearest-even, saturating to +-448
  return *reinterpret_cast<uint8_t*>(&q);
}
DSV4_DEV float e4m3_to_f32(uint8_t b) {
  __nv_fp8_e4m3 q;
  *reinterpret_cast<uint8_t*>(&q) = b;
  return float(q);
}

// ------------------------------------------------------ cache row records
// (layouts: kv8_bytes / kv4_bytes / ik4_bytes in kernels.h)
// E2M1 code of x at scale s (bit 3 = sign): exact midpoint compares, ties to even.
DSV4_DEV uint32_t e2m1_code(float x, float s) {
  const float ax = fabsf(x);
  const uint32_t mag = (ax > 0.25f * s) + (ax >= 0.75f * s) + (ax > 1.25f * s) + (ax >= 1.75f * s) +
                       (ax > 2.5f * s) + (ax >= 3.5f * s) + (ax > 5.0f * s);
  return mag | (signbit(x) ? 8u : 0u);
}

DSV4_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
DSV4_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Byte offset of (row, k) inside the block-scale "chunk" layout: one 512-byte
// chunk per (128-row tile, 128-column k tile); inside, row m of the tile and
// k-block j (32 columns) live at 16*(m%32) + 4*(m/32) + j, which is the layout
// the tensor core reads after a 32x128b.warpx4 copy into TMEM.
__host__ __device__ inline size_t sf_chunk_offset(int row, int kblk, int k_tiles) {
  const int rt = row >> 7, m = row & 127;
  const int kt = kblk >> 2, j = kblk & 3;
  return ((size_t)rt * k_tiles + kt) * 512 + (size_t)((m & 31) * 16 + (m >> 5) * 4 + j);
}

// Row layout of an expert's segment in the permuted activation buffer.  Tiles of
// tile_rows >= 128 rows are packed (a segment is its row count rounded up to
// 128); tiles of 32 or 64 rows each start on a 128-row boundary (a 128-row slot
// per tile), because the GEMM uses every tile's 128-row scale chunk unshifted.
__host__ __device__ inline int seg_rows(int count, int tile_rows) {
  return tile_rows < 128 ? (count + tile_rows - 1) / tile_rows * 128 : (count + 127) & ~127;
}
__host__ __device__ inline int seg_row(int i, int tile_rows) {   // i-th pair of the expert
  return tile_rows < 128 ? (i / tile_rows) * 128 + i % tile_rows : i;
}
__host__ __device__ inline int seg_tile_row(int r0, int tile_rows) {   // first row of the tile holding pair r0
  return tile_rows < 128 ? (r0 / tile_rows) * 128 : r0;
}
__host__ __device__ inline int seg_pairs(int rows, int tile_rows) {   // pairs a segment of `rows` rows holds
  return tile_rows < 128 ? rows / 128 * tile_rows : rows;
}

// Raises a kernel's dynamic shared-memory limit on the current device, once per
// device (the attribute is per device; `done` is the kernel's own bit mask).
template <typename Kernel>
inline cudaError_t smem_attr_once(Kernel kernel, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

}  // namespace dsv4
