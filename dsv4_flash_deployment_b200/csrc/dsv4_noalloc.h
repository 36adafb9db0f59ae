/* Public C interface of the allocation-free GEMM entry point.
 *
 * This entry point has no counterpart in the reference; it is an addition of
 * this library.  It is for callers that cannot allocate device memory while
 * they run: real-time serving loops in which cudaMalloc/cudaFree are forbidden
 * (both can synchronize the device and stall every stream), and embedders that
 * own a fixed, pre-sized memory budget.  Its split-K scratch is a fixed array
 * inside the library (see dsv4_gemm_mx8_noalloc below for the full contract).
 */
#ifndef DSV4_NOALLOC_H_
#define DSV4_NOALLOC_H_

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes besides 0 (success) and positive cudaError_t values. */
#define DSV4_NOALLOC_TOO_LARGE (-1) /* the split-K partials do not fit the built-in scratch */
#define DSV4_NOALLOC_BAD_ARG (-2)   /* null pointer, bad shape or alignment, bad split count */

/* Built-in scratch sizes (per device). */
#define DSV4_NOALLOC_SCRATCH_FLOATS (1 << 20) /* 4 MiB of fp32 split-K partial tiles */
#define DSV4_NOALLOC_MAX_TILES 4096           /* output tiles with a split-K counter (16 KiB) */

/* out[t][j] = sum_k a[j][k] * b[t][k] for t < n, j < m (bf16 output, fp32
 * accumulation), with MXFP8 operands: e4m3 values and ue8m0 scales per 32
 * k-elements, the scales in 512-byte chunks per (128 rows, 128 k).
 *
 *   a      e4m3 weights [m, k], m and k multiples of 128
 *   a_sf   scale chunks of a [m/128][k/128][512]
 *   b      e4m3 activations [b_rows, k], b_rows >= n and a multiple of 128
 *   b_sf   scale chunks of b [b_rows/128][k/128][512]
 *   out    bf16 [n, ldo], ldo >= m
 *   splits split-K factor, 1 <= splits <= k/128 (1: no scratch is used)
 *   err    one uint32 device word; a kernel-side failure writes a nonzero code
 *
 * Contract:
 *  - No cudaMalloc, cudaFree or allocating library call is made.
 *  - The scratch is a file-scope __device__ array that every GPU loading the
 *    library holds until the process exits.  The first call on a device (and
 *    the first call after the current context changed) looks up its device
 *    address with cudaGetSymbolAddress while that device is current; make that
 *    first call before any stream capture.  Only one context per device is
 *    supported at a time (the runtime's primary context is the usual one);
 *    after cudaDeviceReset the next call looks the address up again.
 *  - Every call on a device shares the array, which keeps the last call's
 *    contents; each call clears its tile counters before launching.  Calls
 *    that overlap on the GPU (several streams, or several host threads on one
 *    device) race on the array: serialize them.
 *  - Problems whose partials exceed DSV4_NOALLOC_SCRATCH_FLOATS floats or
 *    DSV4_NOALLOC_MAX_TILES tiles return DSV4_NOALLOC_TOO_LARGE without
 *    launching anything (out and err untouched).
 */
int dsv4_gemm_mx8_noalloc(const void* a, const void* a_sf, const void* b, const void* b_sf, void* out, int m, int n,
                          int k, int b_rows, int ldo, int splits, void* err, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DSV4_NOALLOC_H_ */
