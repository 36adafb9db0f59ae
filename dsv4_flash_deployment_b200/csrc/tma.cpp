// Tensor-map construction for the TMA loads of the GEMM kernels.  The driver
// entry point is fetched through the runtime so the library needs no link-time
// dependency on libcuda.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "gemm.h"

namespace dsv4 {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

bool make_tma_2d(CUtensorMap* map, const void* base, int elem, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeFn enc = get_encode();
  if (!enc) return false;
  CUtensorMapDataType dt;
  cuuint64_t row_bytes;
  cuuint32_t box_k;
  switch (elem) {
    case TMA_U8:
      dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
      row_bytes = cols;
      box_k = 128;
      break;
    case TMA_BF16:
      dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
      row_bytes = cols * 2;
      box_k = 64;
      break;
    case TMA_E2M1:
      dt = CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B;  // each 16 e2m1 values land in 16 smem bytes (unpacked)
      row_bytes = cols / 2;
      box_k = 128;
      break;
    default:
      return false;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_k, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace dsv4
