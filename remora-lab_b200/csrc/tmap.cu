// tmap.cu — host-side encoding of the TMA tensor maps the tensor-core path
// loads through.  cuTensorMapEncodeTiled is a driver API entry point; it is
// looked up once with cudaGetDriverEntryPoint so the library needs no link
// dependency on libcuda beyond what the runtime already loads.
#include <cuda.h>

#include <mutex>

#include "moe_tc.cuh"

namespace har {

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
    cudaGetLastError();
  });
  return fn;
}

// 2-D map over a row-major [rows][cols] array of `elem_bytes`-byte elements
// (cols contiguous, rows `row_stride` bytes apart); box = [box_rows][box_cols].
int32_t encode_tmap_2d(har_cuda_ctx *ctx, TmaDesc *out, const void *base, int elem_bytes,
                       uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_rows,
                       uint32_t box_cols, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(ctx, HAR_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  if (((uintptr_t)base & 15u) || (row_stride & 15u))
    return set_error(ctx, HAR_CUDA_ERR_ARG, "tensor map: base and row stride must be 16-byte aligned");
  const CUtensorMapDataType dt =
      elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap *m = reinterpret_cast<CUtensorMap *>(out->bytes);
  const CUresult r = fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ctx, HAR_CUDA_ERR_CUDA,
                     "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
  return HAR_CUDA_OK;
}

}  // namespace har
