// Host-side creation of TMA tensor maps (cuTensorMapEncodeTiled through the runtime's
// driver entry point, so the extension does not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <c10/util/Exception.h>

namespace mykb {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres);
    TORCH_CHECK(err == cudaSuccess && qres == cudaDriverEntryPointSuccess && ptr != nullptr,
                "cuTensorMapEncodeTiled is not available");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 3-D tiled map with 128-byte swizzle.  dim0 is the contiguous dimension; strides are in
// elements.  A batch of 1 gets a packed batch stride.
inline CUtensorMap make_tmap_3d(void* base, CUtensorMapDataType dtype, int elem_bytes, int64_t dim0, int64_t dim1,
                                int64_t dim2, int64_t stride1, int64_t stride2, int box0, int box1,
                                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap map;
  if (dim2 <= 1 || stride2 == 0) stride2 = stride1 * dim1;
  cuuint64_t dims[3] = {(cuuint64_t)dim0, (cuuint64_t)dim1, (cuuint64_t)(dim2 < 1 ? 1 : dim2)};
  cuuint64_t strides[2] = {(cuuint64_t)(stride1 * elem_bytes), (cuuint64_t)(stride2 * elem_bytes)};
  cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK((stride1 * elem_bytes) % 16 == 0 && (stride2 * elem_bytes) % 16 == 0,
              "TMA strides must be multiples of 16 bytes (row stride ", stride1, " elements)");
  CUresult r = encode_tiled_fn()(&map, dtype, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", (int)r, ")");
  return map;
}

}  // namespace mykb
