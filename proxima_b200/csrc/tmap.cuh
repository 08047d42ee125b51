// tmap.cuh — host-side construction of TMA tensor maps.
//
// cuTensorMapEncodeTiled is a driver API; it is fetched through the runtime's
// driver entry point so the library needs no link-time dependency on libcuda.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace pxc {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess) p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  if (!fn) throw make_failure(PXC_DEVICE, 0, 0, nullptr, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// Row-major u8 matrix [rows][cols] (cols = row pitch in bytes, a multiple of
// 16), loaded in boxes of box_cols bytes x box_rows rows with the 128-byte
// swizzle the tcgen05 K-major descriptors expect.
inline void make_tmap_u8_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                            uint32_t box_cols, uint32_t box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (cols & 15) != 0)
    throw make_failure(PXC_INTERNAL, cols, 0, nullptr, "TMA operand is not 16-byte aligned");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode_tiled_fn()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base),
                                 dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw make_failure(PXC_DEVICE, (uint64_t)r, 0, nullptr, "cuTensorMapEncodeTiled failed (%d)", (int)r);
}

// Row-major f32 matrix with `cols` valid columns and a row pitch of `pitch`
// floats (a multiple of 4), loaded in boxes of box_cols floats (32 = 128 bytes)
// x box_rows rows with the 128-byte swizzle. Columns past `cols` and rows past
// `rows` read as zero.
inline void make_tmap_f32_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t pitch,
                             uint64_t rows, uint32_t box_cols, uint32_t box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (pitch & 3) != 0)
    throw make_failure(PXC_INTERNAL, pitch, 0, nullptr, "TMA operand is not 16-byte aligned");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode_tiled_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base),
                                 dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw make_failure(PXC_DEVICE, (uint64_t)r, 0, nullptr, "cuTensorMapEncodeTiled failed (%d)", (int)r);
}

}  // namespace pxc
