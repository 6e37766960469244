// iw_tmap.cuh -- host-side creation of TMA tensor maps for int8 matrices.
//
// cuTensorMapEncodeTiled is fetched through cudaGetDriverEntryPoint so the
// library needs no link-time dependency on libcuda.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace iw {

typedef CUresult (*PFN_iwEncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                       const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                       CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                       CUtensorMapFloatOOBfill);

inline PFN_iwEncodeTiled encode_tiled_fn() {
    static PFN_iwEncodeTiled fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_iwEncodeTiled>(p);
    }
    return fn;
}

// 2-D uint8 tensor [rows, cols] with row stride `ld` bytes; box
// [box_rows, box_cols] with 128-byte swizzle (box_cols must be <= 128).
// Out-of-bounds elements of a box read as zero.
inline cudaError_t make_tmap_2d_u8(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint64_t ld,
                                   uint32_t box_cols, uint32_t box_rows,
                                   CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
    PFN_iwEncodeTiled fn = encode_tiled_fn();
    if (!fn) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld & 15)) return cudaErrorMisalignedAddress;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// 3-D uint8 tensor: `count` windows of `rows` rows of `cols` bytes; row r of
// window w starts at base + w*win_stride + r*ld. The row stride may be
// smaller than a row (overlapping rows). Box [1, box_rows, box_cols], 128-byte
// swizzle; out-of-bounds elements read as zero.
inline cudaError_t make_tmap_3d_windows_u8(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                                           uint64_t count, uint64_t ld, uint64_t win_stride, uint32_t box_cols,
                                           uint32_t box_rows) {
    PFN_iwEncodeTiled fn = encode_tiled_fn();
    if (!fn) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld & 15) || (win_stride & 15)) return cudaErrorMisalignedAddress;
    cuuint64_t dims[3] = {cols, rows, count};
    cuuint64_t strides[2] = {ld, win_stride};
    cuuint32_t box[3] = {box_cols, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace iw
