// Host side of TMA tensor copies: a 2D tensor map over f16 data, encoded through the driver's
// cuTensorMapEncodeTiled (resolved once through the runtime, so the library needs no link against libcuda).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace neko {

// A [rows] x [cols] f16 matrix (row stride row_stride_bytes) read in boxes of box_rows x box_cols elements with
// the 128-byte swizzle (box_cols * 2 <= 128); elements past the matrix read as zeros. False when the driver entry
// point is unavailable or the map is invalid (alignment, strides).
inline bool encode_f16_2d_sw128(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                                uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows) {
    using Fn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                            const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                            CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static const Fn fn = []() -> Fn {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<Fn>(p);
    }();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || row_stride_bytes % 16 || box_cols * 2 > 128) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1u, 1u};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A [rows] x [cols] byte matrix (row stride row_stride_bytes) read in boxes of box_cols x box_rows bytes (packed
// weight rows: codes, then scales), optionally with the 128-byte swizzle (box_cols <= 128: 16-byte chunk c of box
// row r lands at chunk c ^ (r % 8)); bytes past the matrix read as zeros. box_cols a multiple of 16.
inline bool encode_u8_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t row_stride_bytes,
                         uint32_t box_cols, uint32_t box_rows, bool swizzle128 = false) {
    using Fn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                            const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                            CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static const Fn fn = []() -> Fn {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<Fn>(p);
    }();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || row_stride_bytes % 16 || box_cols % 16 || box_cols > 256 ||
        box_rows > 256 || (swizzle128 && box_cols > 128))
        return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1u, 1u};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace neko
