// g2v_tmap.cuh -- host-side TMA descriptor encoding through the driver entry point (no -lcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

namespace g2v {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Row-major (rows x cols) fp16 matrix with a row pitch of `pitch_elems`; box = box_cols x 1 rows,
// 128-byte swizzle (box_cols * 2 bytes must be 128).  Out-of-range rows/columns read as zero.
inline bool encode_rows_f16_sw128(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                                  int64_t pitch_elems, int box_cols) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)(rows > 0 ? rows : 1)};
    cuuint64_t strides[1] = {(cuuint64_t)pitch_elems * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, 1};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp32 grid of rows [X][Y][Z][C] (C contiguous) as a 4-D tensor {C, Z, Y, X}; box = {box_c, box_z, box_y,
// box_x}, so a box lands in shared memory as [x][y][z][box_c] rows.  swizzle_bytes 0 stores rows plainly;
// 128 (box_c * 4 == 128) stores the 16-byte chunk j of row r at chunk j ^ (r % 8); 64 (box_c * 4 == 64)
// at chunk j ^ ((r / 2) % 4).  Voxels beyond the grid and channels beyond C read as zero.  Needs
// C % 4 == 0 and a 16-byte aligned base (row strides in 16-byte units); returns false otherwise.
inline bool encode_grid_rows_f32(CUtensorMap* map, const void* base, const int dims[3], int64_t C, int box_c,
                                 int box_z, int box_y, int box_x, int swizzle_bytes = 0) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || C <= 0 || C % 4 != 0 || (reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
    cuuint64_t gdims[4] = {(cuuint64_t)C, (cuuint64_t)dims[2], (cuuint64_t)dims[1], (cuuint64_t)dims[0]};
    cuuint64_t strides[3] = {(cuuint64_t)C * 4, (cuuint64_t)C * 4 * dims[2], (cuuint64_t)C * 4 * dims[2] * dims[1]};
    cuuint32_t box[4] = {(cuuint32_t)box_c, (cuuint32_t)box_z, (cuuint32_t)box_y, (cuuint32_t)box_x};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
    if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
    else if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
    else if (swizzle_bytes != 0) return false;
    if (swizzle_bytes != 0 && box_c * 4 != swizzle_bytes) return false;
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), gdims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace g2v
