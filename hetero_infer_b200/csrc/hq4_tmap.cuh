// Host-side tensor-map encoding shared by the GEMV and GEMM launchers.
// cuTensorMapEncodeTiled is reached through the runtime's driver entry point,
// so the library needs no link against libcuda.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace hq4 {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The encoder, looked up once (thread-safe static initialisation); null if
// the driver does not provide it.
static inline EncodeTiledFn encode_fn() {
    static const EncodeTiledFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn>(f);
        return (EncodeTiledFn) nullptr;
    }();
    return fn;
}

// rows x cols row-major matrix of `elem`-byte elements as a 2D map with box
// (box_cols x box_rows) and the given shared-memory swizzle (box_cols * elem
// no wider than the swizzle span).  Out-of-range box elements read as zero.
static inline bool make_map_2d_sw(CUtensorMap* tm, const void* ptr, CUtensorMapDataType dt, int elem, long long rows,
                                  long long cols, int box_cols, int box_rows, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * elem)};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(tm, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// The same with the 128-byte swizzle or none.
static inline bool make_map_2d(CUtensorMap* tm, const void* ptr, CUtensorMapDataType dt, int elem, long long rows,
                               long long cols, int box_cols, int box_rows, bool swizzle128) {
    return make_map_2d_sw(tm, ptr, dt, elem, rows, cols, box_cols, box_rows,
                          swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

// A packed-weight matrix [rows][cols words] seen as 3D (word in chunk,
// row, chunk) with chunks of 32 words (128 B): box (32 words x box_rows rows
// x box_chunks chunks) lands in shared memory as [chunk][row][128 B] with the
// 128-byte swizzle, so one copy brings box_chunks k-chunks of box_rows rows.
static inline bool make_map_chunks(CUtensorMap* tm, const void* ptr, long long rows, long long cols_words,
                                   int box_rows, int box_chunks) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || cols_words % 32) return false;
    cuuint64_t dims[3] = {32, (cuuint64_t)rows, (cuuint64_t)(cols_words / 32)};
    cuuint64_t strides[2] = {(cuuint64_t)(cols_words * 4), 128};
    cuuint32_t box[3] = {32, (cuuint32_t)box_rows, (cuuint32_t)box_chunks};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Swizzle of a scale/bias tile whose rows are sg_cols fp16 values (128, 64 or
// 32 bytes): the 16 rows' reads of one column then fall in different banks.
static inline CUtensorMapSwizzle sb_swizzle(int sg_cols) {
    return sg_cols * 2 >= 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                              : sg_cols * 2 == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
}

}  // namespace hq4
