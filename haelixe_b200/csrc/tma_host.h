// Host-side creation of TMA tensor maps through the driver entry point
// (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hx {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    if (fn == nullptr) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

// 16-bit (bf16, or f16 with `type`) tensor viewed as [B, H, S, D] (D
// contiguous; strides in elements), box = (box_d, box_rows, 1, 1), 128-byte
// swizzle; rows beyond S read as 0.
inline bool make_tmap_bhsd(CUtensorMap* map, const void* base, int B, int H, int S, int D,
                           int64_t sb, int64_t sh, int64_t ss, int box_d, int box_rows,
                           CUtensorMapDataType type = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (fn == nullptr) return false;
    // A dimension of extent 1 never advances, so any legal stride will do.
    const int64_t row_bytes = ss * 2;
    const int64_t head_bytes = (H == 1) ? row_bytes * S : sh * 2;
    const int64_t batch_bytes = (B == 1) ? head_bytes * H : sb * 2;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)row_bytes, (cuuint64_t)head_bytes,
                             (cuuint64_t)batch_bytes};
    cuuint32_t box[4] = {(cuuint32_t)box_d, (cuuint32_t)box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, type, 4, const_cast<void*>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// f32 tensor [n2][n1][n0] (n0 contiguous), box (b0, b1, 1), optional 128B swizzle.
inline bool make_tmap_f32_3d(CUtensorMap* map, const void* base, uint64_t n0, uint64_t n1,
                             uint64_t n2, int b0, int b1, bool swizzle128) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (fn == nullptr) return false;
    cuuint64_t dims[3] = {n0, n1, n2};
    cuuint64_t strides[2] = {n0 * 4, n0 * n1 * 4};
    cuuint32_t box[3] = {(cuuint32_t)b0, (cuuint32_t)b1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Plain row-major bf16 matrix [rows][cols], box (box_cols, box_rows), 128B swizzle.
inline bool make_tmap_2d(CUtensorMap* map, const void* base, int rows, int cols, int box_cols,
                         int box_rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (fn == nullptr) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// bf16 matrix [rows][cols] with a leading dimension of `ld` elements (ld >=
// cols, ld * 2 a multiple of 16), box (box_cols, box_rows), 128B swizzle;
// reads outside the matrix return 0.
inline bool make_tmap_2d_ld(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                            int box_cols, int box_rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (fn == nullptr) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace hx
