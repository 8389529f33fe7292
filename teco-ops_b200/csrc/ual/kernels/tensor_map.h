// Host helpers for TMA tensor maps over the paged K/V cache, shared by the
// prefill and decode launchers.  The driver entry point cuTensorMapEncodeTiled is
// fetched through the runtime (no link against libcuda).
#ifndef TECOOPS_B200_UAL_KERNELS_TENSOR_MAP_H_
#define TECOOPS_B200_UAL_KERNELS_TENSOR_MAP_H_

#include <cuda.h>
#include <cuda_runtime.h>

namespace tecoops {
namespace kern {

typedef CUresult (*PFN_encodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                    const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                    const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion,
                                    CUtensorMapFloatOOBfill);

inline PFN_encodeTiled get_encode_fn() {
    static PFN_encodeTiled fn = [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<PFN_encodeTiled>(ptr);
        return static_cast<PFN_encodeTiled>(nullptr);
    }();
    return fn;
}

// Cache element types of a tensor map.
enum class CacheElem { F16, BF16, E4M3 };

// 4-D map over a paged cache with coordinates (column, row in page, kv head, page):
//   layout 0: [pages, Hkv, block_size, D]   layout 1: [pages, block_size, Hkv, D]
// (the strides differ, the coordinate order does not, so kernels are layout-blind).
// Box {box_cols, box_rows, 1, 1}; 16-bit caches use 64-column boxes with 128-byte
// swizzle, e4m3 caches one box of D bytes per row, swizzled at the row width (128-byte
// swizzle for D = 128, 64-byte for D = 64, none otherwise).  Page ids are TMA
// coordinates, so an out-of-range page reads as zeros.
inline bool encode_cache_map(CUtensorMap *map, const void *base, CacheElem elem, int head_dim,
                             int block_size, int kv_heads, int pages, int box_rows,
                             int layout) {
    PFN_encodeTiled enc = get_encode_fn();
    if (!enc) return false;
    const cuuint64_t eb = elem == CacheElem::E4M3 ? 1 : 2;
    const cuuint64_t row_b = (cuuint64_t)head_dim * eb;
    cuuint64_t dims[4] = {(cuuint64_t)head_dim, (cuuint64_t)block_size, (cuuint64_t)kv_heads,
                          (cuuint64_t)pages};
    cuuint64_t strides[3];
    if (layout == 0) {
        strides[0] = row_b;                                  // row in page
        strides[1] = (cuuint64_t)block_size * row_b;         // kv head
    } else {
        strides[0] = (cuuint64_t)kv_heads * row_b;           // row in page
        strides[1] = row_b;                                  // kv head
    }
    strides[2] = (cuuint64_t)kv_heads * block_size * row_b;  // page
    const bool fp8 = elem == CacheElem::E4M3;
    cuuint32_t box[4] = {fp8 ? (cuuint32_t)head_dim : 64u, (cuuint32_t)box_rows, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    const CUtensorMapDataType dt = fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : elem == CacheElem::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    return enc(map, dt, 4, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE,
               !fp8 || head_dim == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
               : head_dim == 64        ? CU_TENSOR_MAP_SWIZZLE_64B
                                       : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace kern
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_KERNELS_TENSOR_MAP_H_
