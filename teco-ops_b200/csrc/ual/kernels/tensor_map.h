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

// 4-D map over a cache [pages, Hkv, block_size, D] of 2-byte elements with a box
// of {64 columns, box_rows rows, 1 head, 1 page} and 128-byte swizzle.  Page ids are
// TMA coordinates, so an out-of-range page reads as zeros.
inline bool encode_cache_map(CUtensorMap *map, const void *base, bool bf16, int head_dim,
                             int block_size, int kv_heads, int pages, int box_rows) {
    PFN_encodeTiled enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[4] = {(cuuint64_t)head_dim, (cuuint64_t)block_size, (cuuint64_t)kv_heads,
                          (cuuint64_t)pages};
    cuuint64_t strides[3] = {(cuuint64_t)head_dim * 2, (cuuint64_t)block_size * head_dim * 2,
                             (cuuint64_t)kv_heads * block_size * head_dim * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
               const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace kern
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_KERNELS_TENSOR_MAP_H_
