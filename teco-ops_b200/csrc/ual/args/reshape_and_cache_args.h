// Argument block of the reshape_and_cache kernel launcher.
// Mirrors reference teco/ual/args/reshape_and_cache_args.h:43-59, with 64-bit
// element strides (the reference's 32-bit byte strides overflow for caches
// beyond 2 GiB) and the element size carried explicitly.
#ifndef TECOOPS_B200_UAL_ARGS_RESHAPE_AND_CACHE_ARGS_H_
#define TECOOPS_B200_UAL_ARGS_RESHAPE_AND_CACHE_ARGS_H_

#include <cstdint>

namespace tecoops {
namespace ual {
namespace args {

struct ReshapeAndCacheArgs {
    int num_tokens;
    int num_kv_heads;
    int size_per_head;   // head_size (elements)
    int num_blocks;
    int block_size;
    int elem_bytes;      // 2 (fp16 / bf16) for key/value and (unless cache_fp8) the caches
    // cache_fp8: 0 = bit copy; 1 = e4m3(fp16 / scale); 2 = e4m3(bf16 / scale)
    int cache_fp8;
    float k_scale;
    float v_scale;
    // cache strides in cache elements (layout [NB, H, bs, D] or [NB, bs, H, D])
    int64_t block_stride;   // num_kv_heads * block_size * head_size
    int64_t head_stride;    // block_size * head_size   (D for [NB, bs, H, D])
    int64_t entry_stride;   // head_size                (H * D for [NB, bs, H, D])
    int64_t key_stride;     // num_kv_heads * head_size (token stride of key)
    int64_t value_stride;   // token stride of value
    const void *key;
    const void *value;
    const int64_t *slot_mapping;
    void *key_cache;
    void *value_cache;
};

}  // namespace args
}  // namespace ual
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_ARGS_RESHAPE_AND_CACHE_ARGS_H_
