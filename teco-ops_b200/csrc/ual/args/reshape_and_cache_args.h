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
    int elem_bytes;      // 2 (fp16 / bf16)
    // strides in elements
    int64_t block_stride;   // num_kv_heads * block_size * head_size
    int64_t head_stride;    // block_size * head_size
    int64_t entry_stride;   // head_size
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
