// tecoopsReshapeAndCache: argument checks, stride derivation, RUN_OP.
// Follows reference teco/interface/ops/reshape_and_cache.cpp:39-105: null handle
// -> NOT_INITIALIZED; null key/value/slot_mapping/caches or any dim <= 0 ->
// BAD_PARAM; contiguous 2-byte elements ([T, H, D] inputs, [NB, H, bs, D]
// caches).  Strides are kept in elements as 64-bit integers so caches above
// 2 GiB address correctly.
// tecoopsReshapeAndCacheEx adds the vLLM page layout [NB, bs, H, D] (other strides)
// and e4m3 caches (quantising kernel).
#include "interface/common/context.h"
#include "interface/common/run_op.h"
#include "tecoops.h"
#include "ual/ops/reshape_and_cache.hpp"

using tecoops::ual::ops::ReshapeAndCacheLaunch;
using tecoops::ual::ops::ReshapeAndCacheOp;

static tecoopsStatus_t checkReshapeAndCacheInput(tecoopsHandle_t handle, const void *key,
                                                 const void *value, const int64_t *slot_mapping,
                                                 void *key_cache, void *value_cache,
                                                 int num_tokens, int num_kv_heads, int head_size,
                                                 int num_blocks, int block_size) {
    if (handle == nullptr) return TECOOPS_STATUS_NOT_INITIALIZED;
    if (key == nullptr || value == nullptr) return TECOOPS_STATUS_BAD_PARAM;
    if (slot_mapping == nullptr) return TECOOPS_STATUS_BAD_PARAM;
    if (key_cache == nullptr || value_cache == nullptr) return TECOOPS_STATUS_BAD_PARAM;
    if (num_kv_heads <= 0 || head_size <= 0 || num_tokens <= 0 || num_blocks <= 0 ||
        block_size <= 0)
        return TECOOPS_STATUS_BAD_PARAM;
    return TECOOPS_STATUS_SUCCESS;
}

static tecoopsStatus_t reshapeAndCacheImpl(tecoopsHandle_t handle, const void *key,
                                           const void *value, const int64_t *slot_mapping,
                                           void *key_cache, void *value_cache, int num_tokens,
                                           int num_kv_heads, int head_size, int num_blocks,
                                           int block_size, int layout, int cache_fp8,
                                           float k_scale, float v_scale) {
    const tecoopsStatus_t st =
        checkReshapeAndCacheInput(handle, key, value, slot_mapping, key_cache, value_cache,
                                  num_tokens, num_kv_heads, head_size, num_blocks, block_size);
    if (st != TECOOPS_STATUS_SUCCESS) return st;

    ReshapeAndCacheLaunch l;
    auto &a = l.args;
    a.num_tokens = num_tokens;
    a.num_kv_heads = num_kv_heads;
    a.size_per_head = head_size;
    a.num_blocks = num_blocks;
    a.block_size = block_size;
    a.elem_bytes = 2;
    a.cache_fp8 = cache_fp8;
    a.k_scale = k_scale;
    a.v_scale = v_scale;
    if (layout == TECOOPS_KV_LAYOUT_HND) {   // [NB, H, bs, D]
        a.entry_stride = head_size;
        a.head_stride = (int64_t)block_size * head_size;
    } else {                                 // [NB, bs, H, D]
        a.entry_stride = (int64_t)num_kv_heads * head_size;
        a.head_stride = head_size;
    }
    a.block_stride = (int64_t)num_kv_heads * block_size * head_size;
    a.key_stride = (int64_t)num_kv_heads * head_size;
    a.value_stride = a.key_stride;
    a.key = key;
    a.value = value;
    a.slot_mapping = slot_mapping;
    a.key_cache = key_cache;
    a.value_cache = value_cache;
    l.num_sms = handle->num_sms;

    TECOOPS_RUN_OP(ReshapeAndCacheOp, l, l, handle);
    return TECOOPS_STATUS_SUCCESS;
}

extern "C" tecoopsStatus_t tecoopsReshapeAndCache(tecoopsHandle_t handle, const void *key,
                                                  const void *value, const int64_t *slot_mapping,
                                                  void *key_cache, void *value_cache,
                                                  int num_tokens, int num_kv_heads,
                                                  int head_size, int num_blocks, int block_size) {
    return reshapeAndCacheImpl(handle, key, value, slot_mapping, key_cache, value_cache,
                               num_tokens, num_kv_heads, head_size, num_blocks, block_size,
                               TECOOPS_KV_LAYOUT_HND, 0, 1.f, 1.f);
}

extern "C" tecoopsStatus_t tecoopsReshapeAndCacheEx(
    tecoopsHandle_t handle, const void *key, const void *value, const int64_t *slot_mapping,
    void *key_cache, void *value_cache, int num_tokens, int num_kv_heads, int head_size,
    int num_blocks, int block_size, tecoopsDataType_t key_dtype,
    const tecoopsKvCacheConfig_t *cache) {
    if (handle == nullptr) return TECOOPS_STATUS_NOT_INITIALIZED;
    if (key_dtype != TECOOPS_DATA_HALF && key_dtype != TECOOPS_DATA_BFLOAT16)
        return TECOOPS_STATUS_BAD_PARAM;
    int layout = TECOOPS_KV_LAYOUT_HND, fp8 = 0;
    float ks = 1.f, vs = 1.f;
    if (cache != nullptr) {
        layout = cache->kv_layout;
        if (layout != TECOOPS_KV_LAYOUT_HND && layout != TECOOPS_KV_LAYOUT_NHD)
            return TECOOPS_STATUS_BAD_PARAM;
        if (cache->cache_dtype == TECOOPS_DATA_FLOAT8_E4M3) {
            if (!(cache->k_scale == cache->k_scale) || !(cache->v_scale == cache->v_scale))
                return TECOOPS_STATUS_BAD_PARAM;   // NaN scale
            fp8 = key_dtype == TECOOPS_DATA_BFLOAT16 ? 2 : 1;
            ks = cache->k_scale > 0.f ? cache->k_scale : 1.f;
            vs = cache->v_scale > 0.f ? cache->v_scale : 1.f;
        } else if (cache->cache_dtype != key_dtype) {
            return TECOOPS_STATUS_BAD_PARAM;
        }
    }
    return reshapeAndCacheImpl(handle, key, value, slot_mapping, key_cache, value_cache,
                               num_tokens, num_kv_heads, head_size, num_blocks, block_size,
                               layout, fp8, ks, vs);
}
