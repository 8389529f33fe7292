// Inference plugin for reshape_and_cache (Teco-Inference AbstractPluginOp).
// Interface and behaviour of reference teco/plugin/pluginReshapeAndCache/
// plugin_reshape_and_cache.cc:37-131:
//   inputs  key [T, H, D], value [T, H, D], slot_mapping int64 [T]
//   attrs   num_blocks, block_size
//   output  one tensor [2 * num_blocks, H, block_size, D]: the key cache followed by
//           the value cache; it is zero-filled, then the tokens are scattered into it.
// The handle is created on the engine's stream for each Enqueue, as in the reference.
#include <plugin/register_op.h>

#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "tecoops.h"

namespace TECO_INFER {

struct plugin_reshape_and_cacheAttrs : public tvm::AttrsNode<plugin_reshape_and_cacheAttrs> {
    int64_t num_blocks;
    int64_t block_size;
    TVM_DECLARE_ATTRS(plugin_reshape_and_cacheAttrs, "relay.attrs.plugin_reshape_and_cacheAttrs") {
        TVM_ATTR_FIELD(num_blocks).set_default(0).describe("Number of KV cache blocks");
        TVM_ATTR_FIELD(block_size).set_default(0).describe("Block size (tokens per block)");
    }
};
TVM_REGISTER_NODE_TYPE(plugin_reshape_and_cacheAttrs);

class PluginReshapeAndCacheImpl : public AbstractPluginOp {
 public:
    void InferOutputShape(const std::vector<std::vector<int>> &total_input_shape, int n_input,
                          std::vector<std::vector<int>> &total_output_shape, int n_output,
                          const OpAttr &attr) override {
        (void)n_input;
        (void)n_output;
        const int num_kv_heads = total_input_shape[0][1];
        const int head_size = total_input_shape[0][2];
        const int64_t num_blocks = attr.GetAttr<int64_t>("num_blocks");
        const int64_t block_size = attr.GetAttr<int64_t>("block_size");
        total_output_shape[0] = {static_cast<int>(num_blocks * 2), num_kv_heads,
                                 static_cast<int>(block_size), head_size};
    }

    void Enqueue(std::shared_ptr<ComputeContext> &ctx) override {
        void *key = ctx->GetInputDataPtr("key");
        void *value = ctx->GetInputDataPtr("value");
        void *slot_mapping = ctx->GetInputDataPtr("slot_mapping");
        int64_t num_blocks = 0, block_size = 0;
        ctx->GetAttr("num_blocks", num_blocks);
        ctx->GetAttr("block_size", block_size);
        std::vector<int> key_shape;
        ctx->GetInputShape("key", key_shape);
        if (key_shape.size() != 3) throw std::runtime_error("plugin_reshape_and_cache: key rank");
        const int num_tokens = key_shape[0], num_kv_heads = key_shape[1], head_size = key_shape[2];
        void *out = ctx->GetOutputDataPtr(0);
        const size_t cache_bytes = (size_t)num_blocks * block_size * num_kv_heads * head_size * 2;

        tecoopsHandle_t handle;
        tecoopsCreate(&handle);
        tecoopsSetStream(handle, ctx->GetStream());
        tecoopsStatus_t st = tecoopsMemset(handle, out, 0, cache_bytes * 2);
        if (st == TECOOPS_STATUS_SUCCESS)
            st = tecoopsReshapeAndCache(handle, key, value, static_cast<const int64_t *>(slot_mapping),
                                        out, static_cast<char *>(out) + cache_bytes, num_tokens,
                                        num_kv_heads, head_size, static_cast<int>(num_blocks),
                                        static_cast<int>(block_size));
        tecoopsDestroy(handle);
        if (st != TECOOPS_STATUS_SUCCESS)
            throw std::runtime_error(std::string("plugin_reshape_and_cache: ") +
                                     tecoopsGetErrorString(st));
    }
};

REGISTER_PLUGIN_OP_IMPL(plugin_reshape_and_cache, PluginReshapeAndCacheImpl)

PLUGIN_REGISTER_OP("plugin_reshape_and_cache")
    .Input("key")
    .Type("Tensor")
    .Desc("Key input with shape [num_tokens, num_kv_heads, head_size]")
    .Input("value")
    .Type("Tensor")
    .Desc("Value input with shape [num_tokens, num_kv_heads, head_size]")
    .Input("slot_mapping")
    .Type("Tensor")
    .Desc("Slot mapping with shape [num_tokens]")
    .AttrType<plugin_reshape_and_cacheAttrs>()
    .Register();

}  // namespace TECO_INFER
