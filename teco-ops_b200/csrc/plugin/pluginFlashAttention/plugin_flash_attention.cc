// Inference plugin for paged flash attention (Teco-Inference AbstractPluginOp).
// Interface of reference teco/plugin/pluginFlashAttention/plugin_flash_attention.cc:37-149:
//   inputs  q [total, Hq, D], k_cache / v_cache [pages, Hkv, bs, D],
//           block_table int32 [batch, width], cu_seqlens_q int32 [batch + 1],
//           seqused_k int32 [batch]
//   attrs   max_seqlen_q, max_seqlen_k, max_block_num
//   output  [total, Hq, D] (the shape of q)
// Two reference bugs are fixed here:
//   * the reference passes cu_seqlens_q where tecoopsFlashAttention expects
//     per-sequence lengths; this plugin converts the offsets to lengths with a tiny
//     kernel on the engine's stream (seq_lens.cu) into a device buffer owned by the
//     plugin instance;
//   * the reference builds the block-table descriptor from an empty shape; this one
//     reads the block_table input's shape.
// Enqueue never waits for the GPU: no host copy of the offsets and no stream
// synchronisation.  The instance keeps one tecoops handle (and with it the split-KV
// scratch and error word) for all its Enqueue calls, where the reference creates and
// destroys a handle per call; the lengths buffer and the handle's scratch are
// (re)allocated only when a call needs more than any earlier one.
// The dtype of the descriptors follows the element type the engine declares through
// the "dtype" attribute (TECOOPS_DATA_HALF by default, as in the reference).
#include <plugin/register_op.h>

#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "pluginFlashAttention/seq_lens.h"
#include "tecoops.h"

namespace TECO_INFER {

struct plugin_flash_attentionAttrs : public tvm::AttrsNode<plugin_flash_attentionAttrs> {
    int64_t max_seqlen_q;
    int64_t max_seqlen_k;
    int64_t max_block_num;
    TVM_DECLARE_ATTRS(plugin_flash_attentionAttrs, "relay.attrs.plugin_flash_attentionAttrs") {
        TVM_ATTR_FIELD(max_seqlen_q).set_default(0).describe("Max Q length");
        TVM_ATTR_FIELD(max_seqlen_k).set_default(0).describe("Max K length");
        TVM_ATTR_FIELD(max_block_num).set_default(0).describe("Max number of blocks in cache");
    }
};
TVM_REGISTER_NODE_TYPE(plugin_flash_attentionAttrs);

class PluginFlashAttentionImpl : public AbstractPluginOp {
 public:
    ~PluginFlashAttentionImpl() override {
        if (handle_) tecoopsDestroy(handle_);
        if (q_lens_dev_) cudaFree(q_lens_dev_);
    }

    void InferOutputShape(const std::vector<std::vector<int>> &total_input_shape, int n_input,
                          std::vector<std::vector<int>> &total_output_shape, int n_output,
                          const OpAttr &attr) override {
        (void)n_input;
        (void)n_output;
        (void)attr;
        total_output_shape[0] = total_input_shape[0];
    }

    void Enqueue(std::shared_ptr<ComputeContext> &ctx) override {
        void *q = ctx->GetInputDataPtr("q");
        void *k_cache = ctx->GetInputDataPtr("k_cache");
        void *v_cache = ctx->GetInputDataPtr("v_cache");
        void *block_table = ctx->GetInputDataPtr("block_table");
        void *cu_seqlens_q = ctx->GetInputDataPtr("cu_seqlens_q");
        void *seqused_k = ctx->GetInputDataPtr("seqused_k");
        void *out = ctx->GetOutputDataPtr(0);
        int64_t max_seqlen_q = 0, max_seqlen_k = 0, max_block_num = 0;
        ctx->GetAttr("max_seqlen_q", max_seqlen_q);
        ctx->GetAttr("max_seqlen_k", max_seqlen_k);
        ctx->GetAttr("max_block_num", max_block_num);
        int64_t dtype = TECOOPS_DATA_HALF;
        if (ctx->attr.ints.count("dtype")) ctx->GetAttr("dtype", dtype);
        std::vector<int> q_shape, k_shape, bt_shape;
        ctx->GetInputShape("q", q_shape);
        ctx->GetInputShape("k_cache", k_shape);
        ctx->GetInputShape("block_table", bt_shape);
        if (q_shape.size() != 3 || k_shape.size() != 4 || bt_shape.size() != 2)
            throw std::runtime_error("plugin_flash_attention: input ranks");
        const int batch = bt_shape[0];
        cudaStream_t stream = ctx->GetStream();

        if (handle_ == nullptr && tecoopsCreate(&handle_) != TECOOPS_STATUS_SUCCESS) {
            handle_ = nullptr;
            throw std::runtime_error("plugin_flash_attention: tecoopsCreate failed");
        }
        tecoopsSetStream(handle_, stream);
        if (q_lens_cap_ < batch) {
            if (q_lens_dev_) cudaFree(q_lens_dev_);   // waits for the calls that used it
            q_lens_dev_ = nullptr;
            q_lens_cap_ = 0;
            if (cudaMalloc(&q_lens_dev_, sizeof(int) * batch) != cudaSuccess)
                throw std::runtime_error("plugin_flash_attention: allocation failed");
            q_lens_cap_ = batch;
        }
        // offsets -> lengths on the engine's stream, ahead of the attention kernels
        if (launchOffsetsToLengths(static_cast<const int *>(cu_seqlens_q), batch, q_lens_dev_,
                                   stream) != cudaSuccess)
            throw std::runtime_error("plugin_flash_attention: lengths kernel launch failed");

        auto make_desc = [&](tecoopsTensorDescriptor_t &d, tecoopsDataType_t dt,
                             const std::vector<int> &shape) {
            if (d == nullptr) tecoopsCreateTensorDescriptor(&d);
            tecoopsSetTensorNdDescriptor(d, dt, (int)shape.size(), shape.data(), nullptr);
        };
        const tecoopsDataType_t dt = static_cast<tecoopsDataType_t>(dtype);
        Descs &D = descs_;
        make_desc(D.bt, TECOOPS_DATA_INT32, bt_shape);
        make_desc(D.q, dt, q_shape);
        make_desc(D.k, dt, k_shape);
        make_desc(D.v, dt, k_shape);
        make_desc(D.o, dt, q_shape);
        const tecoopsStatus_t st = tecoopsFlashAttention(
            handle_, (int)max_seqlen_q, (int)max_seqlen_k, (int)max_block_num, q_lens_dev_,
            static_cast<const int *>(seqused_k), D.bt, block_table, D.q, q, D.k, k_cache, D.v,
            v_cache, D.o, out, nullptr);
        if (st != TECOOPS_STATUS_SUCCESS)
            throw std::runtime_error(std::string("plugin_flash_attention: ") +
                                     tecoopsGetErrorString(st));
    }

 private:
    struct Descs {
        tecoopsTensorDescriptor_t bt = nullptr, q = nullptr, k = nullptr, v = nullptr,
                                  o = nullptr;
        ~Descs() {
            for (tecoopsTensorDescriptor_t d : {bt, q, k, v, o})
                if (d) tecoopsDestroyTensorDescriptor(d);
        }
    };
    tecoopsHandle_t handle_ = nullptr;   // created on the device current at the first call
    int *q_lens_dev_ = nullptr;
    int q_lens_cap_ = 0;
    Descs descs_;
};

REGISTER_PLUGIN_OP_IMPL(plugin_flash_attention, PluginFlashAttentionImpl)

PLUGIN_REGISTER_OP("plugin_flash_attention")
    .Input("q")
    .Type("Tensor")
    .Desc("Query: [total_tokens, num_heads, head_size]")
    .Input("k_cache")
    .Type("Tensor")
    .Desc("K cache: [num_blocks, kv_heads, block_size, head_size]")
    .Input("v_cache")
    .Type("Tensor")
    .Desc("V cache: [num_blocks, kv_heads, block_size, head_size]")
    .Input("block_table")
    .Type("Tensor")
    .Desc("Block table: [batch_size, block_table_dim]")
    .Input("cu_seqlens_q")
    .Type("Tensor")
    .Desc("Cumulative Q seq lens: [batch_size + 1]")
    .Input("seqused_k")
    .Type("Tensor")
    .Desc("KV seq used per batch: [batch_size]")
    .AttrType<plugin_flash_attentionAttrs>()
    .Register();

}  // namespace TECO_INFER
