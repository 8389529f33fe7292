// Inference plugins plugin_rms_norm (input, weight -> output) and
// plugin_rms_norm_add (input, weight, residual -> output, residual_out), attribute
// eps.  Follows reference teco/plugin/pluginRmsNorm/plugin_rms_norm.cc: the output
// shapes are the input's; Enqueue runs tecoopsRmsNorm on the engine's stream
// (inputs by position, as the reference plugin reads them).
#include <plugin/register_op.h>

#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "tecoops.h"

namespace TECO_INFER {

struct plugin_rms_normAttrs : public tvm::AttrsNode<plugin_rms_normAttrs> {
    double eps;
    TVM_DECLARE_ATTRS(plugin_rms_normAttrs, "relay.attrs.plugin_rms_normAttrs") {
        TVM_ATTR_FIELD(eps).set_default(1e-5).describe("Epsilon for numerical stability");
    }
};
TVM_REGISTER_NODE_TYPE(plugin_rms_normAttrs);

struct plugin_rms_norm_addAttrs : public tvm::AttrsNode<plugin_rms_norm_addAttrs> {
    double eps;
    TVM_DECLARE_ATTRS(plugin_rms_norm_addAttrs, "relay.attrs.plugin_rms_norm_addAttrs") {
        TVM_ATTR_FIELD(eps).set_default(1e-5).describe("Epsilon for numerical stability");
    }
};
TVM_REGISTER_NODE_TYPE(plugin_rms_norm_addAttrs);

namespace {
// run tecoopsRmsNorm with a handle bound to the engine's stream
void run_rms_norm(std::shared_ptr<ComputeContext> &ctx, bool add) {
    std::vector<int> shape;
    ctx->GetInputShape(0, shape);
    if (shape.size() != 2) throw std::runtime_error("rms_norm: input must be [tokens, hidden]");
    float eps = 1e-5f;
    ctx->GetAttr("eps", eps);
    tecoopsHandle_t handle = nullptr;
    if (tecoopsCreate(&handle) != TECOOPS_STATUS_SUCCESS)
        throw std::runtime_error("tecoopsCreate failed");
    tecoopsSetStream(handle, ctx->GetStream());
    const tecoopsStatus_t st = tecoopsRmsNorm(
        handle, ctx->GetInputDataPtr(0), ctx->GetInputDataPtr(1),
        add ? ctx->GetInputDataPtr(2) : nullptr, ctx->GetOutputDataPtr(0),
        add ? ctx->GetOutputDataPtr(1) : nullptr, shape[0], shape[1], eps);
    tecoopsDestroy(handle);
    if (st != TECOOPS_STATUS_SUCCESS)
        throw std::runtime_error(std::string("tecoopsRmsNorm: ") + tecoopsGetErrorString(st));
}
}  // namespace

class PluginRmsNormImpl : public AbstractPluginOp {
 public:
    void InferOutputShape(const std::vector<std::vector<int>> &total_input_shape, int n_input,
                          std::vector<std::vector<int>> &total_output_shape, int n_output,
                          const OpAttr &attr) override {
        (void)n_input;
        (void)n_output;
        (void)attr;
        total_output_shape[0] = total_input_shape[0];
    }
    void Enqueue(std::shared_ptr<ComputeContext> &ctx) override { run_rms_norm(ctx, false); }
};
REGISTER_PLUGIN_OP_IMPL(plugin_rms_norm, PluginRmsNormImpl)

PLUGIN_REGISTER_OP("plugin_rms_norm")
    .Input("input")
    .Type("Tensor")
    .Desc("Input tensor [num_tokens, hidden_size]")
    .Input("weight")
    .Type("Tensor")
    .Desc("Weight tensor [hidden_size]")
    .AttrType<plugin_rms_normAttrs>()
    .Register();

class PluginRmsNormAddImpl : public AbstractPluginOp {
 public:
    void InferOutputShape(const std::vector<std::vector<int>> &total_input_shape, int n_input,
                          std::vector<std::vector<int>> &total_output_shape, int n_output,
                          const OpAttr &attr) override {
        (void)n_input;
        (void)attr;
        total_output_shape[0] = total_input_shape[0];
        if (n_output > 1) total_output_shape[1] = total_input_shape[0];
    }
    void Enqueue(std::shared_ptr<ComputeContext> &ctx) override { run_rms_norm(ctx, true); }
};
REGISTER_PLUGIN_OP_IMPL(plugin_rms_norm_add, PluginRmsNormAddImpl)

PLUGIN_REGISTER_OP("plugin_rms_norm_add")
    .Input("input")
    .Type("Tensor")
    .Desc("Input tensor [num_tokens, hidden_size]")
    .Input("weight")
    .Type("Tensor")
    .Desc("Weight tensor [hidden_size]")
    .Input("residual")
    .Type("Tensor")
    .Desc("Residual tensor [num_tokens, hidden_size]")
    .AttrType<plugin_rms_norm_addAttrs>()
    .Register();

}  // namespace TECO_INFER
