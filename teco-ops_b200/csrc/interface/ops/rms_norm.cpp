// tecoopsRmsNorm (+ the bf16 extension tecoopsRmsNormEx): argument checks, RUN_OP.
// Follows reference teco/interface/ops/rms_norm.cpp: null handle ->
// NOT_INITIALIZED; null input / weight / output, residual without residual_out,
// num_tokens or hidden_size <= 0 -> BAD_PARAM; contiguous rows (stride =
// hidden_size); fp16 (the reference's only type).
#include "interface/common/context.h"
#include "interface/common/run_op.h"
#include "tecoops.h"
#include "ual/ops/rms_norm.hpp"

using tecoops::ual::args::ElemType;
using tecoops::ual::args::RmsNormArgs;
using tecoops::ual::ops::RmsNormOp;

static tecoopsStatus_t rmsNormImpl(tecoopsHandle_t handle, const void *input, const void *weight,
                                   const void *residual, void *output, void *residual_out,
                                   int num_tokens, int hidden_size, float eps,
                                   tecoopsDataType_t dtype) {
    if (handle == nullptr) return TECOOPS_STATUS_NOT_INITIALIZED;
    if (input == nullptr || weight == nullptr || output == nullptr)
        return TECOOPS_STATUS_BAD_PARAM;
    if (residual != nullptr && residual_out == nullptr) return TECOOPS_STATUS_BAD_PARAM;
    if (num_tokens <= 0 || hidden_size <= 0) return TECOOPS_STATUS_BAD_PARAM;
    if (dtype != TECOOPS_DATA_HALF && dtype != TECOOPS_DATA_BFLOAT16)
        return TECOOPS_STATUS_BAD_PARAM;

    RmsNormArgs a;
    a.num_sms = handle->num_sms;
    a.input = input;
    a.weight = weight;
    a.residual = residual;
    a.output = output;
    a.residual_out = residual != nullptr ? residual_out : nullptr;
    a.num_tokens = num_tokens;
    a.hidden_size = hidden_size;
    a.stride = hidden_size;
    a.eps = eps;
    a.dtype = dtype == TECOOPS_DATA_BFLOAT16 ? ElemType::BF16 : ElemType::F16;
    TECOOPS_RUN_OP(RmsNormOp, a, a, handle);
    return TECOOPS_STATUS_SUCCESS;
}

extern "C" tecoopsStatus_t tecoopsRmsNorm(tecoopsHandle_t handle, const void *input,
                                          const void *weight, const void *residual, void *output,
                                          void *residual_out, int num_tokens, int hidden_size,
                                          float eps) {
    return rmsNormImpl(handle, input, weight, residual, output, residual_out, num_tokens,
                       hidden_size, eps, TECOOPS_DATA_HALF);
}

extern "C" tecoopsStatus_t tecoopsRmsNormEx(tecoopsHandle_t handle, const void *input,
                                            const void *weight, const void *residual,
                                            void *output, void *residual_out, int num_tokens,
                                            int hidden_size, float eps, tecoopsDataType_t dtype) {
    return rmsNormImpl(handle, input, weight, residual, output, residual_out, num_tokens,
                       hidden_size, eps, dtype);
}
