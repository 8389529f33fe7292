// Argument block of the rms_norm kernel launcher.
// Mirrors reference teco/ual/args/rms_norm_args.h (RmsNormArgs): input / weight /
// optional residual, output / residual_out, num_tokens x hidden_size, eps.  The
// core count becomes the SM count and the element type (fp16 or bf16) is carried.
#ifndef TECOOPS_B200_UAL_ARGS_RMS_NORM_ARGS_H_
#define TECOOPS_B200_UAL_ARGS_RMS_NORM_ARGS_H_

#include <cstdint>

#include "ual/args/flash_attention_args.h"

namespace tecoops {
namespace ual {
namespace args {

struct RmsNormArgs {
    int num_sms;
    const void *input;      // [num_tokens, stride]
    const void *weight;     // [hidden_size]
    const void *residual;   // [num_tokens, hidden_size] or null
    void *output;           // [num_tokens, hidden_size]
    void *residual_out;     // [num_tokens, hidden_size] (with residual)
    int num_tokens;
    int hidden_size;
    int stride;             // row stride of input (elements, >= hidden_size)
    float eps;
    ElemType dtype;
};

}  // namespace args
}  // namespace ual
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_ARGS_RMS_NORM_ARGS_H_
