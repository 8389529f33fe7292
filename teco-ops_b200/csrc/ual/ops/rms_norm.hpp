// rms_norm UAL operator.
// Mirrors reference teco/ual/ops/rms_norm/rms_norm.hpp and find_rms_norm.cpp
// (one branch per dtype / residual mode; here the launcher picks the row mapping).
#ifndef TECOOPS_B200_UAL_OPS_RMS_NORM_HPP_
#define TECOOPS_B200_UAL_OPS_RMS_NORM_HPP_

#include "ual/args/rms_norm_args.h"
#include "ual/ops/base_op.hpp"

namespace tecoops {
namespace ual {
namespace ops {

struct RmsNormTraits {
    using ArgsType = args::RmsNormArgs;
    using PatchType = args::RmsNormArgs;
    using PImplType = cudaError_t (*)(const args::RmsNormArgs &, cudaStream_t);
};

struct RmsNormOp : BaseOp<RmsNormOp, RmsNormTraits> {
    Status findImpl(const args::RmsNormArgs *a);
};

}  // namespace ops
}  // namespace ual
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_OPS_RMS_NORM_HPP_
