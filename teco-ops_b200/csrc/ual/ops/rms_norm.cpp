// Branch selection and launch bridge of the rms_norm UAL operator
// (reference teco/ual/ops/rms_norm/find_rms_norm.cpp).
#include "ual/ops/rms_norm.hpp"

#include "ual/kernels/launchers.h"

namespace tecoops {
namespace ual {
namespace ops {

static cudaError_t runRmsNorm(const args::RmsNormArgs &a, cudaStream_t stream) {
    return kern::launch_rms_norm(a, stream);
}

Status RmsNormOp::findImpl(const args::RmsNormArgs *a) {
    if (a == nullptr) return Status::BAD_PARAMETER;
    setInstance(&runRmsNorm, a->residual ? "rms_norm_add_sm100" : "rms_norm_sm100");
    return Status::SUCCESS;
}

}  // namespace ops
}  // namespace ual
}  // namespace tecoops
