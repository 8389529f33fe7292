// Branch selection and launch bridge of the reshape_and_cache UAL operator
// (reference teco/ual/ops/reshape_and_cache/find_reshape_and_cache.cpp:35-37).
#include "ual/ops/reshape_and_cache.hpp"

#include "ual/kernels/launchers.h"

namespace tecoops {
namespace ual {
namespace ops {

static cudaError_t runReshapeAndCache(const ReshapeAndCacheLaunch &a, cudaStream_t stream) {
    return kern::launch_reshape_and_cache(a.args, a.num_sms, stream);
}

Status ReshapeAndCacheOp::findImpl(const ReshapeAndCacheLaunch *a) {
    if (a == nullptr || a->args.elem_bytes != 2) return Status::NOT_IMPLEMENTED;
    setInstance(&runReshapeAndCache, "reshape_and_cache_vec16_sm100");
    return Status::SUCCESS;
}

}  // namespace ops
}  // namespace ual
}  // namespace tecoops
