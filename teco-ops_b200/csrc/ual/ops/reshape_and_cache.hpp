// reshape_and_cache UAL operator.
// Mirrors reference teco/ual/ops/reshape_and_cache/reshape_and_cache.hpp:42-78 and
// find_reshape_and_cache.cpp:35-37 (a single branch).
#ifndef TECOOPS_B200_UAL_OPS_RESHAPE_AND_CACHE_HPP_
#define TECOOPS_B200_UAL_OPS_RESHAPE_AND_CACHE_HPP_

#include "ual/args/reshape_and_cache_args.h"
#include "ual/ops/base_op.hpp"

namespace tecoops {
namespace ual {
namespace ops {

struct ReshapeAndCacheLaunch {
    args::ReshapeAndCacheArgs args;
    int num_sms;
};

struct ReshapeAndCacheTraits {
    using ArgsType = ReshapeAndCacheLaunch;
    using PatchType = ReshapeAndCacheLaunch;
    using PImplType = cudaError_t (*)(const ReshapeAndCacheLaunch &, cudaStream_t);
};

enum class ReshapeAndCacheAlgos { VEC16_SCATTER = 0 };

struct ReshapeAndCacheOp : BaseOp<ReshapeAndCacheOp, ReshapeAndCacheTraits> {
    Status findImpl(const ReshapeAndCacheLaunch *a);
};

}  // namespace ops
}  // namespace ual
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_OPS_RESHAPE_AND_CACHE_HPP_
