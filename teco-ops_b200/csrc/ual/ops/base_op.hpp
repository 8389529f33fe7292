// UAL operator base: branch selection (`find`) then launch (`run`).
// Mirrors reference teco/ual/ops/base_op.hpp:47-84 (BaseOp<T, Ty> CRTP with
// find/run and a kernel instance pointer) and the RUN_KERNEL macro (41-45).
// On CUDA a "kernel instance" is a host launcher (it needs grid/smem decisions),
// and run() reports launch errors instead of ignoring them.  Every launch sits in an
// NVTX range named after the selected branch (header-only NVTX: a no-op unless a
// profiler is attached), so nsys / ncu timelines show which branch ran.
#ifndef TECOOPS_B200_UAL_OPS_BASE_OP_HPP_
#define TECOOPS_B200_UAL_OPS_BASE_OP_HPP_

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include "ual/com/log.h"
#include "ual/com/status.h"

namespace tecoops {
namespace ual {
namespace ops {

using common::Status;

template <typename T, typename Ty>
struct BaseOp {
    using ArgsType = typename Ty::ArgsType;
    using PatchType = typename Ty::PatchType;
    using PImplType = typename Ty::PImplType;   // cudaError_t (*)(const ArgsType &, cudaStream_t)

    BaseOp() = default;
    BaseOp(const BaseOp &) = delete;
    BaseOp &operator=(const BaseOp &) = delete;

    Status find(const PatchType *args) { return static_cast<T *>(this)->findImpl(args); }

    Status run(const ArgsType *arg, cudaStream_t stream) {
        if (instance_ == nullptr || description_ == nullptr) {
            TECO_ERROR("no kernel selected for this operator");
            return Status::BAD_PARAMETER;
        }
        nvtxRangePushA(description_);
        const cudaError_t e = instance_(*arg, stream);
        nvtxRangePop();
        if (e != cudaSuccess) {
            TECO_ERROR("%s: launch failed: %s", description_, cudaGetErrorString(e));
            return Status::LAUNCH_FAILED;
        }
        return Status::SUCCESS;
    }

    void setInstance(PImplType instance, const char *description) {
        instance_ = instance;
        description_ = description;
    }
    const char *description() const { return description_; }

 private:
    PImplType instance_ = nullptr;
    const char *description_ = nullptr;
};

}  // namespace ops
}  // namespace ual
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_OPS_BASE_OP_HPP_
