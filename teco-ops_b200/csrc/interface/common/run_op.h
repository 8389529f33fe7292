// RUN_OP: find the UAL branch, then launch it on the handle's stream.
// Mirrors reference teco/interface/common/macro.h:35-42 and
// teco/interface/common/check.h:47-55 (UAL status -> tecoops status).
#ifndef TECOOPS_B200_INTERFACE_COMMON_RUN_OP_H_
#define TECOOPS_B200_INTERFACE_COMMON_RUN_OP_H_

#include "ual/com/status.h"

#define TECOOPS_RUN_OP(op_type, args, patch_args, handle)                               \
    do {                                                                                \
        op_type impl_{};                                                                \
        auto status_ = impl_.find(&(patch_args));                                       \
        if (status_ != ::tecoops::ual::common::Status::SUCCESS)                         \
            return ::tecoops::ual::common::toStatus(status_);                           \
        status_ = impl_.run(&(args), (handle)->stream);                                 \
        if (status_ != ::tecoops::ual::common::Status::SUCCESS)                         \
            return ::tecoops::ual::common::toStatus(status_);                           \
    } while (0)

#endif  // TECOOPS_B200_INTERFACE_COMMON_RUN_OP_H_
