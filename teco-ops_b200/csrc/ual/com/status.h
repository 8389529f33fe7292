// UAL status codes and their mapping to tecoopsStatus_t.
// Mirrors reference teco/ual/com/status.h:34-43 and
// teco/interface/common/convert.cpp:38-51 (NOT_IMPLEMENTED -> NOT_SUPPORTED).
#ifndef TECOOPS_B200_UAL_COM_STATUS_H_
#define TECOOPS_B200_UAL_COM_STATUS_H_

#include "tecoops.h"

namespace tecoops {
namespace ual {
namespace common {

enum class Status {
    SUCCESS = 0,
    BAD_PARAMETER = 1,
    NOT_IMPLEMENTED = 2,
    LAUNCH_FAILED = 3,
    ALLOC_FAILED = 4,
};

inline tecoopsStatus_t toStatus(Status s) {
    switch (s) {
        case Status::SUCCESS: return TECOOPS_STATUS_SUCCESS;
        case Status::BAD_PARAMETER: return TECOOPS_STATUS_BAD_PARAM;
        case Status::NOT_IMPLEMENTED: return TECOOPS_STATUS_NOT_SUPPORTED;
        case Status::ALLOC_FAILED: return TECOOPS_STATUS_ALLOC_FAILED;
        default: return TECOOPS_STATUS_INTERNAL_ERROR;
    }
}

}  // namespace common
}  // namespace ual
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_COM_STATUS_H_
