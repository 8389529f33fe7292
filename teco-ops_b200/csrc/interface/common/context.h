// Internal definitions of the opaque handle and tensor-descriptor types of
// tecoops.h.  Mirrors reference teco/interface/include/builtin_type.h:33-38
// (struct tecoopsContext) and teco/interface/common/tensor.h:38-93
// (struct tecoopsTensorStruct), re-designed for CUDA: the handle carries the
// CUDA stream, the device it was created on, that device's SM count, and the
// lazily grown device scratch used by split-KV decode and the prefill tile
// scheduler.
#ifndef TECOOPS_B200_INTERFACE_COMMON_CONTEXT_H_
#define TECOOPS_B200_INTERFACE_COMMON_CONTEXT_H_

#include <cuda_runtime.h>

#include <cstddef>

#include "tecoops.h"

struct tecoopsContext {
    cudaStream_t stream = nullptr;
    int device = 0;
    int num_sms = 148;
    // handle-owned scratch (grown on demand, freed by tecoopsDestroy)
    void *scratch = nullptr;
    size_t scratch_bytes = 0;
    // four ints of device memory: [0] error word that kernels set when a bounded wait
    // gives up; [1], [2] the prefill kernel's work-unit and finished-CTA counters (zero
    // between launches: the last CTA of each launch resets them)
    int *dev_error = nullptr;
    // limit of every bounded device wait of the split-KV decode kernel, and the test
    // switch that makes its first ring wait wait on a barrier nothing completes
    // (tecoopsSetDeviceWaitLimit)
    unsigned long long wait_limit_ns = 2000000000ull;
    int stall_test = 0;
};

struct tecoopsTensorStruct {
    tecoopsTensorFormat_t format = TECOOPS_TENSOR_NHWC;
    tecoopsDataType_t dataType = TECOOPS_DATA_FLOAT;
    int nbDims = 0;
    int dimA[TECOOPS_DIM_MAX] = {0};
    int strideA[TECOOPS_DIM_MAX] = {0};
};

namespace tecoops {
namespace interface {

// Grow the handle's scratch to at least `bytes` (cudaMalloc on the handle's
// device).  Returns nullptr on allocation failure.
void *handleScratch(tecoopsContext *ctx, size_t bytes);
int *handleErrorWord(tecoopsContext *ctx);
// error word of tecoopsFlashAttentionDecodeNoAlloc on `device` (nullptr before its first
// call there)
int *noAllocErrorWord(int device);

}  // namespace interface
}  // namespace tecoops

#endif  // TECOOPS_B200_INTERFACE_COMMON_CONTEXT_H_
