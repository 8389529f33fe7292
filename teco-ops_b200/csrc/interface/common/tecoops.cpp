// Handle, tensor descriptors, error strings, memset and the NOT_SUPPORTED stubs
// of the reference's off-path operators.
// Behaviour follows reference teco/interface/common/tecoops.cpp:38-258:
//   - tecoopsCreate(nullptr) -> BAD_PARAM; the stream defaults to the legacy
//     default stream (nullptr);
//   - SetTensorNdDescriptor with nbDims <= 0 -> BAD_PARAM, null strideA -> packed
//     row-major strides; GetTensorNdDescriptor copies min(nbDims, requested);
//   - Set/GetTensor4dDescriptor support NCHW/NHWC/CHWN/NWHC strides.
// Differences (documented in the header): nbDims above TECOOPS_DIM_MAX is
// rejected (BAD_PARAM) instead of spilling to heap arrays, and the handle
// records the current CUDA device, its SM count and an owned scratch buffer.
#include <cuda_runtime.h>

#include <cstring>
#include <new>

#include "interface/common/context.h"
#include "tecoops.h"
#include "ual/com/log.h"

namespace tecoops {
namespace interface {

void *handleScratch(tecoopsContext *ctx, size_t bytes) {
    if (bytes == 0) return ctx->scratch;
    if (ctx->scratch_bytes >= bytes) return ctx->scratch;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != ctx->device) cudaSetDevice(ctx->device);
    if (ctx->scratch) cudaFree(ctx->scratch);   // synchronises: no kernel still uses it
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
    size_t grow = bytes + bytes / 4;
    void *p = nullptr;
    if (cudaMalloc(&p, grow) == cudaSuccess) {
        ctx->scratch = p;
        ctx->scratch_bytes = grow;
    } else {
        cudaGetLastError();
    }
    if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
    return ctx->scratch;
}

int *handleErrorWord(tecoopsContext *ctx) {
    if (ctx->dev_error) return ctx->dev_error;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != ctx->device) cudaSetDevice(ctx->device);
    int *p = nullptr;
    if (cudaMalloc(&p, 4 * sizeof(int)) == cudaSuccess) {
        cudaMemset(p, 0, 4 * sizeof(int));
        ctx->dev_error = p;
    } else {
        cudaGetLastError();
    }
    if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
    return ctx->dev_error;
}

}  // namespace interface
}  // namespace tecoops

extern "C" {

tecoopsStatus_t tecoopsCreate(tecoopsHandle_t *handle) {
    if (handle == nullptr) return TECOOPS_STATUS_BAD_PARAM;
    tecoopsContext *ctx = new (std::nothrow) tecoopsContext();
    if (ctx == nullptr) return TECOOPS_STATUS_ALLOC_FAILED;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        ctx->device = dev;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
            sms > 0)
            ctx->num_sms = sms;
    } else {
        cudaGetLastError();   // no device visible: keep defaults, fail at launch time
    }
    *handle = ctx;
    return TECOOPS_STATUS_SUCCESS;
}

tecoopsStatus_t tecoopsDestroy(tecoopsHandle_t handle) {
    if (handle == nullptr) return TECOOPS_STATUS_BAD_PARAM;
    if (handle->scratch) cudaFree(handle->scratch);
    if (handle->dev_error) cudaFree(handle->dev_error);
    delete handle;
    return TECOOPS_STATUS_SUCCESS;
}

tecoopsStatus_t tecoopsSetStream(tecoopsHandle_t handle, cudaStream_t stream) {
    if (handle == nullptr) return TECOOPS_STATUS_BAD_PARAM;
    handle->stream = stream;
    return TECOOPS_STATUS_SUCCESS;
}

tecoopsStatus_t tecoopsGetStream(tecoopsHandle_t handle, cudaStream_t *stream) {
    if (handle == nullptr || stream == nullptr) return TECOOPS_STATUS_BAD_PARAM;
    *stream = handle->stream;
    return TECOOPS_STATUS_SUCCESS;
}

const char *tecoopsGetErrorString(tecoopsStatus_t status) {
    switch (status) {
        case TECOOPS_STATUS_SUCCESS: return "TECOOPS_STATUS_SUCCESS";
        case TECOOPS_STATUS_NOT_INITIALIZED: return "TECOOPS_STATUS_NOT_INITIALIZED";
        case TECOOPS_STATUS_ALLOC_FAILED: return "TECOOPS_STATUS_ALLOC_FAILED";
        case TECOOPS_STATUS_BAD_PARAM: return "TECOOPS_STATUS_BAD_PARAM";
        case TECOOPS_STATUS_INTERNAL_ERROR: return "TECOOPS_STATUS_INTERNAL_ERROR";
        case TECOOPS_STATUS_INVALID_VALUE: return "TECOOPS_STATUS_INVALID_VALUE";
        case TECOOPS_STATUS_NOT_SUPPORTED: return "TECOOPS_STATUS_NOT_SUPPORTED";
        default: return "UNKNOWN_ERROR";
    }
}

tecoopsStatus_t tecoopsCreateTensorDescriptor(tecoopsTensorDescriptor_t *tensorDesc) {
    if (tensorDesc == nullptr) return TECOOPS_STATUS_BAD_PARAM;
    *tensorDesc = new (std::nothrow) tecoopsTensorStruct();
    return *tensorDesc ? TECOOPS_STATUS_SUCCESS : TECOOPS_STATUS_ALLOC_FAILED;
}

tecoopsStatus_t tecoopsSetTensor4dDescriptor(tecoopsTensorDescriptor_t d,
                                             tecoopsTensorFormat_t format,
                                             tecoopsDataType_t dataType, int n, int c, int h,
                                             int w) {
    if (d == nullptr || n <= 0 || c <= 0 || h <= 0 || w <= 0) return TECOOPS_STATUS_BAD_PARAM;
    int ns, cs, hs, ws;
    switch (format) {
        case TECOOPS_TENSOR_NCHW: ns = c * h * w; cs = h * w; hs = w; ws = 1; break;
        case TECOOPS_TENSOR_NHWC: ns = h * w * c; cs = 1; hs = w * c; ws = c; break;
        case TECOOPS_TENSOR_CHWN: ns = 1; cs = h * w * n; hs = w * n; ws = n; break;
        case TECOOPS_TENSOR_NWHC: ns = w * h * c; cs = 1; hs = c; ws = h * c; break;
        default: return TECOOPS_STATUS_BAD_PARAM;
    }
    d->format = format;
    d->dataType = dataType;
    d->nbDims = 4;
    const int dims[4] = {n, c, h, w};
    const int strides[4] = {ns, cs, hs, ws};
    std::memcpy(d->dimA, dims, sizeof(dims));
    std::memcpy(d->strideA, strides, sizeof(strides));
    return TECOOPS_STATUS_SUCCESS;
}

tecoopsStatus_t tecoopsGetTensor4dDescriptor(const tecoopsTensorDescriptor_t d,
                                             tecoopsDataType_t *dataType, int *n, int *c, int *h,
                                             int *w, int *nStride, int *cStride, int *hStride,
                                             int *wStride) {
    if (d == nullptr || d->nbDims != 4) return TECOOPS_STATUS_BAD_PARAM;
    if (dataType) *dataType = d->dataType;
    if (n) *n = d->dimA[0];
    if (c) *c = d->dimA[1];
    if (h) *h = d->dimA[2];
    if (w) *w = d->dimA[3];
    if (nStride) *nStride = d->strideA[0];
    if (cStride) *cStride = d->strideA[1];
    if (hStride) *hStride = d->strideA[2];
    if (wStride) *wStride = d->strideA[3];
    return TECOOPS_STATUS_SUCCESS;
}

tecoopsStatus_t tecoopsSetTensorNdDescriptor(tecoopsTensorDescriptor_t d,
                                             tecoopsDataType_t dataType, int nbDims,
                                             const int dimA[], const int strideA[]) {
    if (d == nullptr || nbDims <= 0 || nbDims > TECOOPS_DIM_MAX || dimA == nullptr)
        return TECOOPS_STATUS_BAD_PARAM;
    d->dataType = dataType;
    d->format = TECOOPS_TENSOR_NCHW;
    d->nbDims = nbDims;
    std::memcpy(d->dimA, dimA, sizeof(int) * nbDims);
    if (strideA != nullptr) {
        std::memcpy(d->strideA, strideA, sizeof(int) * nbDims);
    } else {
        d->strideA[nbDims - 1] = 1;
        for (int i = nbDims - 2; i >= 0; --i) d->strideA[i] = d->strideA[i + 1] * dimA[i + 1];
    }
    return TECOOPS_STATUS_SUCCESS;
}

tecoopsStatus_t tecoopsGetTensorNdDescriptor(const tecoopsTensorDescriptor_t d,
                                             int nbDimsRequested, tecoopsDataType_t *dataType,
                                             int *nbDims, int dimA[], int strideA[]) {
    if (d == nullptr || nbDimsRequested <= 0) return TECOOPS_STATUS_BAD_PARAM;
    if (dataType) *dataType = d->dataType;
    int n = d->nbDims;
    if (nbDims) {
        *nbDims = d->nbDims;
        n = n < nbDimsRequested ? n : nbDimsRequested;
    }
    if (dimA) std::memcpy(dimA, d->dimA, sizeof(int) * n);
    if (strideA) std::memcpy(strideA, d->strideA, sizeof(int) * n);
    return TECOOPS_STATUS_SUCCESS;
}

tecoopsStatus_t tecoopsDestroyTensorDescriptor(tecoopsTensorDescriptor_t d) {
    delete d;
    return TECOOPS_STATUS_SUCCESS;
}

tecoopsStatus_t tecoopsMemset(tecoopsHandle_t handle, void *x, const int value, size_t size) {
    if (handle == nullptr) return TECOOPS_STATUS_NOT_INITIALIZED;
    if (x == nullptr && size > 0) return TECOOPS_STATUS_BAD_PARAM;
    if (size == 0) return TECOOPS_STATUS_SUCCESS;
    return cudaMemsetAsync(x, value, size, handle->stream) == cudaSuccess
               ? TECOOPS_STATUS_SUCCESS
               : TECOOPS_STATUS_INTERNAL_ERROR;
}

tecoopsStatus_t tecoopsGetDeviceErrorStatus(tecoopsHandle_t handle, int *error_code) {
    if (handle == nullptr) return TECOOPS_STATUS_NOT_INITIALIZED;
    if (error_code) *error_code = 0;
    // the handle's own word, then the word of tecoopsFlashAttentionDecodeNoAlloc on the
    // handle's device (that entry point allocates nothing, so its word is static)
    int *words[2] = {handle->dev_error,
                     tecoops::interface::noAllocErrorWord(handle->device)};
    if (words[0] == nullptr && words[1] == nullptr) return TECOOPS_STATUS_SUCCESS;
    if (cudaStreamSynchronize(handle->stream) != cudaSuccess) return TECOOPS_STATUS_INTERNAL_ERROR;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != handle->device) cudaSetDevice(handle->device);
    tecoopsStatus_t st = TECOOPS_STATUS_SUCCESS;
    for (int *w : words) {
        if (w == nullptr) continue;
        int v = 0;
        if (cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
            st = TECOOPS_STATUS_INTERNAL_ERROR;
            break;
        }
        if (v != 0) {
            cudaMemset(w, 0, sizeof(int));
            if (st == TECOOPS_STATUS_SUCCESS && error_code) *error_code = v;
            st = TECOOPS_STATUS_INTERNAL_ERROR;
        }
    }
    if (prev >= 0 && prev != handle->device) cudaSetDevice(prev);
    return st;
}

tecoopsStatus_t tecoopsSetDeviceWaitLimit(tecoopsHandle_t handle, unsigned long long limit_ns,
                                          int stall_test) {
    if (handle == nullptr) return TECOOPS_STATUS_NOT_INITIALIZED;
    if (limit_ns == 0) return TECOOPS_STATUS_BAD_PARAM;
    handle->wait_limit_ns = limit_ns;
    handle->stall_test = stall_test != 0 ? 1 : 0;
    return TECOOPS_STATUS_SUCCESS;
}

// ---- reference operators that are not on the attention path ----
tecoopsStatus_t tecoopsFlattenRays(tecoopsHandle_t, const int *, uint32_t, uint32_t, int *,
                                   tecoopsAlgo_t) {
    return TECOOPS_STATUS_NOT_SUPPORTED;
}
tecoopsStatus_t tecoopsReduceVariance(const tecoopsHandle_t, int, int,
                                      const tecoopsTensorDescriptor_t, const void *,
                                      const tecoopsTensorDescriptor_t, void *) {
    return TECOOPS_STATUS_NOT_SUPPORTED;
}
tecoopsStatus_t tecoopsMorton3DInvert(tecoopsHandle_t, const int *, uint32_t, int *) {
    return TECOOPS_STATUS_NOT_SUPPORTED;
}
tecoopsStatus_t tecoopsCausalConv1d(tecoopsHandle_t, int, int, int, int, int, int, int, int, int,
                                    int, const void *, void *, const void *, void *, const int *,
                                    const int *, const int8_t *) {
    return TECOOPS_STATUS_NOT_SUPPORTED;
}

}  // extern "C"
