// Per-sequence query lengths from cu_seqlens_q offsets, on the device and on the
// engine's stream, so the plugin's Enqueue never waits for the GPU (the reference's
// torch binding makes a host round trip here, api/torch_ext.cpp:118-126).
#include <cuda_runtime.h>

#include "pluginFlashAttention/seq_lens.h"

namespace {

__global__ void offsets_to_lengths_kernel(const int *cu, int batch, int *lens) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < batch) lens[i] = cu[i + 1] - cu[i];
}

}  // namespace

namespace TECO_INFER {

cudaError_t launchOffsetsToLengths(const int *cu_seqlens, int batch, int *lens,
                                   cudaStream_t stream) {
    if (batch <= 0) return cudaSuccess;
    offsets_to_lengths_kernel<<<(batch + 255) / 256, 256, 0, stream>>>(cu_seqlens, batch, lens);
    return cudaGetLastError();
}

}  // namespace TECO_INFER
