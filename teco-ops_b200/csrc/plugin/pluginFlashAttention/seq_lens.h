// Device-side cu_seqlens_q -> q_seq_lens of the flash-attention plugin.
#ifndef TECOOPS_B200_PLUGIN_FLASH_ATTENTION_SEQ_LENS_H_
#define TECOOPS_B200_PLUGIN_FLASH_ATTENTION_SEQ_LENS_H_

#include <cuda_runtime.h>

namespace TECO_INFER {

// lens[i] = cu_seqlens[i + 1] - cu_seqlens[i] for i < batch, enqueued on `stream`
cudaError_t launchOffsetsToLengths(const int *cu_seqlens, int batch, int *lens,
                                   cudaStream_t stream);

}  // namespace TECO_INFER

#endif  // TECOOPS_B200_PLUGIN_FLASH_ATTENTION_SEQ_LENS_H_
