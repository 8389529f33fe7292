// flash_attention UAL operator with its branch table.
// Mirrors reference teco/ual/ops/flash_attention/flash_attention.hpp:43-82 and
// find_flash_attention.cpp:39-43, where one branch always runs.  Here `find`
// chooses between three sm_100a kernels:
//   DECODE_SPLITKV  max_seqlen_q == 1 and the shape is covered (head_dim 64/128,
//                   block_size a multiple of 16)
//   PREFILL_TCGEN05 everything else the tcgen05 kernel covers (head_dim 64/128,
//                   block_size a power of two >= 8 or a multiple of 128)
//   GENERIC         any other head_dim <= 256 / block_size (CUDA-core kernel)
#ifndef TECOOPS_B200_UAL_OPS_FLASH_ATTENTION_HPP_
#define TECOOPS_B200_UAL_OPS_FLASH_ATTENTION_HPP_

#include <cstddef>

#include "ual/args/flash_attention_args.h"
#include "ual/ops/base_op.hpp"

namespace tecoops {
namespace ual {
namespace ops {

struct FlashAttentionTraits {
    using ArgsType = args::FlashAttentionArgs;
    using PatchType = args::FlashAttentionPatchArgs;
    using PImplType = cudaError_t (*)(const args::FlashAttentionArgs &, cudaStream_t);
};

enum class FlashAttentionAlgos { DECODE_SPLITKV = 0, PREFILL_TCGEN05 = 1, GENERIC = 2 };

struct FlashAttentionOp : BaseOp<FlashAttentionOp, FlashAttentionTraits> {
    Status findImpl(const args::FlashAttentionPatchArgs *p);
    FlashAttentionAlgos algo() const { return algo_; }
    // device scratch the selected branch needs (bytes)
    static size_t workspaceSize(const args::FlashAttentionArgs &a);
    static FlashAttentionAlgos selectAlgo(const args::FlashAttentionArgs &a);

 private:
    FlashAttentionAlgos algo_ = FlashAttentionAlgos::GENERIC;
};

}  // namespace ops
}  // namespace ual
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_OPS_FLASH_ATTENTION_HPP_
