// Argument blocks of the flash-attention kernel launchers.
// Mirrors reference teco/ual/args/flash_attention_args.h:37-62
// (FlashAttentionArgs / FlashAttentionPatchArgs).  `spe_num` becomes the SM
// count, `workspace` is actually used (split-KV partials and the prefill tile
// scheduler), and the dtype is carried so that fp16 and bf16 both dispatch.
#ifndef TECOOPS_B200_UAL_ARGS_FLASH_ATTENTION_ARGS_H_
#define TECOOPS_B200_UAL_ARGS_FLASH_ATTENTION_ARGS_H_

#include <cstddef>
#include <cstdint>

namespace tecoops {
namespace ual {
namespace args {

enum class ElemType { F16 = 0, BF16 = 1 };

struct FlashAttentionArgs {
    int num_sms;
    int batch_size;
    int size_per_head;       // D
    int local_head_num;      // Hq
    int local_kv_head_num;   // Hkv
    int block_size;          // tokens per cache page
    int block_table_dim;     // pages per block_table row
    int max_q_seq_len;
    int max_k_seq_len;
    int max_block_num;       // pages in the cache pool
    int total_q;             // rows of q / out
    float softmax_scale;
    ElemType dtype;
    const int *q_seq_lens;   // device [batch]
    const int *kv_seq_lens;  // device [batch]
    const int *block_table;  // device [batch, block_table_dim]
    const void *q;           // [total_q, Hq, D]
    const void *key_cache;   // [max_block_num, Hkv, block_size, D]
    const void *value_cache;
    void *fmha_out;          // [total_q, Hq, D]
    void *workspace;         // device scratch (size from the op's workspaceSize)
    size_t workspace_bytes;
    int *dev_error;          // error word for bounded waits (may be null)
    // options of tecoopsFlashAttentionEx (defaults: the reference's behaviour)
    int causal;              // 1: bottom-right causal
    int window_left;         // < 0: unbounded
    int window_right;        // < 0: unbounded (ignored when causal)
    float *softmax_lse;      // optional fp32 [Hq, total_q], natural log
    // fused reshape_and_cache of each sequence's new token (decode branch only)
    const void *new_key;     // [total_q, Hkv, D] or null
    const void *new_value;
    const int64_t *slot_mapping;
    // cache storage: 0 = [pages, Hkv, bs, D] (reference), 1 = [pages, bs, Hkv, D];
    // cache_fp8: e4m3 elements dequantised as x * k_scale / x * v_scale
    int kv_layout;
    int cache_fp8;
    float k_scale;
    float v_scale;
    // bounded device waits of the decode kernel (tecoopsSetDeviceWaitLimit)
    unsigned long long wait_limit_ns;
    int stall_test;
};

// Branch selection input (reference FlashAttentionPatchArgs).
struct FlashAttentionPatchArgs {
    const FlashAttentionArgs *rvargs;
};

}  // namespace args
}  // namespace ual
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_ARGS_FLASH_ATTENTION_ARGS_H_
