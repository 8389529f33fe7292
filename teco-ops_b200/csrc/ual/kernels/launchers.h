// Host-side launch entry points of the device kernels (the UAL kernel table
// points at these).  Parameter blocks are plain structs passed by value to the
// kernels.
#ifndef TECOOPS_B200_UAL_KERNELS_LAUNCHERS_H_
#define TECOOPS_B200_UAL_KERNELS_LAUNCHERS_H_

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "ual/args/reshape_and_cache_args.h"
#include "ual/args/rms_norm_args.h"

namespace tecoops {
namespace kern {

// ---- reshape_and_cache ---------------------------------------------------------
cudaError_t launch_reshape_and_cache(const ual::args::ReshapeAndCacheArgs &a, int num_sms,
                                     cudaStream_t stream);

// ---- paged attention: shared shape block ---------------------------------------
struct AttnShape {
    const void *q;            // [total_q, Hq, D]
    const void *key_cache;    // [num_pages, Hkv, block_size, D]
    const void *value_cache;
    void *out;                // [total_q, Hq, D]
    const int *q_seq_lens;    // [batch]
    const int *kv_seq_lens;   // [batch]
    const int *block_table;   // [batch, block_table_dim]
    int batch;
    int num_heads;
    int num_kv_heads;
    int head_dim;
    int block_size;
    int block_table_dim;
    int num_pages;
    int total_q;
    int max_q;
    int max_k;
    float scale_log2;         // softmax_scale * log2(e)
    // key j is admissible for row i (off = kv_len - q_len) when j < kv_len and
    //   j <= off + i (causal) or j <= off + i + window_right (non-causal, right >= 0)
    //   j >= off + i - window_left (window_left >= 0)
    int causal;
    int window_left;
    int window_right;
    float *lse;               // optional [Hq, total_q] natural-log log-sum-exp
    int kv_layout;            // 0: [pages, Hkv, bs, D]; 1: [pages, bs, Hkv, D]
    int cache_fp8;            // e4m3 cache elements, dequantised with k_scale / v_scale
    float k_scale;
    float v_scale;
};

// ---- split-KV decode -------------------------------------------------------------
struct DecodeParams {
    const void *q;
    const void *key_cache;
    const void *value_cache;
    void *out;
    const int *q_seq_lens;
    const int *kv_seq_lens;
    const int *block_table;
    int batch;
    int num_heads;
    int num_kv_heads;
    int group;          // num_heads / num_kv_heads
    int num_slices;     // ceil(group / 16)
    int head_dim;
    int block_size;
    int block_table_dim;
    int num_pages;      // pages in the cache pool (ids outside read as zeros)
    int total_q;        // rows of q / out
    int split_tokens;   // multiple of 64
    int max_splits;
    float scale_log2;
    float *part_o;      // [batch, Hq, max_splits, D]
    float *part_lse;    // [batch, Hq, max_splits]
    int *dev_error;     // error word for bounded waits (may be null)
    int window_left;    // < 0: unbounded; else keys j >= kv_len - 1 - window_left
    float *lse;         // optional [Hq, total_q] natural-log log-sum-exp
    // fused reshape_and_cache (all null when unfused): the new token of sequence b is
    // q row b's key/value [total_q, Hkv, D], written to cache slot slot_mapping[row]
    // (skipped when < 0) and attended at position kv_len - 1 from these inputs
    const void *new_key;
    const void *new_value;
    const int64_t *slot_mapping;
    int kv_layout;      // 0: [pages, Hkv, bs, D]; 1: [pages, bs, Hkv, D]
    int cache_fp8;      // e4m3 cache: K*k_scale folded into scale_log2, O *= v_scale
    float v_scale;
    unsigned long long wait_limit_ns;   // limit of each bounded mbarrier wait
    int stall_test;     // test of the give-up path: the first ring wait of each consumer
                        // waits on a barrier that nothing completes
};

bool decode_supported(int head_dim, int block_size, int group);
// cache_fp8: an e4m3 cache (with a GQA group above 8 its splits are longer)
void decode_plan(int num_sms, int batch, int kv_heads, int group, int max_k, int *split_tokens,
                 int *max_splits, bool cache_fp8 = false);
size_t decode_workspace_bytes(int batch, int num_heads, int head_dim, int max_splits);
cudaError_t launch_decode(const DecodeParams &p, bool bf16, cudaStream_t stream);

// ---- tcgen05 prefill -------------------------------------------------------------
bool prefill_supported(int head_dim, int block_size, int group);
size_t prefill_workspace_bytes(const AttnShape &s);
cudaError_t launch_prefill(const AttnShape &s, bool bf16, void *workspace, int *dev_error,
                           int num_sms, cudaStream_t stream);

// ---- e4m3 cache -> 16-bit compact cache for the tcgen05 prefill ------------------
struct KvDequantParams {
    const void *key_cache;     // e4m3, layout kv_layout
    const void *value_cache;
    const int *kv_seq_lens;
    const int *block_table;    // [batch, block_table_dim]
    void *key_out;             // 16-bit [batch * pages_per_seq, Hkv, block_size, D]
    void *value_out;
    int *bt_out;               // [batch, pages_per_seq]: b * pages_per_seq + i
    int batch;
    int pages_per_seq;         // ceil(max_seqlen_k / block_size)
    int block_table_dim;
    int num_pages;
    int num_kv_heads;
    int block_size;
    int head_dim;
    int kv_layout;
    float k_scale;
    float v_scale;
};
size_t kv_dequant_workspace_bytes(int batch, int pages_per_seq, int num_kv_heads, int block_size,
                                  int head_dim);
cudaError_t launch_kv_dequant(const KvDequantParams &p, bool bf16, int num_sms,
                              cudaStream_t stream);

// ---- rms_norm --------------------------------------------------------------------
cudaError_t launch_rms_norm(const ual::args::RmsNormArgs &a, cudaStream_t stream);

// ---- generic (any head_dim <= 256, any block_size) --------------------------------
cudaError_t launch_generic_attention(const AttnShape &s, bool bf16, cudaStream_t stream);

}  // namespace kern
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_KERNELS_LAUNCHERS_H_
