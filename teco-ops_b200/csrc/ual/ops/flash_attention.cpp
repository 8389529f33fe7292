// Branch selection, workspace sizing and launch bridges of the flash_attention
// UAL operator (reference teco/ual/ops/flash_attention/find_flash_attention.cpp:39-43).
#include "ual/ops/flash_attention.hpp"

#include <cmath>
#include <cstdint>

#include "ual/kernels/launchers.h"

namespace tecoops {
namespace ual {
namespace ops {

using args::ElemType;
using args::FlashAttentionArgs;

static kern::AttnShape toShape(const FlashAttentionArgs &a) {
    kern::AttnShape s;
    s.q = a.q;
    s.key_cache = a.key_cache;
    s.value_cache = a.value_cache;
    s.out = a.fmha_out;
    s.q_seq_lens = a.q_seq_lens;
    s.kv_seq_lens = a.kv_seq_lens;
    s.block_table = a.block_table;
    s.batch = a.batch_size;
    s.num_heads = a.local_head_num;
    s.num_kv_heads = a.local_kv_head_num;
    s.head_dim = a.size_per_head;
    s.block_size = a.block_size;
    s.block_table_dim = a.block_table_dim;
    s.num_pages = a.max_block_num;
    s.total_q = a.total_q;
    s.max_q = a.max_q_seq_len;
    s.max_k = a.max_k_seq_len;
    s.scale_log2 = a.softmax_scale * 1.4426950408889634f;
    s.causal = a.causal;
    s.window_left = a.window_left;
    s.window_right = a.window_right;
    s.lse = a.softmax_lse;
    s.kv_layout = a.kv_layout;
    s.cache_fp8 = a.cache_fp8;
    s.k_scale = a.k_scale;
    s.v_scale = a.v_scale;
    return s;
}

static void decodePlan(const FlashAttentionArgs &a, int *split, int *max_splits) {
    kern::decode_plan(a.num_sms, a.batch_size, a.local_kv_head_num,
                      a.local_head_num / a.local_kv_head_num, a.max_k_seq_len, split, max_splits,
                      a.cache_fp8 != 0);
}

static cudaError_t runDecode(const FlashAttentionArgs &a, cudaStream_t stream) {
    kern::DecodeParams p;
    p.q = a.q;
    p.key_cache = a.key_cache;
    p.value_cache = a.value_cache;
    p.out = a.fmha_out;
    p.q_seq_lens = a.q_seq_lens;
    p.kv_seq_lens = a.kv_seq_lens;
    p.block_table = a.block_table;
    p.batch = a.batch_size;
    p.num_heads = a.local_head_num;
    p.num_kv_heads = a.local_kv_head_num;
    p.group = a.local_head_num / a.local_kv_head_num;
    p.num_slices = (p.group + 15) / 16;
    p.head_dim = a.size_per_head;
    p.block_size = a.block_size;
    p.block_table_dim = a.block_table_dim;
    p.num_pages = a.max_block_num;
    p.total_q = a.total_q;
    decodePlan(a, &p.split_tokens, &p.max_splits);
    // an e4m3 cache's k_scale multiplies every score: folded into the softmax scale
    p.scale_log2 = a.softmax_scale * (a.cache_fp8 ? a.k_scale : 1.f) * 1.4426950408889634f;
    p.kv_layout = a.kv_layout;
    p.cache_fp8 = a.cache_fp8;
    p.v_scale = a.cache_fp8 ? a.v_scale : 1.f;
    p.part_o = nullptr;
    p.part_lse = nullptr;
    p.dev_error = a.dev_error;
    p.window_left = a.window_left;   // q_len 1: causal and the right side change nothing
    p.lse = a.softmax_lse;
    p.new_key = a.new_key;
    p.new_value = a.new_value;
    p.slot_mapping = a.slot_mapping;
    p.wait_limit_ns = a.wait_limit_ns;
    p.stall_test = a.stall_test;
    if (p.max_splits > 1) {
        const size_t need = kern::decode_workspace_bytes(p.batch, p.num_heads, p.head_dim,
                                                         p.max_splits);
        if (a.workspace == nullptr || a.workspace_bytes < need) return cudaErrorInvalidValue;
        const size_t recs = (size_t)p.batch * p.num_heads * p.max_splits;
        p.part_o = static_cast<float *>(a.workspace);
        p.part_lse = p.part_o + recs * p.head_dim;
    }
    return kern::launch_decode(p, a.dtype == ElemType::BF16, stream);
}

static int pagesPerSeq(const FlashAttentionArgs &a) {
    return (a.max_k_seq_len + a.block_size - 1) / a.block_size;
}

// e4m3 cache: its referenced pages are dequantised into a compact 16-bit cache in the
// workspace first (kern::launch_kv_dequant), then the tcgen05 prefill runs on that
static cudaError_t runPrefill(const FlashAttentionArgs &a, cudaStream_t stream) {
    const bool bf16 = a.dtype == ElemType::BF16;
    kern::AttnShape s = toShape(a);
    if (a.cache_fp8) {
        kern::KvDequantParams d;
        d.key_cache = a.key_cache;
        d.value_cache = a.value_cache;
        d.kv_seq_lens = a.kv_seq_lens;
        d.block_table = a.block_table;
        d.batch = a.batch_size;
        d.pages_per_seq = pagesPerSeq(a);
        d.block_table_dim = a.block_table_dim;
        d.num_pages = a.max_block_num;
        d.num_kv_heads = a.local_kv_head_num;
        d.block_size = a.block_size;
        d.head_dim = a.size_per_head;
        d.kv_layout = a.kv_layout;
        d.k_scale = a.k_scale;
        d.v_scale = a.v_scale;
        const size_t need = kern::kv_dequant_workspace_bytes(d.batch, d.pages_per_seq,
                                                             d.num_kv_heads, d.block_size,
                                                             d.head_dim);
        if (a.workspace == nullptr || a.workspace_bytes < need) return cudaErrorInvalidValue;
        const size_t cache = (size_t)d.batch * d.pages_per_seq * d.num_kv_heads * d.block_size *
                             d.head_dim * 2;
        uint8_t *base = static_cast<uint8_t *>(a.workspace);
        d.key_out = base;
        d.value_out = base + cache;
        d.bt_out = reinterpret_cast<int *>(base + 2 * cache);
        cudaError_t e = kern::launch_kv_dequant(d, bf16, a.num_sms, stream);
        if (e != cudaSuccess) return e;
        s.key_cache = d.key_out;
        s.value_cache = d.value_out;
        s.block_table = d.bt_out;
        s.block_table_dim = d.pages_per_seq;
        s.num_pages = d.batch * d.pages_per_seq;
        s.kv_layout = 0;
        s.cache_fp8 = 0;
    }
    return kern::launch_prefill(s, bf16, nullptr, a.dev_error, a.num_sms, stream);
}

static cudaError_t runGeneric(const FlashAttentionArgs &a, cudaStream_t stream) {
    return kern::launch_generic_attention(toShape(a), a.dtype == ElemType::BF16, stream);
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

FlashAttentionAlgos FlashAttentionOp::selectAlgo(const FlashAttentionArgs &a) {
    const int group = a.local_head_num / a.local_kv_head_num;
    // the tuned kernels move q, out and the caches in 16-byte vectors, TMA boxes and TMA
    // stores; a view that is only element-aligned takes the generic kernel (scalar access)
    if (!aligned16(a.q) || !aligned16(a.fmha_out) || !aligned16(a.key_cache) ||
        !aligned16(a.value_cache) || !aligned16(a.new_key) || !aligned16(a.new_value))
        return FlashAttentionAlgos::GENERIC;
    // the split-KV grid is (splits, KV heads x head slices, sequences): its y and z
    // extents are limited to 65,535
    if (a.max_q_seq_len == 1 && kern::decode_supported(a.size_per_head, a.block_size, group) &&
        a.batch_size <= 65535 && a.local_kv_head_num * ((group + 15) / 16) <= 65535)
        return FlashAttentionAlgos::DECODE_SPLITKV;
    // e4m3 caches reach the tcgen05 prefill through a dequantised compact copy
    if (kern::prefill_supported(a.size_per_head, a.block_size, group))
        return FlashAttentionAlgos::PREFILL_TCGEN05;
    return FlashAttentionAlgos::GENERIC;
}

size_t FlashAttentionOp::workspaceSize(const FlashAttentionArgs &a) {
    switch (selectAlgo(a)) {
        case FlashAttentionAlgos::DECODE_SPLITKV: {
            int split = 0, ms = 0;
            decodePlan(a, &split, &ms);
            return kern::decode_workspace_bytes(a.batch_size, a.local_head_num, a.size_per_head,
                                                ms);
        }
        case FlashAttentionAlgos::PREFILL_TCGEN05:
            if (a.cache_fp8)
                return kern::kv_dequant_workspace_bytes(a.batch_size, pagesPerSeq(a),
                                                        a.local_kv_head_num, a.block_size,
                                                        a.size_per_head);
            return kern::prefill_workspace_bytes(toShape(a));
        default:
            return 0;
    }
}

Status FlashAttentionOp::findImpl(const args::FlashAttentionPatchArgs *p) {
    if (p == nullptr || p->rvargs == nullptr) return Status::BAD_PARAMETER;
    const FlashAttentionArgs &a = *p->rvargs;
    if (a.size_per_head > 256) return Status::NOT_IMPLEMENTED;
    algo_ = selectAlgo(a);
    switch (algo_) {
        case FlashAttentionAlgos::DECODE_SPLITKV:
            setInstance(&runDecode, "fa_decode_splitkv_sm100");
            break;
        case FlashAttentionAlgos::PREFILL_TCGEN05:
            setInstance(&runPrefill, "fa_prefill_tcgen05_sm100");
            break;
        default:
            setInstance(&runGeneric, "fa_generic_sm100");
            break;
    }
    return Status::SUCCESS;
}

}  // namespace ops
}  // namespace ual
}  // namespace tecoops
