// tecoopsFlashAttention and its workspace query.
// Follows reference teco/interface/ops/flash_attention.cpp:44-119:
//   - null handle -> NOT_INITIALIZED; k/v cache dtypes differ or shapes differ ->
//     BAD_PARAM; shapes come from the descriptors: batch = blockTable.dim0,
//     D = q.dim2, Hq = q.dim1, Hkv = kCache.dim1, block_size = kCache.dim2,
//     block_table_dim = blockTable.dim1, pages = kCache.dim0 (the max_block_num
//     argument is ignored, as in the reference); scale = 1/sqrt(D).
//   - extension: BFLOAT16 caches are accepted besides HALF (q, out and caches
//     must share the dtype); null pointers, wrong ranks, Hq % Hkv != 0,
//     non-packed strides and an INT32-less block table are rejected
//     (BAD_PARAM / NOT_SUPPORTED) instead of reaching the kernel.
//   - workspace == nullptr: the handle's own scratch is used (grown on demand).
//   - tecoopsFlashAttentionEx: the same call with the binding's flags honoured
//     (scale, causal, window) and an optional log-sum-exp output.
#include <cmath>

#include "interface/common/context.h"
#include "interface/common/run_op.h"
#include "tecoops.h"
#include "ual/com/log.h"
#include "ual/ops/flash_attention.hpp"

using tecoops::ual::args::ElemType;
using tecoops::ual::args::FlashAttentionArgs;
using tecoops::ual::args::FlashAttentionPatchArgs;
using tecoops::ual::ops::FlashAttentionOp;

static bool packed(const tecoopsTensorStruct *d) {
    int s = 1;
    for (int i = d->nbDims - 1; i >= 0; --i) {
        if (d->strideA[i] != s) return false;
        s *= d->dimA[i];
    }
    return true;
}

static bool is16(tecoopsDataType_t t) {
    return t == TECOOPS_DATA_HALF || t == TECOOPS_DATA_BFLOAT16;
}

// layout: cache dims [NB, Hkv, bs, D] (0) or [NB, bs, Hkv, D] (1); allow_fp8: the
// caches may be TECOOPS_DATA_FLOAT8_E4M3 (then q / out carry the 16-bit dtype)
static tecoopsStatus_t flashAttentionCheckArgs(tecoopsHandle_t handle,
                                               const tecoopsTensorDescriptor_t bt,
                                               const tecoopsTensorDescriptor_t q,
                                               const tecoopsTensorDescriptor_t k,
                                               const tecoopsTensorDescriptor_t v,
                                               const tecoopsTensorDescriptor_t o,
                                               int layout = 0, bool allow_fp8 = false) {
    if (handle == nullptr) {
        TECO_ERROR("tecoopsHandle_t is nullptr");
        return TECOOPS_STATUS_NOT_INITIALIZED;
    }
    if (!bt || !q || !k || !v || !o) return TECOOPS_STATUS_BAD_PARAM;
    if (k->dataType != v->dataType) {
        TECO_ERROR("k_cache data_type must be equal to v_cache data_type");
        return TECOOPS_STATUS_BAD_PARAM;
    }
    const bool fp8 = allow_fp8 && k->dataType == TECOOPS_DATA_FLOAT8_E4M3;
    if (!is16(k->dataType) && !fp8) {
        TECO_ERROR("k/v cache must be TECOOPS_DATA_HALF or TECOOPS_DATA_BFLOAT16");
        return TECOOPS_STATUS_BAD_PARAM;
    }
    if (k->nbDims != 4 || v->nbDims != 4 || q->nbDims != 3 || o->nbDims != 3 || bt->nbDims != 2)
        return TECOOPS_STATUS_BAD_PARAM;
    for (int i = 0; i < 4; ++i) {
        if (k->dimA[i] != v->dimA[i]) {
            TECO_ERROR("shape of k v cache is not equal");
            return TECOOPS_STATUS_BAD_PARAM;
        }
    }
    if (!is16(q->dataType) || o->dataType != q->dataType || (!fp8 && q->dataType != k->dataType))
        return TECOOPS_STATUS_BAD_PARAM;
    for (int i = 0; i < 3; ++i)
        if (q->dimA[i] != o->dimA[i]) return TECOOPS_STATUS_BAD_PARAM;
    if (bt->dataType != TECOOPS_DATA_INT32) return TECOOPS_STATUS_BAD_PARAM;
    if (q->dimA[2] != k->dimA[3]) return TECOOPS_STATUS_BAD_PARAM;
    if (bt->dimA[0] <= 0 || bt->dimA[1] <= 0 || q->dimA[1] <= 0 || k->dimA[1] <= 0 ||
        k->dimA[2] <= 0 || k->dimA[0] <= 0 || q->dimA[2] <= 0 || q->dimA[0] < 0)
        return TECOOPS_STATUS_BAD_PARAM;
    const int hkv = layout == 1 ? k->dimA[2] : k->dimA[1];
    if (q->dimA[1] % hkv != 0) return TECOOPS_STATUS_BAD_PARAM;
    if (q->dimA[2] > 256 || (q->dimA[2] & 1)) return TECOOPS_STATUS_NOT_SUPPORTED;
    if (!packed(q) || !packed(o) || !packed(k) || !packed(v) || !packed(bt))
        return TECOOPS_STATUS_NOT_SUPPORTED;
    return TECOOPS_STATUS_SUCCESS;
}

static void fillArgs(FlashAttentionArgs &a, tecoopsHandle_t handle, int max_seqlen_q,
                     int max_seqlen_k, const tecoopsTensorDescriptor_t bt,
                     const tecoopsTensorDescriptor_t q, const tecoopsTensorDescriptor_t k) {
    a.num_sms = handle->num_sms;
    a.batch_size = bt->dimA[0];
    a.size_per_head = q->dimA[2];
    a.local_head_num = q->dimA[1];
    a.local_kv_head_num = k->dimA[1];   // reference layout; tecoopsFlashAttentionEx may swap
    a.block_size = k->dimA[2];
    a.block_table_dim = bt->dimA[1];
    a.max_q_seq_len = max_seqlen_q;
    a.max_k_seq_len = max_seqlen_k;
    a.max_block_num = k->dimA[0];
    a.total_q = q->dimA[0];
    a.softmax_scale = (float)(1.0 / std::sqrt((double)a.size_per_head));
    a.dtype = q->dataType == TECOOPS_DATA_BFLOAT16 ? ElemType::BF16 : ElemType::F16;
    a.causal = 1;
    a.window_left = -1;
    a.window_right = -1;
    a.softmax_lse = nullptr;
    a.new_key = nullptr;
    a.new_value = nullptr;
    a.slot_mapping = nullptr;
    a.kv_layout = 0;
    a.cache_fp8 = 0;
    a.k_scale = 1.f;
    a.v_scale = 1.f;
    a.wait_limit_ns = handle->wait_limit_ns;
    a.stall_test = handle->stall_test;
}

extern "C" tecoopsStatus_t tecoopsGetFlashAttentionWorkspaceSize(
    tecoopsHandle_t handle, int max_seqlen_q, int max_seqlen_k,
    const tecoopsTensorDescriptor_t blockTableDesc, const tecoopsTensorDescriptor_t qDataDesc,
    const tecoopsTensorDescriptor_t kCacheDesc, size_t *workspace_bytes) {
    if (handle == nullptr) return TECOOPS_STATUS_NOT_INITIALIZED;
    if (workspace_bytes == nullptr) return TECOOPS_STATUS_BAD_PARAM;
    const tecoopsStatus_t st = flashAttentionCheckArgs(handle, blockTableDesc, qDataDesc,
                                                       kCacheDesc, kCacheDesc, qDataDesc);
    if (st != TECOOPS_STATUS_SUCCESS) return st;
    FlashAttentionArgs a{};
    fillArgs(a, handle, max_seqlen_q, max_seqlen_k, blockTableDesc, qDataDesc, kCacheDesc);
    *workspace_bytes = FlashAttentionOp::workspaceSize(a);
    return TECOOPS_STATUS_SUCCESS;
}

static tecoopsStatus_t flashAttentionImpl(
    tecoopsHandle_t handle, int max_seqlen_q, int max_seqlen_k, const int *q_seq_lens,
    const int *kv_seq_lens, const tecoopsTensorDescriptor_t blockTableDesc,
    const void *blockTable, const tecoopsTensorDescriptor_t qDataDesc, const void *qData,
    const tecoopsTensorDescriptor_t kCacheDesc, const void *kCache,
    const tecoopsTensorDescriptor_t vCacheDesc, const void *vCache,
    const tecoopsTensorDescriptor_t oDataDesc, void *oData, void *workspace,
    const tecoopsFlashAttentionOptions_t *options, float *softmax_lse) {
    const int layout = options != nullptr ? options->kv_layout : 0;
    if (layout != TECOOPS_KV_LAYOUT_HND && layout != TECOOPS_KV_LAYOUT_NHD)
        return TECOOPS_STATUS_BAD_PARAM;
    tecoopsStatus_t st = flashAttentionCheckArgs(handle, blockTableDesc, qDataDesc, kCacheDesc,
                                                 vCacheDesc, oDataDesc, layout,
                                                 options != nullptr);
    if (st != TECOOPS_STATUS_SUCCESS) return st;
    if (!q_seq_lens || !kv_seq_lens || !blockTable || !kCache || !vCache) return TECOOPS_STATUS_BAD_PARAM;
    if (qDataDesc->dimA[0] > 0 && (!qData || !oData)) return TECOOPS_STATUS_BAD_PARAM;
    if (max_seqlen_q < 0 || max_seqlen_k < 0) return TECOOPS_STATUS_BAD_PARAM;
    if (options != nullptr &&
        (!(options->softmax_scale == options->softmax_scale) ||
         !(options->k_scale == options->k_scale) || !(options->v_scale == options->v_scale)))
        return TECOOPS_STATUS_BAD_PARAM;   // NaN scale
    if (qDataDesc->dimA[0] == 0 || max_seqlen_q == 0) return TECOOPS_STATUS_SUCCESS;

    FlashAttentionArgs args{};
    fillArgs(args, handle, max_seqlen_q, max_seqlen_k, blockTableDesc, qDataDesc, kCacheDesc);
    if (options != nullptr) {
        if (options->softmax_scale > 0.f) args.softmax_scale = options->softmax_scale;
        args.causal = options->causal != 0 ? 1 : 0;
        args.window_left = options->window_left < 0 ? -1 : options->window_left;
        args.window_right = options->window_right < 0 ? -1 : options->window_right;
        args.kv_layout = layout;
        if (layout == TECOOPS_KV_LAYOUT_NHD) {
            args.local_kv_head_num = kCacheDesc->dimA[2];
            args.block_size = kCacheDesc->dimA[1];
        }
        args.cache_fp8 = kCacheDesc->dataType == TECOOPS_DATA_FLOAT8_E4M3 ? 1 : 0;
        args.k_scale = options->k_scale > 0.f ? options->k_scale : 1.f;
        args.v_scale = options->v_scale > 0.f ? options->v_scale : 1.f;
    }
    args.softmax_lse = softmax_lse;
    args.q_seq_lens = q_seq_lens;
    args.kv_seq_lens = kv_seq_lens;
    args.block_table = static_cast<const int *>(blockTable);
    args.q = qData;
    args.key_cache = kCache;
    args.value_cache = vCache;
    args.fmha_out = oData;
    const size_t need = FlashAttentionOp::workspaceSize(args);
    if (workspace != nullptr) {
        args.workspace = workspace;
        args.workspace_bytes = need;
    } else if (need > 0) {
        args.workspace = tecoops::interface::handleScratch(handle, need);
        if (args.workspace == nullptr) return TECOOPS_STATUS_ALLOC_FAILED;
        args.workspace_bytes = handle->scratch_bytes;
    }
    args.dev_error = tecoops::interface::handleErrorWord(handle);

    FlashAttentionPatchArgs patch{&args};
    TECOOPS_RUN_OP(FlashAttentionOp, args, patch, handle);
    return TECOOPS_STATUS_SUCCESS;
}

extern "C" tecoopsStatus_t tecoopsFlashAttention(
    tecoopsHandle_t handle, int max_seqlen_q, int max_seqlen_k, int max_block_num,
    const int *q_seq_lens, const int *kv_seq_lens, const tecoopsTensorDescriptor_t blockTableDesc,
    const void *blockTable, const tecoopsTensorDescriptor_t qDataDesc, const void *qData,
    const tecoopsTensorDescriptor_t kCacheDesc, const void *kCache,
    const tecoopsTensorDescriptor_t vCacheDesc, const void *vCache,
    const tecoopsTensorDescriptor_t oDataDesc, void *oData, void *workspace) {
    (void)max_block_num;   // the reference also takes the page count from kCacheDesc
    return flashAttentionImpl(handle, max_seqlen_q, max_seqlen_k, q_seq_lens, kv_seq_lens,
                              blockTableDesc, blockTable, qDataDesc, qData, kCacheDesc, kCache,
                              vCacheDesc, vCache, oDataDesc, oData, workspace, nullptr, nullptr);
}

extern "C" tecoopsStatus_t tecoopsReshapeAndCacheFlashAttentionDecode(
    tecoopsHandle_t handle, const void *key, const void *value, const int64_t *slot_mapping,
    int max_seqlen_k, const int *q_seq_lens, const int *kv_seq_lens,
    const tecoopsTensorDescriptor_t blockTableDesc, const void *blockTable,
    const tecoopsTensorDescriptor_t qDataDesc, const void *qData,
    const tecoopsTensorDescriptor_t kCacheDesc, void *kCache,
    const tecoopsTensorDescriptor_t vCacheDesc, void *vCache,
    const tecoopsTensorDescriptor_t oDataDesc, void *oData, void *workspace) {
    tecoopsStatus_t st = flashAttentionCheckArgs(handle, blockTableDesc, qDataDesc, kCacheDesc,
                                                 vCacheDesc, oDataDesc);
    if (st != TECOOPS_STATUS_SUCCESS) return st;
    if (!key || !value || !slot_mapping || !q_seq_lens || !kv_seq_lens || !blockTable ||
        !kCache || !vCache || max_seqlen_k < 0)
        return TECOOPS_STATUS_BAD_PARAM;
    const int T = qDataDesc->dimA[0];
    if (T == 0) return TECOOPS_STATUS_SUCCESS;
    if (!qData || !oData) return TECOOPS_STATUS_BAD_PARAM;
    FlashAttentionArgs args{};
    fillArgs(args, handle, 1, max_seqlen_k, blockTableDesc, qDataDesc, kCacheDesc);
    // every pointer before the branch choice: it depends on their alignment, and only the
    // split-KV kernel performs the scatter of the new tokens itself
    args.q_seq_lens = q_seq_lens;
    args.kv_seq_lens = kv_seq_lens;
    args.block_table = static_cast<const int *>(blockTable);
    args.q = qData;
    args.key_cache = kCache;
    args.value_cache = vCache;
    args.fmha_out = oData;
    args.new_key = key;
    args.new_value = value;
    args.slot_mapping = slot_mapping;
    if (FlashAttentionOp::selectAlgo(args) !=
            tecoops::ual::ops::FlashAttentionAlgos::DECODE_SPLITKV ||
        (args.size_per_head % 8) != 0) {
        // shapes outside the split-KV kernel: the two operators back to back
        st = tecoopsReshapeAndCache(handle, key, value, slot_mapping, kCache, vCache, T,
                                    args.local_kv_head_num, args.size_per_head,
                                    args.max_block_num, args.block_size);
        if (st != TECOOPS_STATUS_SUCCESS) return st;
        return flashAttentionImpl(handle, 1, max_seqlen_k, q_seq_lens, kv_seq_lens,
                                  blockTableDesc, blockTable, qDataDesc, qData, kCacheDesc,
                                  kCache, vCacheDesc, vCache, oDataDesc, oData, workspace,
                                  nullptr, nullptr);
    }
    const size_t need = FlashAttentionOp::workspaceSize(args);
    if (workspace != nullptr) {
        args.workspace = workspace;
        args.workspace_bytes = need;
    } else if (need > 0) {
        args.workspace = tecoops::interface::handleScratch(handle, need);
        if (args.workspace == nullptr) return TECOOPS_STATUS_ALLOC_FAILED;
        args.workspace_bytes = handle->scratch_bytes;
    }
    args.dev_error = tecoops::interface::handleErrorWord(handle);
    FlashAttentionPatchArgs patch{&args};
    TECOOPS_RUN_OP(FlashAttentionOp, args, patch, handle);
    return TECOOPS_STATUS_SUCCESS;
}

extern "C" tecoopsStatus_t tecoopsFlashAttentionEx(
    tecoopsHandle_t handle, int max_seqlen_q, int max_seqlen_k, int max_block_num,
    const int *q_seq_lens, const int *kv_seq_lens, const tecoopsTensorDescriptor_t blockTableDesc,
    const void *blockTable, const tecoopsTensorDescriptor_t qDataDesc, const void *qData,
    const tecoopsTensorDescriptor_t kCacheDesc, const void *kCache,
    const tecoopsTensorDescriptor_t vCacheDesc, const void *vCache,
    const tecoopsTensorDescriptor_t oDataDesc, void *oData, void *workspace,
    const tecoopsFlashAttentionOptions_t *options, float *softmax_lse) {
    (void)max_block_num;
    return flashAttentionImpl(handle, max_seqlen_q, max_seqlen_k, q_seq_lens, kv_seq_lens,
                              blockTableDesc, blockTable, qDataDesc, qData, kCacheDesc, kCache,
                              vCacheDesc, vCache, oDataDesc, oData, workspace, options,
                              softmax_lse);
}
