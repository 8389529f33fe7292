/*
 * tecoops.h — C API of the B200 (sm_100a) implementation of the Teco-Ops
 * paged-KV attention path.
 *
 * Drop-in for the reference header teco/interface/include/tecoops.h:
 * same enums (values included), same handle / tensor-descriptor API and the
 * same signatures for the two hot-path operators.  The only type change is
 * the stream: the reference's `sdaaStream_t` is a CUDA stream here; a typedef
 * keeps sources that spell `sdaaStream_t` compiling.
 *
 * All data pointers are caller-owned DEVICE memory.  Every operator call is
 * asynchronous on the handle's stream and never synchronises the host.
 *
 * rms_norm (with the fused residual add), the step before the QKV projection in
 * the same decoder layer, is implemented.  The reference's other operators
 * (causal_conv1d, reduce_variance, flatten_rays, morton3D_invert) are exported so
 * that a program linking the reference library still links, but they return
 * TECOOPS_STATUS_NOT_SUPPORTED (they are not on this path).
 */
#ifndef TECOOPS_B200_INCLUDE_TECOOPS_H_
#define TECOOPS_B200_INCLUDE_TECOOPS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* CUDA stream handle without dragging in the CUDA headers (identical to the
 * runtime's own definition of cudaStream_t). */
#ifndef __CUDA_RUNTIME_API_H__
struct CUstream_st;
typedef struct CUstream_st *cudaStream_t;
#endif
typedef cudaStream_t sdaaStream_t; /* source compatibility with the reference */

#define TECOOPS_DIM_MAX 8

/* reference: teco/interface/include/tecoops.h:39-47 */
typedef enum {
    TECOOPS_STATUS_SUCCESS = 0,
    TECOOPS_STATUS_NOT_INITIALIZED = 1,
    TECOOPS_STATUS_ALLOC_FAILED = 2,
    TECOOPS_STATUS_BAD_PARAM = 3,
    TECOOPS_STATUS_INTERNAL_ERROR = 4,
    TECOOPS_STATUS_INVALID_VALUE = 5,
    TECOOPS_STATUS_NOT_SUPPORTED = 6,
} tecoopsStatus_t;

/* reference: tecoops.h:49-58 */
typedef enum {
    TECOOPS_TENSOR_NCHW = 0,
    TECOOPS_TENSOR_NHWC = 1,
    TECOOPS_TENSOR_CHWN = 2,
    TECOOPS_TENSOR_NWHC = 3,
    TECOOPS_TENSOR_NCDHW = 4,
    TECOOPS_TENSOR_NDHWC = 5,
    TECOOPS_TENSOR_CDHWN = 6,
} tecoopsTensorFormat_t;

/* reference: tecoops.h:60-71 */
typedef enum {
    TECOOPS_ALGO_0 = 0,
    TECOOPS_ALGO_1,
    TECOOPS_ALGO_2,
    TECOOPS_ALGO_3,
    TECOOPS_ALGO_4,
    TECOOPS_ALGO_5,
    TECOOPS_ALGO_6,
    TECOOPS_ALGO_7,
    TECOOPS_ALGO_8,
    TECOOPS_ALGO_9,
} tecoopsAlgo_t;

/* reference: tecoops.h:73-85 */
typedef enum {
    TECOOPS_DATA_FLOAT = 0,
    TECOOPS_DATA_HALF = 1,
    TECOOPS_DATA_INT8 = 2,
    TECOOPS_DATA_INT16 = 3,
    TECOOPS_DATA_INT32 = 4,
    TECOOPS_DATA_INT64 = 5,
    TECOOPS_DATA_UINT8 = 6,
    TECOOPS_DATA_BOOL = 7,
    TECOOPS_DATA_DOUBLE = 8,
    TECOOPS_DATA_BFLOAT16 = 9,
    TECOOPS_DATA_COMPLEX_FLOAT = 10,
    /* extension: 8-bit float KV cache (e4m3, finite saturation) with a per-tensor scale */
    TECOOPS_DATA_FLOAT8_E4M3 = 32,
} tecoopsDataType_t;

/* extension: page layouts of the paged K/V cache */
typedef enum {
    TECOOPS_KV_LAYOUT_HND = 0, /* [num_blocks, num_kv_heads, block_size, head_size] (reference) */
    TECOOPS_KV_LAYOUT_NHD = 1, /* [num_blocks, block_size, num_kv_heads, head_size] (vLLM)      */
} tecoopsKvLayout_t;

/*
 * extension: how a paged K/V cache is stored.
 *   kv_layout    : tecoopsKvLayout_t
 *   cache_dtype  : TECOOPS_DATA_HALF / TECOOPS_DATA_BFLOAT16 (the key's dtype; bit-exact
 *                  copy) or TECOOPS_DATA_FLOAT8_E4M3 (cache = e4m3(x / scale), saturated
 *                  to +-448; attention reads back e4m3 * scale)
 *   k_scale, v_scale : per-tensor scales of an FP8 cache (<= 0 means 1)
 */
typedef struct tecoopsKvCacheConfig {
    int kv_layout;
    tecoopsDataType_t cache_dtype;
    float k_scale;
    float v_scale;
} tecoopsKvCacheConfig_t;

typedef struct tecoopsContext *tecoopsHandle_t;
typedef struct tecoopsTensorStruct *tecoopsTensorDescriptor_t;

/* ---- handle (reference: tecoops.h:90-94; interface/common/tecoops.cpp:38-76) ---- */
tecoopsStatus_t tecoopsCreate(tecoopsHandle_t *handle);
tecoopsStatus_t tecoopsDestroy(tecoopsHandle_t handle);
tecoopsStatus_t tecoopsSetStream(tecoopsHandle_t handle, cudaStream_t stream);
tecoopsStatus_t tecoopsGetStream(tecoopsHandle_t handle, cudaStream_t *stream);
const char *tecoopsGetErrorString(tecoopsStatus_t status);

/* ---- tensor descriptors (reference: tecoops.h:96-122; tecoops.cpp:78-237) ---- */
tecoopsStatus_t tecoopsCreateTensorDescriptor(tecoopsTensorDescriptor_t *tensorDesc);
tecoopsStatus_t tecoopsSetTensor4dDescriptor(tecoopsTensorDescriptor_t tensorDesc,
                                             tecoopsTensorFormat_t format,
                                             tecoopsDataType_t dataType,
                                             int n, int c, int h, int w);
tecoopsStatus_t tecoopsGetTensor4dDescriptor(const tecoopsTensorDescriptor_t tensorDesc,
                                             tecoopsDataType_t *dataType,
                                             int *n, int *c, int *h, int *w,
                                             int *nStride, int *cStride, int *hStride,
                                             int *wStride);
tecoopsStatus_t tecoopsSetTensorNdDescriptor(tecoopsTensorDescriptor_t tensorDesc,
                                             tecoopsDataType_t dataType, int nbDims,
                                             const int dimA[], const int strideA[]);
tecoopsStatus_t tecoopsGetTensorNdDescriptor(const tecoopsTensorDescriptor_t tensorDesc,
                                             int nbDimsRequested, tecoopsDataType_t *dataType,
                                             int *nbDims, int dimA[], int strideA[]);
tecoopsStatus_t tecoopsDestroyTensorDescriptor(tecoopsTensorDescriptor_t tensorDesc);

/* ---- memset (reference: tecoops.h:128; used by the reshape plugin) ---- */
tecoopsStatus_t tecoopsMemset(tecoopsHandle_t handle, void *x, const int value, size_t size);

/*
 * reshape_and_cache — scatter K/V rows into the paged cache.
 * Replaces reference tecoops.h:130-136 (teco/interface/ops/reshape_and_cache.cpp:64-105).
 *   key, value    : [num_tokens, num_kv_heads, head_size], 2-byte elements (fp16 or bf16)
 *   slot_mapping  : int64 [num_tokens]; slot < 0 means "padding, skip"
 *   key_cache,
 *   value_cache   : [num_blocks, num_kv_heads, block_size, head_size]
 *   cache[slot / block_size][h][slot % block_size][:] = key[t][h][:]
 * The copy is bit-exact.  Slots >= num_blocks*block_size are skipped too (the
 * reference writes out of bounds there).  Two tokens mapped to the same slot
 * race, as in the reference.
 */
/*
 * Extension: reshape_and_cache into a cache described by `cache` (nullptr: the
 * reference's layout and a bit-exact copy).  key_dtype is TECOOPS_DATA_HALF or
 * TECOOPS_DATA_BFLOAT16; num_kv_heads / block_size keep their meaning whatever the
 * layout.
 */
tecoopsStatus_t tecoopsReshapeAndCacheEx(tecoopsHandle_t handle, const void *key,
                                         const void *value, const int64_t *slot_mapping,
                                         void *key_cache, void *value_cache, int num_tokens,
                                         int num_kv_heads, int head_size, int num_blocks,
                                         int block_size, tecoopsDataType_t key_dtype,
                                         const tecoopsKvCacheConfig_t *cache);

tecoopsStatus_t tecoopsReshapeAndCache(tecoopsHandle_t handle,
                                       const void *key, const void *value,
                                       const int64_t *slot_mapping,
                                       void *key_cache, void *value_cache,
                                       int num_tokens, int num_kv_heads, int head_size,
                                       int num_blocks, int block_size);

/*
 * flash_attention — paged, varlen, causal (bottom-right aligned), GQA attention
 * with softmax scale 1/sqrt(head_size).
 * Replaces reference tecoops.h:156-169 (teco/interface/ops/flash_attention.cpp:71-119).
 *   q_seq_lens, kv_seq_lens : DEVICE int32 [batch] (lengths, not offsets); q_len <= kv_len
 *   blockTableDesc/blockTable: int32 [batch, block_table_dim]
 *   qDataDesc/qData, oDataDesc/oData : [sum(q_len), num_heads, head_size]
 *   k/vCacheDesc, k/vCache : [num_blocks, num_kv_heads, block_size, head_size]
 *   dtype: TECOOPS_DATA_HALF (reference) or TECOOPS_DATA_BFLOAT16 (extension)
 *   max_seqlen_q == 1 selects the split-KV decode kernel; anything else the
 *   tcgen05 prefill kernel (chunked and mixed batches included).
 *   workspace: optional device scratch of at least
 *   tecoopsGetFlashAttentionWorkspaceSize() bytes; nullptr makes the handle
 *   allocate (and keep) its own scratch on first use.
 */
tecoopsStatus_t tecoopsFlashAttention(tecoopsHandle_t handle,
                                      int max_seqlen_q, int max_seqlen_k,
                                      int max_block_num, const int *q_seq_lens,
                                      const int *kv_seq_lens,
                                      const tecoopsTensorDescriptor_t blockTableDesc,
                                      const void *blockTable,
                                      const tecoopsTensorDescriptor_t qDataDesc,
                                      const void *qData,
                                      const tecoopsTensorDescriptor_t kCacheDesc,
                                      const void *kCache,
                                      const tecoopsTensorDescriptor_t vCacheDesc,
                                      const void *vCache,
                                      const tecoopsTensorDescriptor_t oDataDesc,
                                      void *oData, void *workspace);

/*
 * Extension: the flags the reference's Python binding accepts and ignores
 * (api/torch_ext.cpp:99-113: softmax_scale, causal, window_size,
 * return_softmax_lse), honoured.  For query row i of a sequence with q_len L
 * and kv_len S (off = S - L), key j is admissible when
 *   j <= off + i              (causal != 0; the reference's only mode)
 *   j <= off + i + right      (causal == 0, window_right >= 0)
 *   j >= off + i - left       (window_left >= 0)
 * and j < S; negative window sides are unbounded (flash-attn convention).
 * softmax_scale <= 0 selects 1/sqrt(head_size).  Rows with no admissible key
 * are written as zeros (log-sum-exp -inf).
 */
typedef struct tecoopsFlashAttentionOptions {
    float softmax_scale;
    int causal;
    int window_left;
    int window_right;
    /* cache storage: layout (the cache descriptors' dims follow it) and, for a
       TECOOPS_DATA_FLOAT8_E4M3 cache (descriptor dtype), the dequantisation scales */
    int kv_layout;
    float k_scale;
    float v_scale;
} tecoopsFlashAttentionOptions_t;

/*
 * tecoopsFlashAttention with options (nullptr = the reference's behaviour:
 * causal, no window, scale 1/sqrt(head_size)) and an optional fp32 output
 * softmax_lse [num_heads, sum(q_len)] of natural-log log-sum-exp values of the
 * scaled, masked scores (nullptr: not written).  Same kernels and workspace.
 */
tecoopsStatus_t tecoopsFlashAttentionEx(tecoopsHandle_t handle,
                                        int max_seqlen_q, int max_seqlen_k,
                                        int max_block_num, const int *q_seq_lens,
                                        const int *kv_seq_lens,
                                        const tecoopsTensorDescriptor_t blockTableDesc,
                                        const void *blockTable,
                                        const tecoopsTensorDescriptor_t qDataDesc,
                                        const void *qData,
                                        const tecoopsTensorDescriptor_t kCacheDesc,
                                        const void *kCache,
                                        const tecoopsTensorDescriptor_t vCacheDesc,
                                        const void *vCache,
                                        const tecoopsTensorDescriptor_t oDataDesc,
                                        void *oData, void *workspace,
                                        const tecoopsFlashAttentionOptions_t *options,
                                        float *softmax_lse);

/*
 * Extension: one decode step's tecoopsReshapeAndCache + tecoopsFlashAttention in
 * one launch (reference reshape_and_cache_fp16.scpp:47-96 followed by
 * flash_attention.scpp:237-245 with q_len 1).  Every sequence has q_len 0 or 1;
 * row t of key/value ([sum(q_len), num_kv_heads, head_size], the cache dtype) is
 * the new token of the sequence whose query is row t, stored at cache slot
 * slot_mapping[t] (int64, -1 = skip) and attended at position kv_len - 1
 * (kv_seq_lens count the new token).  Results equal tecoopsReshapeAndCache
 * followed by tecoopsFlashAttention(max_seqlen_q = 1) when slot_mapping[t] is
 * the slot of position kv_len - 1 in the block table.  Shapes outside the
 * split-KV kernel run the two operators back to back.
 */
tecoopsStatus_t tecoopsReshapeAndCacheFlashAttentionDecode(
    tecoopsHandle_t handle, const void *key, const void *value, const int64_t *slot_mapping,
    int max_seqlen_k, const int *q_seq_lens, const int *kv_seq_lens,
    const tecoopsTensorDescriptor_t blockTableDesc, const void *blockTable,
    const tecoopsTensorDescriptor_t qDataDesc, const void *qData,
    const tecoopsTensorDescriptor_t kCacheDesc, void *kCache,
    const tecoopsTensorDescriptor_t vCacheDesc, void *vCache,
    const tecoopsTensorDescriptor_t oDataDesc, void *oData, void *workspace);

/*
 * Extension (no counterpart in the reference, whose `workspace` is always
 * nullptr): bytes of device scratch tecoopsFlashAttention needs for these
 * shapes, so that a caller can pass its own `workspace`.
 */
tecoopsStatus_t tecoopsGetFlashAttentionWorkspaceSize(tecoopsHandle_t handle,
                                                      int max_seqlen_q, int max_seqlen_k,
                                                      const tecoopsTensorDescriptor_t blockTableDesc,
                                                      const tecoopsTensorDescriptor_t qDataDesc,
                                                      const tecoopsTensorDescriptor_t kCacheDesc,
                                                      size_t *workspace_bytes);

/*
 * Extension with no counterpart in the reference: the split-KV decode of
 * tecoopsFlashAttention for callers that cannot allocate device memory, such as an
 * engine plugin that is handed only its input and output buffers, or a server
 * whose memory planner forbids allocations after start-up.  It allocates nothing:
 * the split scratch is a static 16 MiB device array inside the library (minus 256
 * bytes for its error word); shapes whose split plan needs more are rejected with
 * TECOOPS_STATUS_NOT_SUPPORTED.  A GPU holds the array from the first call on that
 * device (CUDA loads the library's device code lazily) until the process exits, so
 * make one warm-up call per device at start-up, before carving up the memory pool
 * and before any stream capture; that first call also looks up the array's device
 * address.  All calls share the array: calls that overlap on the GPU race and must
 * be serialised.  Preconditions: the calling thread's current device is the
 * handle's; q has at most one row per sequence (BAD_PARAM otherwise) and every
 * q_seq_lens entry is 0 or 1 (a larger one is reported as 0x1400 by
 * tecoopsGetDeviceErrorStatus, which also reports waits that gave up).
 * Arguments as tecoopsFlashAttention (max_seqlen_q is implicitly 1, no workspace);
 * results are identical to it for the same inputs.
 */
tecoopsStatus_t tecoopsFlashAttentionDecodeNoAlloc(tecoopsHandle_t handle, int max_seqlen_k,
                                                   const int *q_seq_lens, const int *kv_seq_lens,
                                                   const tecoopsTensorDescriptor_t blockTableDesc,
                                                   const void *blockTable,
                                                   const tecoopsTensorDescriptor_t qDataDesc,
                                                   const void *qData,
                                                   const tecoopsTensorDescriptor_t kCacheDesc,
                                                   const void *kCache,
                                                   const tecoopsTensorDescriptor_t vCacheDesc,
                                                   const void *vCache,
                                                   const tecoopsTensorDescriptor_t oDataDesc,
                                                   void *oData);

/*
 * Extension: status of the last device-side checks of this handle's stream.
 * Synchronises the handle's stream.  Returns TECOOPS_STATUS_INTERNAL_ERROR if a
 * kernel reported an error since the previous call (and clears it),
 * TECOOPS_STATUS_SUCCESS otherwise; *error_code receives the first code found:
 *   0x1nn-0xann  tcgen05 prefill: a bounded wait gave up (site in the high byte)
 *   0xb00        tcgen05 prefill: a q_seq_lens entry exceeds max_seqlen_q (rows past
 *                the planned work units were not computed)
 *   0x11nn       split-KV decode: the producer's wait for a free ring stage gave up
 *   0x12nn       split-KV decode: a consumer's wait for a loaded chunk gave up
 *   0x1300       split-KV decode: a kv_seq_lens entry exceeds max_seqlen_k (the keys
 *                past the planned splits were not attended)
 *   0x1400       split-KV decode: a q_seq_lens entry exceeds 1 (only the sequence's
 *                first query row was computed)
 * Reads the handle's own error word and, on the handle's device, the one of
 * tecoopsFlashAttentionDecodeNoAlloc.
 */
tecoopsStatus_t tecoopsGetDeviceErrorStatus(tecoopsHandle_t handle, int *error_code);

/*
 * Extension for tests of the failure path: sets the limit of every bounded device
 * wait of the split-KV decode kernel launched through this handle (default
 * 2,000,000,000 ns; 0 is BAD_PARAM).  stall_test != 0 makes the first ring wait of
 * each consumer warp wait on a barrier that nothing completes, so that the wait runs
 * out after limit_ns (and with it the producer's wait for the stage that consumer
 * holds); the first wait to give up records its site (0x12nn or 0x11nn), and the
 * kernel drains its copies and returns; the host then reads the code with
 * tecoopsGetDeviceErrorStatus.
 * Nothing faults, traps or waits without a bound.  stall_test = 0 restores normal
 * operation.
 */
tecoopsStatus_t tecoopsSetDeviceWaitLimit(tecoopsHandle_t handle, unsigned long long limit_ns,
                                          int stall_test);

/*
 * rms_norm — RMSNorm, optionally fused with the residual add (the step before the
 * QKV projection that feeds reshape_and_cache / flash_attention).
 * Replaces reference tecoops.h rms_norm (teco/interface/ops/rms_norm.cpp).
 *   input, output            : [num_tokens, hidden_size] fp16
 *   weight                   : [hidden_size]
 *   residual, residual_out   : [num_tokens, hidden_size] or nullptr (both or neither
 *                              are used: residual_out = input + residual)
 *   y = h * rstd * weight, rstd = 1 / sqrt(mean(h^2) + eps), h = input (+ residual)
 * fp32 arithmetic; with a residual the sum of squares uses the unrounded h and the
 * output the rounded residual_out, as the reference kernel does.
 */
tecoopsStatus_t tecoopsRmsNorm(tecoopsHandle_t handle, const void *input, const void *weight,
                               const void *residual, void *output, void *residual_out,
                               int num_tokens, int hidden_size, float eps);
/* Extension: the same for TECOOPS_DATA_HALF or TECOOPS_DATA_BFLOAT16 tensors. */
tecoopsStatus_t tecoopsRmsNormEx(tecoopsHandle_t handle, const void *input, const void *weight,
                                 const void *residual, void *output, void *residual_out,
                                 int num_tokens, int hidden_size, float eps,
                                 tecoopsDataType_t dtype);

/* ---- reference operators off this path: exported, NOT_SUPPORTED ---- */
tecoopsStatus_t tecoopsFlattenRays(tecoopsHandle_t handle, const int *rays, uint32_t N,
                                   uint32_t M, int *res, tecoopsAlgo_t algo);
tecoopsStatus_t tecoopsReduceVariance(const tecoopsHandle_t handle, int axis, int correction,
                                      const tecoopsTensorDescriptor_t xDesc, const void *x,
                                      const tecoopsTensorDescriptor_t yDesc, void *y);
tecoopsStatus_t tecoopsMorton3DInvert(tecoopsHandle_t handle, const int *indices, uint32_t N,
                                      int *coords);
tecoopsStatus_t tecoopsCausalConv1d(tecoopsHandle_t handle, int batch, int totalSeqLen,
                                    int dim, int width, int convStateStride, int xSeqStride,
                                    int outSeqStride, int padSlotId, int api_mode, int actMode,
                                    const void *x, void *convState, const void *weight,
                                    void *out, const int *queryStartLoc,
                                    const int *convStateIndices,
                                    const int8_t *hasInitialState);

#ifdef __cplusplus
}
#endif

#endif /* TECOOPS_B200_INCLUDE_TECOOPS_H_ */
