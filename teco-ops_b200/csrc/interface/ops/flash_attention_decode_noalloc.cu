// tecoopsFlashAttentionDecodeNoAlloc: the split-KV decode path for callers that
// cannot allocate device memory.
//
// Some callers cannot call cudaMalloc at the point where they run attention.
// One example is an inference-engine plugin whose Enqueue receives only the
// input and output buffers from the engine (the reference's plugin passes
// workspace = nullptr).  Another is a serving loop whose memory planner forbids
// allocations after start-up, because cudaMalloc synchronises the device and can
// fail once the pool is carved up.  tecoopsFlashAttention would then fall back
// to the handle's lazily grown scratch, and that fallback calls cudaMalloc.
//
// This entry point runs the same split-KV decode kernels with the same split
// plan.  Its scratch lives in a file-scope __device__ array of
// kNoAllocScratchBytes (16 MiB): the first 256 bytes hold the error word that the
// kernels set when a bounded wait gives up or a length breaks the decode
// preconditions, the rest the per-split partial outputs and log-sum-exp values.
// A GPU holds the array from the moment this library's device code is loaded on
// it until the process exits.  With CUDA's lazy module loading (the default since
// CUDA 12.2) that moment is the first call of this entry point on the device, so
// the 16 MiB are reserved by that call: make one warm-up call per device at
// start-up, before the caller carves up its memory pool and before any stream
// capture.
//
// Host code cannot use the array's name as a device address: in host code the
// symbol is only a stand-in.  So the array's device address is looked up with
// cudaGetSymbolAddress, once per device with that device current, on the first
// call made on that device.
//
// All calls share the one array, and it keeps the contents of the last call.
// The partials need no clearing: every partial is written before it is read
// within the same call.  The error word starts at zero (static device memory is
// zero-initialised) and tecoopsGetDeviceErrorStatus clears it after reporting it.
// Calls that overlap on the GPU (for example on two streams of one device at
// once) race on the array; serialise them.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "interface/common/context.h"
#include "tecoops.h"
#include "ual/com/log.h"
#include "ual/kernels/launchers.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;   // 16 MiB per device
constexpr size_t kErrorBytes = 256;                   // error word, then the partials
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void *g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_decode_scratch on `device` (which must be current).
// Looked up once per device; returns nullptr if the lookup fails.
void *scratchFor(int device) {
    if (device < 0 || device >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_ptr[device] == nullptr) {
        void *ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
        if (e != cudaSuccess) {
            TECO_ERROR("tecoopsFlashAttentionDecodeNoAlloc: cudaGetSymbolAddress failed on device "
                       "%d: %s",
                       device, cudaGetErrorString(e));
            cudaGetLastError();
            return nullptr;
        }
        g_scratch_ptr[device] = ptr;
    }
    return g_scratch_ptr[device];
}

}  // namespace

namespace tecoops {
namespace interface {

// The error word of this entry point on `device`, or nullptr if no call has set the
// array up on that device yet (then no kernel of this entry point can have set it).
int *noAllocErrorWord(int device) {
    if (device < 0 || device >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    return static_cast<int *>(g_scratch_ptr[device]);
}

}  // namespace interface
}  // namespace tecoops

namespace {

bool packedDesc(const tecoopsTensorStruct *d) {
    int s = 1;
    for (int i = d->nbDims - 1; i >= 0; --i) {
        if (d->strideA[i] != s) return false;
        s *= d->dimA[i];
    }
    return true;
}

}  // namespace

extern "C" tecoopsStatus_t tecoopsFlashAttentionDecodeNoAlloc(
    tecoopsHandle_t handle, int max_seqlen_k, const int *q_seq_lens, const int *kv_seq_lens,
    const tecoopsTensorDescriptor_t blockTableDesc, const void *blockTable,
    const tecoopsTensorDescriptor_t qDataDesc, const void *qData,
    const tecoopsTensorDescriptor_t kCacheDesc, const void *kCache,
    const tecoopsTensorDescriptor_t vCacheDesc, const void *vCache,
    const tecoopsTensorDescriptor_t oDataDesc, void *oData) {
    if (handle == nullptr) return TECOOPS_STATUS_NOT_INITIALIZED;
    const tecoopsTensorStruct *bt = blockTableDesc, *q = qDataDesc, *k = kCacheDesc,
                              *v = vCacheDesc, *o = oDataDesc;
    if (!bt || !q || !k || !v || !o || !q_seq_lens || !kv_seq_lens || !blockTable || !qData ||
        !kCache || !vCache || !oData || max_seqlen_k < 0)
        return TECOOPS_STATUS_BAD_PARAM;
    if (k->dataType != v->dataType ||
        (k->dataType != TECOOPS_DATA_HALF && k->dataType != TECOOPS_DATA_BFLOAT16) ||
        q->dataType != k->dataType || o->dataType != k->dataType ||
        bt->dataType != TECOOPS_DATA_INT32)
        return TECOOPS_STATUS_BAD_PARAM;
    if (k->nbDims != 4 || v->nbDims != 4 || q->nbDims != 3 || o->nbDims != 3 || bt->nbDims != 2)
        return TECOOPS_STATUS_BAD_PARAM;
    for (int i = 0; i < 4; ++i)
        if (k->dimA[i] != v->dimA[i]) return TECOOPS_STATUS_BAD_PARAM;
    for (int i = 0; i < 3; ++i)
        if (q->dimA[i] != o->dimA[i]) return TECOOPS_STATUS_BAD_PARAM;
    if (q->dimA[2] != k->dimA[3] || q->dimA[1] <= 0 || k->dimA[1] <= 0 ||
        q->dimA[1] % k->dimA[1] != 0 || bt->dimA[0] <= 0 || bt->dimA[1] <= 0 ||
        k->dimA[0] <= 0 || k->dimA[2] <= 0)
        return TECOOPS_STATUS_BAD_PARAM;
    if (!packedDesc(q) || !packedDesc(o) || !packedDesc(k) || !packedDesc(v) || !packedDesc(bt))
        return TECOOPS_STATUS_NOT_SUPPORTED;
    // the split-KV kernel reads q in 32-bit words and the caches by TMA (16-byte aligned)
    const uintptr_t al = reinterpret_cast<uintptr_t>(qData) | reinterpret_cast<uintptr_t>(oData) |
                         reinterpret_cast<uintptr_t>(kCache) | reinterpret_cast<uintptr_t>(vCache);
    if (al & 15u) {
        TECO_ERROR("tecoopsFlashAttentionDecodeNoAlloc: q, out and the caches must be 16-byte "
                   "aligned");
        return TECOOPS_STATUS_NOT_SUPPORTED;
    }
    const int batch = bt->dimA[0], heads = q->dimA[1], kv_heads = k->dimA[1];
    const int head_dim = q->dimA[2], block_size = k->dimA[2];
    const int group = heads / kv_heads;
    if (!tecoops::kern::decode_supported(head_dim, block_size, group) || batch > 65535 ||
        kv_heads * ((group + 15) / 16) > 65535) {
        TECO_ERROR("tecoopsFlashAttentionDecodeNoAlloc: head_dim %d / block_size %d / batch %d "
                   "not covered by the split-KV decode kernel",
                   head_dim, block_size, batch);
        return TECOOPS_STATUS_NOT_SUPPORTED;
    }
    // decode precondition: at most one query row per sequence (every q_seq_lens[b] is 0
    // or 1; a length above 1 is reported through the error word)
    if (q->dimA[0] > batch) {
        TECO_ERROR("tecoopsFlashAttentionDecodeNoAlloc: q has %d rows for %d sequences; decode "
                   "takes at most one query row per sequence",
                   q->dimA[0], batch);
        return TECOOPS_STATUS_BAD_PARAM;
    }

    tecoops::kern::DecodeParams p;
    p.q = qData;
    p.key_cache = kCache;
    p.value_cache = vCache;
    p.out = oData;
    p.q_seq_lens = q_seq_lens;
    p.kv_seq_lens = kv_seq_lens;
    p.block_table = static_cast<const int *>(blockTable);
    p.batch = batch;
    p.num_heads = heads;
    p.num_kv_heads = kv_heads;
    p.group = group;
    p.num_slices = (group + 15) / 16;
    p.head_dim = head_dim;
    p.block_size = block_size;
    p.block_table_dim = bt->dimA[1];
    p.num_pages = k->dimA[0];
    p.total_q = q->dimA[0];
    tecoops::kern::decode_plan(handle->num_sms, batch, kv_heads, group, max_seqlen_k,
                               &p.split_tokens, &p.max_splits);
    p.scale_log2 = (float)(1.0 / std::sqrt((double)head_dim)) * 1.4426950408889634f;
    p.part_o = nullptr;
    p.part_lse = nullptr;
    p.dev_error = nullptr;   // set below to the array's error word
    p.wait_limit_ns = handle->wait_limit_ns;
    p.stall_test = handle->stall_test;
    p.window_left = -1;
    p.lse = nullptr;
    p.new_key = nullptr;
    p.new_value = nullptr;
    p.slot_mapping = nullptr;
    p.kv_layout = 0;
    p.cache_fp8 = 0;
    p.v_scale = 1.f;
    const size_t need =
        tecoops::kern::decode_workspace_bytes(batch, heads, head_dim, p.max_splits);
    if (need > kNoAllocScratchBytes - kErrorBytes) {
        TECO_ERROR("tecoopsFlashAttentionDecodeNoAlloc: these shapes need %zu bytes of split "
                   "scratch; the static scratch holds %zu bytes (16 MiB). Use "
                   "tecoopsFlashAttention with a workspace instead.",
                   need, kNoAllocScratchBytes);
        return TECOOPS_STATUS_NOT_SUPPORTED;
    }
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess) return TECOOPS_STATUS_INTERNAL_ERROR;
    if (device != handle->device) {
        TECO_ERROR("tecoopsFlashAttentionDecodeNoAlloc: the current device %d is not the "
                   "handle's device %d",
                   device, handle->device);
        return TECOOPS_STATUS_BAD_PARAM;
    }
    unsigned char *scratch = static_cast<unsigned char *>(scratchFor(device));
    if (scratch == nullptr) return TECOOPS_STATUS_INTERNAL_ERROR;
    p.dev_error = reinterpret_cast<int *>(scratch);
    if (p.max_splits > 1) {
        const size_t recs = (size_t)batch * heads * p.max_splits;
        p.part_o = reinterpret_cast<float *>(scratch + kErrorBytes);
        p.part_lse = p.part_o + recs * head_dim;
    }
    const cudaError_t e =
        tecoops::kern::launch_decode(p, k->dataType == TECOOPS_DATA_BFLOAT16, handle->stream);
    if (e != cudaSuccess) {
        TECO_ERROR("tecoopsFlashAttentionDecodeNoAlloc: launch failed: %s", cudaGetErrorString(e));
        return TECOOPS_STATUS_INTERNAL_ERROR;
    }
    return TECOOPS_STATUS_SUCCESS;
}
