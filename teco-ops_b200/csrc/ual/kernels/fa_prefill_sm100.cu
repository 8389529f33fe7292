// Causal varlen paged prefill attention on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), sm_100a.
//
// Semantics: reference kernel teco/ual/kernel/flash_attention/flash_attention.scpp:179-416
// as pinned by its golden test/zoo/teco/flash_attention/flash_attention.py:79-140:
//   for each sequence b (q_len L, kv_len S, L <= S) and q head h:
//     O[i] = softmax_j( Q[i] . K[j] / sqrt(D) , j <= S - L + i ) . V
//   with K/V read from the paged cache [pages, Hkv, block_size, D] through
//   block_table[b][j / block_size], kv head h / (Hq / Hkv).
//
// B200 design (one CTA = one 128-row Q tile of one q head):
//   warp 0      TMA producer: Q tile once, then K/V tiles of 128 tokens assembled
//               from 128/block_size page boxes of the 4-D cache tensor map (the page
//               id is a TMA coordinate, so the gather costs nothing extra); 2-stage
//               ring; pages past kv_len use an out-of-range page coordinate so TMA
//               zero-fills them.  128-byte swizzle, 64-column boxes.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer:
//                 S_j = Q K_j^T   (SS form, M=128, N=128, K=D, fp32 in TMEM, 2 buffers)
//                 O  += P_j V_j   (TS form: P bf16/fp16 from TMEM, V MN-major in smem)
//   warps 4-7   softmax: thread r owns row r = TMEM lane r; loads S with
//               tcgen05.ld, masks (bottom-right causal + kv_len tail), online softmax in
//               the exp2 domain with a lazy O rescale (only when the running max grows
//               by more than 2^8), writes P back to TMEM with tcgen05.st, and runs the
//               epilogue O / l -> global.
// TMEM columns: S0 [0,128) S1 [128,256) P0 [256,320) P1 [320,384) O [384,384+D).
// Every mbarrier wait is bounded (~2 s); a wait that gives up records its site in
// the device error word and the CTA drains its MMAs, frees TMEM and exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <type_traits>

#include "ual/kernels/common.cuh"
#include "ual/kernels/launchers.h"
#include "ual/kernels/sm100_primitives.cuh"

namespace tecoops {
namespace kern {

using namespace sm100;

namespace {

constexpr int kBM = 128;        // Q rows per tile
constexpr int kBN = 128;        // KV tokens per tile
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;
constexpr uint32_t kColP = 256;
constexpr uint32_t kColO = 384;

template <int D>
struct PrefillSmem {
    static constexpr int kHalves = D / 64;
    static constexpr int kHalfBytes = 128 * 128;              // 128 rows x 128 B
    static constexpr int kTileBytes = kHalves * kHalfBytes;   // Q, K or V tile
    static constexpr int kQ = 0;
    static constexpr int kK0 = kTileBytes;
    static constexpr int kV0 = kK0 + 2 * kTileBytes;
    static constexpr int kBytes = kV0 + 2 * kTileBytes;
    static constexpr int kAlloc = kBytes + 1024;   // slack for 1024-byte alignment
};

struct PrefillParams {
    const int *q_seq_lens;
    const int *kv_seq_lens;
    const int *block_table;
    void *out;
    int *dev_error;
    int num_heads;
    int num_kv_heads;
    int group;
    int block_size;
    int rows_per_box;   // min(block_size, 128)
    int block_table_dim;
    int num_pages;
    int num_qtiles;     // ceil(max_q / 128)
    int total_q;
    float scale_log2;
};

enum WaitSite : int {
    kSiteQ = 0x100, kSiteK = 0x200, kSiteV = 0x300, kSiteEmpty = 0x400, kSiteS = 0x500,
    kSiteP = 0x600, kSiteO = 0x700, kSiteDrain = 0x800, kSiteVz = 0x900
};

}  // namespace

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    fa_prefill_sm100_kernel(const __grid_constant__ CUtensorMap qmap,
                            const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap, PrefillParams p) {
    using Sm = PrefillSmem<D>;
    constexpr bool kBF16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[16];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;

    const int h = blockIdx.x;
    const int b = blockIdx.y;
    const int qt = p.num_qtiles - 1 - (int)blockIdx.z;   // heaviest tiles launch first
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const int L = __ldg(p.q_seq_lens + b);
    const int S = __ldg(p.kv_seq_lens + b);
    const int q0 = qt * kBM;
    if (q0 >= L) return;   // uniform: tile beyond this sequence
    const int rows_valid = min(kBM, L - q0);
    const int off = S - L;                                   // bottom-right causal offset
    const int kv_hi = min(S, off + q0 + rows_valid);         // exclusive key bound of tile
    const int n_tiles = kv_hi > 0 ? (kv_hi + kBN - 1) / kBN : 0;
    const int kvh = h / p.group;

    // 1024-byte aligned dynamic smem base
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t sbase = (raw_base + 1023u) & ~1023u;
    uint8_t *sgen = smem_raw + (sbase - raw_base);

    const uint32_t bar0 = smem_u32(&bars[0]);
    auto BAR = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
    // barrier ids
    constexpr int Q_FULL = 0, K_FULL = 1, V_FULL = 3, KV_EMPTY = 5, S_FULL = 7, P_FULL = 9,
                  O_DONE = 11, DRAIN = 12;

    if (n_tiles == 0) {
        // no admissible key for any row (q_len > kv_len): write zeros
        if (warp >= 4) {
            const int r = threadIdx.x - 128;
            const int qs = warp_seq_start(p.q_seq_lens, b);
            if (r < rows_valid && qs + q0 + r < p.total_q) {
                T *o = static_cast<T *>(p.out) + ((int64_t)(qs + q0 + r) * p.num_heads + h) * D;
                for (int d = 0; d < D; ++d) o[d] = Elem<T>::from_float(0.f);
            }
        }
        return;
    }

    if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(BAR(Q_FULL), 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(BAR(K_FULL + s), 1);
            mbar_init(BAR(V_FULL + s), 1);
            mbar_init(BAR(KV_EMPTY + s), 1);
            mbar_init(BAR(S_FULL + s), 1);
            mbar_init(BAR(P_FULL + s), 128);
        }
        mbar_init(BAR(O_DONE), 1);
        mbar_init(BAR(DRAIN), 1);
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    volatile int *abortp = &abort_flag;

    if (warp == 0) {
        // ===================== TMA producer =====================
        const int qs = warp_seq_start(p.q_seq_lens, b);
        if (lane == 0) {
            tma_prefetch_desc(&qmap);
            tma_prefetch_desc(&kmap);
            tma_prefetch_desc(&vmap);
            mbar_arrive_expect_tx(BAR(Q_FULL), Sm::kTileBytes);
#pragma unroll
            for (int hh = 0; hh < Sm::kHalves; ++hh)
                tma_load_3d(sbase + Sm::kQ + hh * Sm::kHalfBytes, &qmap, BAR(Q_FULL), hh * 64, h,
                            qs + q0);
        }
        const int rpb = p.rows_per_box;
        const int nbox = kBN / rpb;
        const int *bt = p.block_table + (int64_t)b * p.block_table_dim;
        int issued[2] = {0, 0};
        for (int j = 0; j < n_tiles; ++j) {
            const int s = j & 1;
            if (j >= 2 && !mbar_wait_bounded(BAR(KV_EMPTY + s), ((j >> 1) - 1) & 1, abortp,
                                             p.dev_error, kSiteEmpty + j))
                break;
            int blk = p.num_pages, row = 0;
            if (lane < nbox) {
                const int tok = j * kBN + lane * rpb;
                const int pi = tok / p.block_size;
                row = tok - pi * p.block_size;
                if (tok < S && pi < p.block_table_dim) blk = __ldg(bt + pi);
                if (blk < 0 || blk >= p.num_pages) blk = p.num_pages;   // out of range -> zeros
            }
            if (lane == 0) {
                mbar_arrive_expect_tx(BAR(K_FULL + s), Sm::kTileBytes);
                mbar_arrive_expect_tx(BAR(V_FULL + s), Sm::kTileBytes);
            }
            __syncwarp();
            if (lane < nbox) {
                const uint32_t kdst = sbase + Sm::kK0 + s * Sm::kTileBytes + lane * rpb * 128;
                const uint32_t vdst = sbase + Sm::kV0 + s * Sm::kTileBytes + lane * rpb * 128;
#pragma unroll
                for (int hh = 0; hh < Sm::kHalves; ++hh) {
                    tma_load_4d(kdst + hh * Sm::kHalfBytes, &kmap, BAR(K_FULL + s), hh * 64, row,
                                kvh, blk);
                    tma_load_4d(vdst + hh * Sm::kHalfBytes, &vmap, BAR(V_FULL + s), hh * 64, row,
                                kvh, blk);
                }
            }
            issued[s] = j + 1;
        }
        // on abort: let this warp's own copies in flight land before the CTA exits
        if (*abortp && lane == 0) {
            for (int s = 0; s < 2; ++s) {
                if (issued[s] == 0) continue;
                const int j = issued[s] - 1;
                mbar_wait_bounded(BAR(K_FULL + s), (j >> 1) & 1, nullptr, nullptr, 0, 100000000ull);
                mbar_wait_bounded(BAR(V_FULL + s), (j >> 1) & 1, nullptr, nullptr, 0, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // ===================== MMA issuer (one thread) =====================
        if (lane == 0) {
            const uint32_t idesc_qk = idesc_f16(kBF16, false, kBM, kBN);
            const uint32_t idesc_pv = idesc_f16(kBF16, true, kBM, D);
            bool ok = mbar_wait_bounded(BAR(Q_FULL), 0, abortp, p.dev_error, kSiteQ);
            tc_fence_after();
            auto issue_pv = [&](int i) -> bool {
                const int s = i & 1;
                if (!mbar_wait_bounded(BAR(P_FULL + s), (i >> 1) & 1, abortp, p.dev_error,
                                       kSiteP + i))
                    return false;
                if (!mbar_wait_bounded(BAR(V_FULL + s), (i >> 1) & 1, abortp, p.dev_error,
                                       kSiteV + i))
                    return false;
                tc_fence_after();
                const uint32_t vbase = sbase + Sm::kV0 + s * Sm::kTileBytes;
#pragma unroll
                for (int t = 0; t < kBN / 16; ++t) {
                    const uint64_t bdesc =
                        smem_desc_sw128(vbase + t * 16 * 128, Sm::kHalfBytes, 1024);
                    tc_mma_ts(tmem + kColO, tmem + kColP + s * 64 + t * 8, bdesc, idesc_pv,
                              (i > 0 || t > 0) ? 1u : 0u);
                }
                tc_commit(BAR(O_DONE));
                tc_commit(BAR(KV_EMPTY + s));
                return true;
            };
            for (int j = 0; ok && j < n_tiles; ++j) {
                const int s = j & 1;
                if (!mbar_wait_bounded(BAR(K_FULL + s), (j >> 1) & 1, abortp, p.dev_error,
                                       kSiteK + j)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t kbase = sbase + Sm::kK0 + s * Sm::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t koff = (kk >> 2) * Sm::kHalfBytes + (kk & 3) * 32;
                    const uint64_t adesc = smem_desc_sw128(sbase + Sm::kQ + koff, 16, 1024);
                    const uint64_t bdesc = smem_desc_sw128(kbase + koff, 16, 1024);
                    tc_mma_ss(tmem + kColS + s * 128, adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
                }
                tc_commit(BAR(S_FULL + s));
                if (j >= 1 && !issue_pv(j - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok) issue_pv(n_tiles - 1);
            // drain: every MMA issued by this thread has completed before TMEM is freed
            tc_commit(BAR(DRAIN));
            mbar_wait_bounded(BAR(DRAIN), 0, nullptr, p.dev_error, kSiteDrain);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ===================== softmax + epilogue (one row per thread) =====================
        const int r = threadIdx.x - 128;
        const uint32_t lane_addr = (uint32_t)(32 * (warp & 3)) << 16;
        const int qi = q0 + r;
        const int lim = off + qi;   // last admissible key of this row (inclusive)
        const float sl2 = p.scale_log2;
        const int qs = warp_seq_start(p.q_seq_lens, b);
        float m_s = -INFINITY;       // running max in scaled (log2) units
        float l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_tiles && ok; ++j) {
            const int s = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(BAR(S_FULL + s), (j >> 1) & 1, abortp, p.dev_error,
                                   kSiteS + j))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float x[kBN];
            {
                uint32_t u[32];
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c) {
                    tmem_ld32(tmem + lane_addr + kColS + s * 128 + c * 32, u);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(u[e]);
                }
            }
            const int kbase = j * kBN;
            const int klim = min(lim, S - 1);   // inclusive admissible bound
            if (kbase + kBN - 1 > klim) {
#pragma unroll
                for (int c = 0; c < kBN; ++c)
                    if (kbase + c > klim) x[c] = -INFINITY;
            }
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < kBN; ++c) mx = fmaxf(mx, x[c]);
            const float m_new = fmaxf(m_s, mx * sl2);
            const bool need = (j == 0) || (m_new > m_s + 8.0f);
            const bool warp_need = __any_sync(0xffffffffu, need);
            float alpha = 1.f;
            if (warp_need) {
                alpha = (m_s == -INFINITY) ? 0.f : fast_exp2(m_s - m_new);
                m_s = m_new;
            }
            const float m_use = (m_s == -INFINITY) ? 0.f : m_s;
            float rs = 0.f;
            uint32_t pk[kBN / 2];
#pragma unroll
            for (int c = 0; c < kBN; c += 2) {
                const float p0 = fast_exp2(fmaf(x[c], sl2, -m_use));
                const float p1 = fast_exp2(fmaf(x[c + 1], sl2, -m_use));
                rs += p0 + p1;
                pk[c / 2] = Elem<T>::pack2(p0, p1);
            }
            l = l * alpha + rs;

            if (j >= 1) {
                // PV_{j-1} complete: O is stable and P buffer s is free
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(BAR(O_DONE), (j - 1) & 1, abortp, p.dev_error,
                                       kSiteO + j))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (warp_need) {
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t u[32];
                        const uint32_t a = tmem + lane_addr + kColO + c * 32;
                        tmem_ld32(a, u);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
                        tmem_st32(a, u);
                    }
                }
            }
            if (j == n_tiles - 1 && kbase + kBN > S) {
                // rows of the last V tile past kv_len may hold arbitrary bits: zero them
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(BAR(V_FULL + s), (j >> 1) & 1, abortp, p.dev_error,
                                       kSiteVz))) {
                    ok = false;
                    break;
                }
                if (kbase + r >= S) {
                    uint8_t *vrow = sgen + Sm::kV0 + s * Sm::kTileBytes + r * 128;
#pragma unroll
                    for (int hh = 0; hh < Sm::kHalves; ++hh) {
                        uint4 *q4 = reinterpret_cast<uint4 *>(vrow + hh * Sm::kHalfBytes);
#pragma unroll
                        for (int e = 0; e < 8; ++e) q4[e] = make_uint4(0, 0, 0, 0);
                    }
                }
                fence_proxy_async_smem();
            }
            {
                uint32_t u[32];
#pragma unroll
                for (int c = 0; c < kBN / 64; ++c) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) u[e] = pk[c * 32 + e];
                    tmem_st32(tmem + lane_addr + kColP + s * 64 + c * 32, u);
                }
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(BAR(P_FULL + s));
        }
        // epilogue
        if (__all_sync(0xffffffffu, ok && mbar_wait_bounded(BAR(O_DONE), (n_tiles - 1) & 1,
                                                            abortp, p.dev_error, kSiteO + 0xff))) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            T *orow = static_cast<T *>(p.out) + ((int64_t)(qs + qi) * p.num_heads + h) * D;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint32_t u[32];
                tmem_ld32(tmem + lane_addr + kColO + c * 32, u);
                tmem_ld_wait();
                if (r < rows_valid && qs + qi < p.total_q) {
                    uint32_t pkd[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        pkd[e] = Elem<T>::pack2(__uint_as_float(u[2 * e]) * inv,
                                                __uint_as_float(u[2 * e + 1]) * inv);
                    uint4 *dst = reinterpret_cast<uint4 *>(orow + c * 32);
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        dst[e] = make_uint4(pkd[4 * e], pkd[4 * e + 1], pkd[4 * e + 2],
                                            pkd[4 * e + 3]);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---- host side ------------------------------------------------------------------------

typedef CUresult (*PFN_encodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                    const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                    const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion,
                                    CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
    static PFN_encodeTiled fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled>(ptr);
    }
    return fn;
}

bool prefill_supported(int head_dim, int block_size, int group) {
    (void)group;
    if (head_dim != 64 && head_dim != 128) return false;
    if (block_size <= 0) return false;
    if (block_size <= 128) return block_size >= 8 && (128 % block_size) == 0;
    return (block_size % 128) == 0;
}

size_t prefill_workspace_bytes(const AttnShape &) { return 0; }

template <typename T, int D>
static cudaError_t launch_prefill_t(const AttnShape &s, int *dev_error, cudaStream_t stream) {
    PFN_encodeTiled enc = get_encode_fn();
    if (!enc) return cudaErrorNotSupported;
    const CUtensorMapDataType dt =
        std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap qmap, kmap, vmap;
    {
        cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)s.num_heads, (cuuint64_t)s.total_q};
        cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)s.num_heads * D * 2};
        cuuint32_t box[3] = {64, 1, 128};
        cuuint32_t es[3] = {1, 1, 1};
        if (enc(&qmap, dt, 3, const_cast<void *>(s.q), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    const int rpb = s.block_size < 128 ? s.block_size : 128;
    {
        cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)s.block_size,
                              (cuuint64_t)s.num_kv_heads, (cuuint64_t)s.num_pages};
        cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)s.block_size * D * 2,
                                 (cuuint64_t)s.num_kv_heads * s.block_size * D * 2};
        cuuint32_t box[4] = {64, (cuuint32_t)rpb, 1, 1};
        cuuint32_t es[4] = {1, 1, 1, 1};
        if (enc(&kmap, dt, 4, const_cast<void *>(s.key_cache), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
        if (enc(&vmap, dt, 4, const_cast<void *>(s.value_cache), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    PrefillParams p;
    p.q_seq_lens = s.q_seq_lens;
    p.kv_seq_lens = s.kv_seq_lens;
    p.block_table = s.block_table;
    p.out = s.out;
    p.dev_error = dev_error;
    p.num_heads = s.num_heads;
    p.num_kv_heads = s.num_kv_heads;
    p.group = s.num_heads / s.num_kv_heads;
    p.block_size = s.block_size;
    p.rows_per_box = rpb;
    p.block_table_dim = s.block_table_dim;
    p.num_pages = s.num_pages;
    p.num_qtiles = (s.max_q + kBM - 1) / kBM;
    p.total_q = s.total_q;
    p.scale_log2 = s.scale_log2;
    if (p.num_qtiles <= 0 || s.batch <= 0) return cudaSuccess;

    auto kfn = fa_prefill_sm100_kernel<T, D>;
    const int smem = PrefillSmem<D>::kAlloc;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid(s.num_heads, s.batch, p.num_qtiles);
    kfn<<<grid, kThreads, smem, stream>>>(qmap, kmap, vmap, p);
    return cudaGetLastError();
}

cudaError_t launch_prefill(const AttnShape &s, bool bf16, void *workspace, int *dev_error,
                           int num_sms, cudaStream_t stream) {
    (void)workspace;
    (void)num_sms;
    const uintptr_t a = reinterpret_cast<uintptr_t>(s.q) | reinterpret_cast<uintptr_t>(s.key_cache) |
                        reinterpret_cast<uintptr_t>(s.value_cache);
    if (a & 15u) return cudaErrorMisalignedAddress;
    if (s.head_dim == 128)
        return bf16 ? launch_prefill_t<__nv_bfloat16, 128>(s, dev_error, stream)
                    : launch_prefill_t<__half, 128>(s, dev_error, stream);
    if (s.head_dim == 64)
        return bf16 ? launch_prefill_t<__nv_bfloat16, 64>(s, dev_error, stream)
                    : launch_prefill_t<__half, 64>(s, dev_error, stream);
    return cudaErrorInvalidValue;
}

}  // namespace kern
}  // namespace tecoops
