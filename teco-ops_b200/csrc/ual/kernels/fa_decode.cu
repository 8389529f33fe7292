// Paged single-token decode attention for sm_100a (split-KV / flash-decoding).
//
// Semantics: the reference kernel teco/ual/kernel/flash_attention/flash_attention.scpp
// (179-416) with q_len == 1, as pinned by its golden
// test/zoo/teco/flash_attention/flash_attention.py:79-140: one query row per sequence
// attends to all kv_len cached tokens (bottom-right causal with L == 1), keys and
// values gathered page by page through block_table, scale 1/sqrt(D), GQA head
// h -> kv head h / (Hq/Hkv).
//
// B200 design (bandwidth-bound: ~4 FLOP per cache byte):
//  * one CTA per (sequence, KV head, 16-head Q slice, KV split).  All Q heads of
//    a GQA group are packed into the 16 rows of one warp MMA tile so every K/V
//    byte is read from HBM exactly once;
//  * the KV range of a sequence is cut into splits of `split_tokens` so that even
//    64 sequences fill 148 SMs;
//  * warp 4 is a TMA producer: each 16-token page chunk of K and V is one box (per
//    64 columns) of a 4-D tensor map over the paged cache, with the page id as a
//    coordinate (out-of-range ids read as zeros) and 128-byte swizzle, into a
//    mbarrier ring (8 stages and 3 CTAs per SM for 16-bit caches, 24 stages and
//    2 CTAs per SM for e4m3, so 192 KB of K and V in flight per SM); block-table ids
//    are fetched 32 chunks at a time and the chunks are issued 4 (8 for e4m3) at a
//    time, one per lane (a single issuing lane measured ~550 cycles per chunk and
//    left the consumers waiting);
//  * warps 0-3 consume chunks round-robin: QK^T and PV on the warp MMA
//    (m16n8k16, fp32 accumulate) fed by conflict-free ldmatrix on the swizzled
//    tiles, online softmax in the exp2 domain with the O rescale skipped when no
//    row max grows, P kept in registers as the A operand;
//  * the 4 warps merge through shared memory; a sequence that needs one split
//    writes its output directly, otherwise (O/l, log2-sum-exp) partials go to
//    the workspace and fa_decode_merge combines them.
//  * options: a left window (keys j >= kv_len - 1 - window_left) moves the first
//    split to the window's 16-token chunk and masks the keys before it; the
//    log-sum-exp (natural log) of each row is written when requested.
//  * fused reshape_and_cache (tecoopsReshapeAndCacheFlashAttentionDecode): the CTA of a
//    sequence's last split (Q slice 0) stores the new token's K/V row of its KV head
//    into the cache slot, and the consumer warp whose chunk holds position kv_len - 1
//    overwrites that row of the staged K/V tiles from the new key/value, so the
//    attention never depends on the ordering of the store and the TMA read of the
//    same slot; one launch replaces the scatter kernel + decode.
//  * cache layouts [pages, Hkv, bs, D] and [pages, bs, Hkv, D] differ only in the
//    tensor maps' strides.  An e4m3 cache (FP8) is loaded raw (half the bytes) into
//    the ring, swizzled at its row width; each consumer warp reads its chunk straight
//    into registers with conflict-free 16-byte loads, releases the ring stage at once
//    and converts the bytes into f16 MMA fragments (exact for e4m3).  The fragments
//    need no transposed load because two index orders are free: QK^T sums over the
//    head dimension, so lane (g, c) takes the D/4 contiguous bytes at (D/4)*c of a key
//    row (Q is loaded in the same order), and PV's output column n of n-tile nn is
//    stored as d = (D/8)*n + nn, so the lane takes D/8 contiguous bytes of four value
//    rows and pairs them with a byte permute.  k_scale is folded into the softmax
//    scale and v_scale into the output.
//  * a GQA group of at most 8 heads runs transposed: S^T = K Q^T puts the 16 tokens of
//    a chunk in the MMA rows and the (<= 8) heads in its 8 columns, and O^T += V^T P^T
//    (16-bit: K by ldmatrix, V^T by transposing ldmatrix; e4m3: output row
//    d = (D/16)*m + n-tile from byte-paired registers), so no MMA row is padding: half
//    the MMAs and exp2 of the head-rows form and 32 accumulator registers instead of 64
//    (3 CTAs per SM for e4m3 too); P^T reaches the B-operand layout with 4 shuffles.
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <type_traits>

#include "ual/kernels/common.cuh"
#include "ual/kernels/launchers.h"
#include "ual/kernels/sm100_primitives.cuh"
#include "ual/kernels/tensor_map.h"

namespace tecoops {
namespace kern {

namespace {

constexpr int kChunk = 16;        // tokens per ring stage (one MMA n-tile pair)
// error-word codes of caller errors the kernel detects (bounded waits use 0x11xx, 0x12xx)
constexpr int kErrKvBeyondPlan = 0x1300;   // kv_seq_lens[b] above max_seqlen_k: keys cut
constexpr int kErrQLenAboveOne = 0x1400;   // q_seq_lens[b] > 1: only the first row computed
constexpr int kConsumers = 4;
constexpr int kThreads = 32 * (kConsumers + 1);

template <int D, bool FP8, bool TP = false>
struct DecodeSmem {
    static constexpr int kHalves = D / 64;
    static constexpr int kHalfBytes = kChunk * 128;            // 16 rows x 64 columns
    static constexpr int kTileBytes = kHalves * kHalfBytes;    // 16-bit K or V of one chunk
    static constexpr int kRawTileBytes = FP8 ? kChunk * D : kTileBytes;   // as loaded
    static constexpr int kStageBytes = 2 * kRawTileBytes;
    // ring stages, a multiple of the 4 consumer warps.  The page gathers are latency
    // bound, so the bytes in flight per SM set the bandwidth: 3 CTAs x 8 stages x 8 KB
    // for 16-bit caches, 2 CTAs x 24 stages x 4 KB for e4m3 (3 x 16 in the transposed
    // form, whose smaller register footprint fits 3 CTAs per SM).
    static constexpr int kStages = FP8 ? (TP ? 16 : 24) : 8;
    // chunks the producer issues at once (a power of two dividing 32, below kStages:
    // a batch never waits for a stage that it fills itself)
    static constexpr int kBatch = FP8 ? 8 : 4;
    static constexpr int kRingBytes = kStages * kStageBytes;
    static constexpr int kMergeBytes = 4 * 16 * D * 4 + 4 * 16 * 2 * 4;
    static constexpr int kUsed = kRingBytes;
    static constexpr int kBytes = (kUsed > kMergeBytes ? kUsed : kMergeBytes) + 1024;
};

// 16 e4m3 bytes -> 16 f16 (two 16-byte chunks), exact: one cvt per byte pair
__device__ __forceinline__ void e4m3x4_to_f16(uint32_t w, uint32_t &o0, uint32_t &o1) {
    asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n"
        " cvt.rn.f16x2.e4m3x2 %0, l;\n cvt.rn.f16x2.e4m3x2 %1, h;\n}\n"
        : "=r"(o0), "=r"(o1)
        : "r"(w));
}
__device__ __forceinline__ void e4m3x16_to_f16(const uint4 &in, uint4 &lo, uint4 &hi) {
    e4m3x4_to_f16(in.x, lo.x, lo.y);
    e4m3x4_to_f16(in.y, lo.z, lo.w);
    e4m3x4_to_f16(in.z, hi.x, hi.y);
    e4m3x4_to_f16(in.w, hi.z, hi.w);
}

// byte offset of 16-byte chunk `ch` of row `r` in an e4m3 [16][D] tile as the TMA
// swizzle at the row width stores it (D = 128: 128-byte swizzle, D = 64: 64-byte)
template <int D>
__device__ __forceinline__ uint32_t swz_fp8(int r, int ch) {
    if constexpr (D == 128) return (uint32_t)(r * 128 + ((ch ^ (r & 7)) << 4));
    else return (uint32_t)(r * 64 + ((ch ^ ((r >> 1) & 3)) << 4));
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// bf16x2 / f16x2 word -> f16x2 word
template <typename T>
__device__ __forceinline__ uint32_t to_f16x2(uint32_t w) {
    if constexpr (std::is_same<T, __half>::value) {
        return w;
    } else {
        const float a = __uint_as_float(w << 16), b = __uint_as_float(w & 0xffff0000u);
        return Elem<__half>::pack2(a, b);
    }
}

// byte offset of 16-byte column chunk `ch` (0..D/8-1) of row `r` in a 128B-swizzled
// [16][D] tile stored as D/64 halves of 16 rows x 128 bytes
__device__ __forceinline__ uint32_t swz128(int r, int ch) {
    return (uint32_t)((ch >> 3) * (kChunk * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

}  // namespace

// FP8: 2 CTAs per SM (the raw key/value words and their conversions need registers)
// TP: the transposed form (GQA group of at most 8 heads)
template <typename T, int D, bool FP8, bool TP>
__global__ void __launch_bounds__(kThreads, FP8 && !TP ? 2 : 3)
    fa_decode_splitkv_kernel(const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap, DecodeParams p) {
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    using Sm = DecodeSmem<D, FP8, TP>;
    constexpr int kStages = Sm::kStages;
    // ring FULL / EMPTY barriers, then one barrier that nothing ever completes (the
    // target of the give-up test, DecodeParams::stall_test)
    __shared__ __align__(8) uint64_t bars[2 * kStages + 1];
    __shared__ int abort_flag;
    using MT = typename std::conditional<FP8, __half, T>::type;   // MMA operand type

    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.num_slices;
    const int slice = blockIdx.y - kvh * p.num_slices;
    const int b = blockIdx.z;
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    // the merge kernel may be scheduled from now on (it waits for this grid to complete
    // before it reads anything), so its launch overlaps this grid's last wave
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

    const int q_len = __ldg(p.q_seq_lens + b);
    const int kv_len = __ldg(p.kv_seq_lens + b);
    if (q_len <= 0) return;
    // first admissible key; splits start at its 16-token chunk (page-aligned boxes)
    const int kv_lo = p.window_left >= 0 ? max(0, kv_len - 1 - p.window_left) : 0;
    const int kv_base = kv_lo & ~(kChunk - 1);
    const int kv_begin = kv_base + split * p.split_tokens;
    // the grid has max_splits splits (planned from max_seqlen_k) and the scratch holds
    // max_splits records per row: a kv_len beyond that plan is cut to it and reported
    const int n_split_need = (kv_len - kv_base + p.split_tokens - 1) / p.split_tokens;
    const int n_split_b = min(n_split_need, p.max_splits);
    if (split == 0 && blockIdx.y == 0 && threadIdx.x == 0 && p.dev_error != nullptr) {
        if (n_split_need > p.max_splits) atomicCAS(p.dev_error, 0, kErrKvBeyondPlan);
        if (q_len > 1) atomicCAS(p.dev_error, 0, kErrQLenAboveOne);
    }
    if (kv_begin >= kv_len && !(split == 0 && kv_len - kv_base <= 0)) return;
    const int kv_end = min(kv_len, kv_begin + p.split_tokens);
    const int qrow = warp_seq_start(p.q_seq_lens, b);   // q_len == 1 on this path
    if (qrow >= p.total_q) return;                      // lengths beyond q's rows
    const bool fused = !FP8 && p.new_key != nullptr;
    if (fused && slice == 0 && split == max(n_split_b, 1) - 1 && tid < D / 8) {
        // reshape_and_cache of the new token, this KV head: one 16-byte chunk per thread
        const int64_t slot = __ldg(p.slot_mapping + qrow);
        if (slot >= 0 && slot < (int64_t)p.num_pages * p.block_size) {
            const int64_t page = slot / p.block_size;
            const int64_t row = slot - page * p.block_size;
            const int64_t dst =
                (p.kv_layout == 0 ? (page * p.num_kv_heads + kvh) * p.block_size + row
                                  : (page * p.block_size + row) * p.num_kv_heads + kvh) * D;
            const int64_t src = ((int64_t)qrow * p.num_kv_heads + kvh) * D;
            reinterpret_cast<uint4 *>(const_cast<void *>(p.key_cache))[(dst >> 3) + tid] =
                __ldg(reinterpret_cast<const uint4 *>(p.new_key) + (src >> 3) + tid);
            reinterpret_cast<uint4 *>(const_cast<void *>(p.value_cache))[(dst >> 3) + tid] =
                __ldg(reinterpret_cast<const uint4 *>(p.new_value) + (src >> 3) + tid);
        }
    }
    const int nch = kv_end > kv_begin ? (kv_end - kv_begin + kChunk - 1) / kChunk : 0;

    const int head0 = kvh * p.group + slice * 16;   // first q head of this tile
    const int rows = min(16, p.group - slice * 16);  // valid q heads

    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t *sgen = smem_raw + (sbase - raw);
    const uint32_t bar0 = smem_u32(&bars[0]);
    auto FULL = [&](int s) { return bar0 + 8u * (uint32_t)s; };
    auto EMPTY = [&](int s) { return bar0 + 8u * (uint32_t)(kStages + s); };
    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(FULL(s), 1);
            mbar_init(EMPTY(s), 1);
        }
        mbar_init(bar0 + 16u * kStages, 1);
        mbar_fence_init();
    }
    __syncthreads();
    volatile int *abortp = &abort_flag;

    float m_r[2] = {-INFINITY, -INFINITY};
    float l_r[2] = {0.f, 0.f};
    float o[D / 8][4];
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    const int g = lane >> 2;
    const int c = lane & 3;

    if (warp == kConsumers) {
        // ===================== TMA producer =====================
        if (lane == 0) {
            tma_prefetch_desc(&kmap);
            tma_prefetch_desc(&vmap);
        }
        const int *bt = p.block_table + (int64_t)b * p.block_table_dim;
        // Chunks are issued kBatch at a time, one per lane: lane i waits for its own
        // stage to be released and issues its chunk's copies, so the per-chunk cost is
        // one lane's work rather than a serial loop through lane 0.
        constexpr int kBatch = Sm::kBatch;
        bool ok = true;
        int issued = 0;   // chunks [0, issued) have their copies in flight or landed
        for (int g0 = 0; ok && g0 < nch; g0 += 32) {
            // page id and in-page row of chunk g0 + lane
            int blk = p.num_pages, row = 0;
            const int cc = g0 + lane;
            if (cc < nch) {
                const int tok = kv_begin + cc * kChunk;
                const int pi = tok / p.block_size;
                row = tok - pi * p.block_size;
                if (pi < p.block_table_dim) blk = __ldg(bt + pi);
                if (blk < 0 || blk >= p.num_pages) blk = p.num_pages;   // read as zeros
            }
            const int cnt = min(32, nch - g0);
            for (int b0 = 0; b0 < cnt; b0 += kBatch) {
                const int i = b0 + (lane & (kBatch - 1));
                const int bi = __shfl_sync(0xffffffffu, blk, i & 31);
                const int ri = __shfl_sync(0xffffffffu, row, i & 31);
                const int ci = g0 + i;
                bool lok = true;
                if (lane < kBatch && i < cnt) {
                    const int st = ci % kStages;
                    if (ci >= kStages)
                        lok = mbar_wait_bounded(EMPTY(st), ((ci / kStages) - 1) & 1, abortp,
                                                p.dev_error, 0x1100 + (ci & 0xff),
                                                p.wait_limit_ns);
                    if (lok) {
                        mbar_arrive_expect_tx(FULL(st), Sm::kStageBytes);
                        const uint32_t kd = sbase + st * Sm::kStageBytes;
                        const uint32_t vd = kd + Sm::kRawTileBytes;
                        if (FP8) {   // one box of 16 rows x D bytes
                            tma_load_4d(kd, &kmap, FULL(st), 0, ri, kvh, bi);
                            tma_load_4d(vd, &vmap, FULL(st), 0, ri, kvh, bi);
                        } else {
#pragma unroll
                            for (int hh = 0; hh < Sm::kHalves; ++hh) {
                                tma_load_4d(kd + hh * Sm::kHalfBytes, &kmap, FULL(st), hh * 64,
                                            ri, kvh, bi);
                                tma_load_4d(vd + hh * Sm::kHalfBytes, &vmap, FULL(st), hh * 64,
                                            ri, kvh, bi);
                            }
                        }
                    }
                }
                ok = __all_sync(0xffffffffu, lok);
                if (!ok) break;
                issued = g0 + min(cnt, b0 + kBatch);
            }
        }
        // on abort: wait (bounded) for this warp's copies still in flight (a batch cut
        // short by the abort may have issued a few more: they are waited for as well)
        if (*abortp && lane == 0) {
            const int hi = min(nch, issued + kBatch);
            for (int ci = hi - kStages < 0 ? 0 : hi - kStages; ci < hi; ++ci)
                mbar_wait_bounded(FULL(ci % kStages), (ci / kStages) & 1, nullptr, nullptr, 0,
                                  100000000ull);
        }
    } else {
        // ===================== consumers =====================
        uint32_t qa[D / 16][4];
        {
            const T *qbase =
                static_cast<const T *>(p.q) + ((int64_t)qrow * p.num_heads + head0) * D;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                // k pairs (2c, 2c+1) and (2c+8, 2c+9) of k-step kk; the FP8 path reads
                // them at d = (D/4)*c + 4*kk + {0,1} and {2,3} (the key order below)
                const int k0 = FP8 ? (D / 4) * c + 4 * kk : kk * 16 + 2 * c;
                const int hi = FP8 ? 1 : 4;   // words from the first pair to the second
                const uint32_t *r0 =
                    reinterpret_cast<const uint32_t *>(qbase + (int64_t)g * D + k0);
                const uint32_t *r1 =
                    reinterpret_cast<const uint32_t *>(qbase + (int64_t)(g + 8) * D + k0);
                qa[kk][0] = g < rows ? __ldg(r0) : 0u;
                qa[kk][1] = g + 8 < rows ? __ldg(r1) : 0u;
                qa[kk][2] = g < rows ? __ldg(r0 + hi) : 0u;
                qa[kk][3] = g + 8 < rows ? __ldg(r1 + hi) : 0u;
                if (FP8) {   // the MMAs run in f16 against the converted cache
#pragma unroll
                    for (int i = 0; i < 4; ++i) qa[kk][i] = to_f16x2<T>(qa[kk][i]);
                }
            }
        }
        const float sl2 = p.scale_log2;
        const int mi = lane >> 3;   // ldmatrix matrix index of this lane's address
        const int ri = lane & 7;
        for (int ci = warp; ci < nch; ci += kConsumers) {
            const int st = ci % kStages;
            // (stall_test: the first wait of each consumer targets the barrier nothing
            // completes, so it runs out and takes the abort path below)
            const bool stall = p.stall_test && ci == warp;
            if (!__all_sync(0xffffffffu,
                            mbar_wait_bounded(stall ? bar0 + 16u * kStages : FULL(st),
                                              stall ? 0u : (ci / kStages) & 1, abortp,
                                              p.dev_error, 0x1200 + (ci & 0xff),
                                              p.wait_limit_ns)))
                break;
            const int tok0 = kv_begin + ci * kChunk;
            const int nv = kv_end - tok0;   // tokens of this chunk before kv_end
            const int nlo = kv_lo - tok0;   // tokens of this chunk before the window
            const uint32_t ktile = sbase + st * Sm::kStageBytes;
            const uint32_t vtile = ktile + Sm::kRawTileBytes;
            // 16-bit tiles: V rows past kv_len may hold arbitrary bits (unwritten slots),
            // so they are cleared; the fused step's new token comes from the inputs
            auto prep16 = [&]() {
            if (nv < kChunk) {
                // V rows past kv_len may hold arbitrary bits (unwritten slots): clear them
                uint8_t *vt = sgen + (vtile - sbase);
                for (int idx = lane; idx < (kChunk - nv) * (D / 8); idx += 32) {
                    const int r = nv + idx / (D / 8);
                    const int ch = idx % (D / 8);
                    *reinterpret_cast<uint4 *>(vt + swz128(r, ch)) = make_uint4(0, 0, 0, 0);
                }
                fence_proxy_async_smem();   // ordered before TMA refills this stage
                __syncwarp();
            }
            const int rn = kv_len - 1 - tok0;   // row of the new token in this chunk
            if (fused && rn >= 0 && rn < kChunk) {
                // the new token's K and V come from the inputs, not from the cache
                uint8_t *kt = sgen + (ktile - sbase);
                uint8_t *vt = kt + Sm::kTileBytes;
                const int64_t src = ((int64_t)qrow * p.num_kv_heads + kvh) * D;
                for (int ch = lane; ch < D / 8; ch += 32) {
                    *reinterpret_cast<uint4 *>(kt + swz128(rn, ch)) =
                        __ldg(reinterpret_cast<const uint4 *>(p.new_key) + (src >> 3) + ch);
                    *reinterpret_cast<uint4 *>(vt + swz128(rn, ch)) =
                        __ldg(reinterpret_cast<const uint4 *>(p.new_value) + (src >> 3) + ch);
                }
                fence_proxy_async_smem();   // ordered before TMA refills this stage
                __syncwarp();
            }
            };
            if constexpr (TP) {
                // ---- transposed form (e4m3, GQA group <= 8): S^T = K Q^T with the 16
                // tokens of the chunk as MMA rows and the heads as its 8 columns, then
                // O^T += V^T P^T, so no MMA row is padding
                float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
                uint32_t tv[4][2][FP8 ? D / 64 : 1];
                if constexpr (FP8) {
                const uint8_t *rk = sgen + (ktile - sbase);
                const uint8_t *rv = rk + Sm::kRawTileBytes;
                uint32_t kw[2][D / 16];   // key rows g and g + 8: D/4 bytes at (D/4)*c
#pragma unroll
                for (int j = 0; j < 2; ++j) {
#pragma unroll
                    for (int q = 0; q < D / 64; ++q) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(
                            rk + swz_fp8<D>(8 * j + g, (D / 64) * c + q));
                        kw[j][4 * q] = v.x;
                        kw[j][4 * q + 1] = v.y;
                        kw[j][4 * q + 2] = v.z;
                        kw[j][4 * q + 3] = v.w;
                    }
                }
                // value rows 2c, 2c+1, 2c+8, 2c+9 at output rows m = g and g + 8 of every
                // m-tile: D/16 bytes at column (D/16)*m (zeros past kv_len)
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int r = 2 * c + (t & 1) + 8 * (t >> 1);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int m = g + 8 * h;
                        if constexpr (D == 128) {
                            uint2 v = *reinterpret_cast<const uint2 *>(
                                rv + swz_fp8<D>(r, m >> 1) + 8 * (m & 1));
                            if (r >= nv) v = make_uint2(0, 0);
                            tv[t][h][0] = v.x;
                            tv[t][h][1] = v.y;
                        } else {
                            uint32_t v = *reinterpret_cast<const uint32_t *>(
                                rv + swz_fp8<D>(r, m >> 2) + 4 * (m & 3));
                            tv[t][h][0] = r >= nv ? 0u : v;
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(EMPTY(st));
                // S^T: A = key rows (k-step kk is word kk of the lane's segment), B = Q^T
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    uint32_t af[4];
                    e4m3x4_to_f16(kw[0][kk], af[0], af[2]);
                    e4m3x4_to_f16(kw[1][kk], af[1], af[3]);
                    mma16816<__half>((kk & 1) ? sb : sa, af, qa[kk][0], qa[kk][2]);
                }
                } else {
                    prep16();
                    // S^T: A = key rows by ldmatrix (matrices: tokens 0-7 / 8-15 x the two
                    // 8-column halves of k-step kk), B = Q^T
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        uint32_t af[4];
                        ldmatrix_x4(af, ktile + swz128((mi & 1) * 8 + ri, 2 * kk + (mi >> 1)));
                        mma16816<MT>((kk & 1) ? sb : sa, af, qa[kk][0], qa[kk][2]);
                    }
                }
                // sa[0..1]: token g, heads 2c, 2c+1; sa[2..3]: token g + 8
                float x[4], mx[2];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = g + 8 * (e >> 1);
                    x[e] = (unsigned)(t - nlo) < (unsigned)(nv - nlo) ? (sa[e] + sb[e]) * sl2
                                                                      : -INFINITY;
                }
                mx[0] = fmaxf(x[0], x[2]);
                mx[1] = fmaxf(x[1], x[3]);
                float mu[2], alpha[2];
                bool grow = false;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
#pragma unroll
                    for (int o2 = 4; o2 < 32; o2 <<= 1)
                        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], o2));
                    const float m_new = fmaxf(m_r[h], mx[h]);
                    grow |= m_new > m_r[h];
                    mu[h] = m_new == -INFINITY ? 0.f : m_new;
                    alpha[h] = fast_exp2(m_r[h] - mu[h]);
                    m_r[h] = m_new;
                }
                float pe[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) pe[e] = fast_exp2(x[e] - mu[e & 1]);
                // per-lane partial row sums (reduced over the 8 token lanes at the end)
                l_r[0] = l_r[0] * alpha[0] + (pe[0] + pe[2]);
                l_r[1] = l_r[1] * alpha[1] + (pe[1] + pe[3]);
                if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
                    for (int n = 0; n < D / 16; ++n) {
                        o[n][0] *= alpha[0];
                        o[n][1] *= alpha[1];
                        o[n][2] *= alpha[0];
                        o[n][3] *= alpha[1];
                    }
                }
                // P^T as the B operand: b0 = P[2c][head g], P[2c+1][g]; b1 = P[2c+8][g],
                // P[2c+9][g].  P[t][h] sits in lane 4*(t&7) + h/2, word t/8, half h&1.
                const uint32_t w0 = Elem<MT>::pack2(pe[0], pe[1]);
                const uint32_t w1 = Elem<MT>::pack2(pe[2], pe[3]);
                const int src0 = 4 * (2 * c) + (g >> 1), src1 = src0 + 4;
                const uint32_t x0 = __shfl_sync(0xffffffffu, w0, src0);
                const uint32_t x1 = __shfl_sync(0xffffffffu, w0, src1);
                const uint32_t y0 = __shfl_sync(0xffffffffu, w1, src0);
                const uint32_t y1 = __shfl_sync(0xffffffffu, w1, src1);
                const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;
                const uint32_t b0 = prmt(x0, x1, sel), b1 = prmt(y0, y1, sel);
                if constexpr (FP8) {
                // O^T m-tile mt: rows d = (D/16)*m + mt (m = g, g + 8), byte mt of the
                // lane's value segments, paired by token row
#pragma unroll
                for (int w = 0; w < D / 64; ++w) {
                    uint32_t a0[4], a1[4], a2[4], a3[4];
                    e4m3x4_to_f16(prmt(tv[0][0][w], tv[1][0][w], 0x5140u), a0[0], a0[1]);
                    e4m3x4_to_f16(prmt(tv[0][0][w], tv[1][0][w], 0x7362u), a0[2], a0[3]);
                    e4m3x4_to_f16(prmt(tv[0][1][w], tv[1][1][w], 0x5140u), a1[0], a1[1]);
                    e4m3x4_to_f16(prmt(tv[0][1][w], tv[1][1][w], 0x7362u), a1[2], a1[3]);
                    e4m3x4_to_f16(prmt(tv[2][0][w], tv[3][0][w], 0x5140u), a2[0], a2[1]);
                    e4m3x4_to_f16(prmt(tv[2][0][w], tv[3][0][w], 0x7362u), a2[2], a2[3]);
                    e4m3x4_to_f16(prmt(tv[2][1][w], tv[3][1][w], 0x5140u), a3[0], a3[1]);
                    e4m3x4_to_f16(prmt(tv[2][1][w], tv[3][1][w], 0x7362u), a3[2], a3[3]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t af[4] = {a0[i], a1[i], a2[i], a3[i]};
                        mma16816<__half>(o[4 * w + i], af, b0, b1);
                    }
                }
                } else {
                    // O^T m-tile mt: rows d = 16*mt + m; A = V^T by transposing loads of the
                    // value tile (matrices: d 0-7 / 8-15 x tokens 0-7 / 8-15)
#pragma unroll
                    for (int mt = 0; mt < D / 16; ++mt) {
                        uint32_t af[4];
                        ldmatrix_x4_trans(af, vtile + swz128(8 * (mi >> 1) + ri, 2 * mt + (mi & 1)));
                        mma16816<MT>(o[mt], af, b0, b1);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(EMPTY(st));
                }
                continue;
            }
            float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            uint32_t vw[4][FP8 ? D / 32 : 1];   // FP8: value rows 2c, 2c+1, 2c+8, 2c+9
            if constexpr (FP8) {
                // raw e4m3 chunk -> registers, then the stage is free for the next copy
                const uint8_t *rk = sgen + (ktile - sbase);
                const uint8_t *rv = rk + Sm::kRawTileBytes;
                uint32_t kw[2][D / 16];   // key rows g and g + 8: D/4 bytes at (D/4)*c
#pragma unroll
                for (int j = 0; j < 2; ++j) {
#pragma unroll
                    for (int q = 0; q < D / 64; ++q) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(
                            rk + swz_fp8<D>(8 * j + g, (D / 64) * c + q));
                        kw[j][4 * q] = v.x;
                        kw[j][4 * q + 1] = v.y;
                        kw[j][4 * q + 2] = v.z;
                        kw[j][4 * q + 3] = v.w;
                    }
                }
                // value rows past kv_len as zeros (their bytes may be NaN patterns)
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int r = 2 * c + (t & 1) + 8 * (t >> 1);
                    if constexpr (D == 128) {
                        uint4 v = *reinterpret_cast<const uint4 *>(rv + swz_fp8<D>(r, g));
                        if (r >= nv) v = make_uint4(0, 0, 0, 0);
                        vw[t][0] = v.x;
                        vw[t][1] = v.y;
                        vw[t][2] = v.z;
                        vw[t][3] = v.w;
                    } else {
                        uint2 v = *reinterpret_cast<const uint2 *>(rv + swz_fp8<D>(r, g >> 1) +
                                                                   8 * (g & 1));
                        if (r >= nv) v = make_uint2(0, 0);
                        vw[t][0] = v.x;
                        vw[t][1] = v.y;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(EMPTY(st));
                // S = Q K^T: the key bytes of k-step kk are word kk of the lane's segment
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        uint32_t b0, b1;
                        e4m3x4_to_f16(kw[j][kk], b0, b1);
                        mma16816<__half>(s[j], qa[kk], b0, b1);
                    }
                }
            } else {
                prep16();
                // S = Q K^T: two n-tiles of 8 tokens
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    uint32_t kb[4];
                    const int r = (mi >> 1) * 8 + ri;
                    ldmatrix_x4(kb, ktile + swz128(r, 2 * kk + (mi & 1)));
                    mma16816<MT>(s[0], qa[kk], kb[0], kb[1]);
                    mma16816<MT>(s[1], qa[kk], kb[2], kb[3]);
                }
            }
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < 2; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = 8 * j + 2 * c + (e & 1);
                    // nlo <= t < nv as one unsigned compare (nlo < 16 <= ... and nv > nlo)
                    const float x =
                        (unsigned)(t - nlo) < (unsigned)(nv - nlo) ? s[j][e] * sl2 : -INFINITY;
                    s[j][e] = x;
                    mx[e >> 1] = fmaxf(mx[e >> 1], x);
                }
            }
            float mu[2], alpha[2];
            bool grow = false;
#pragma unroll
            for (int r2 = 0; r2 < 2; ++r2) {
                mx[r2] = fmaxf(mx[r2], __shfl_xor_sync(0xffffffffu, mx[r2], 1));
                mx[r2] = fmaxf(mx[r2], __shfl_xor_sync(0xffffffffu, mx[r2], 2));
                const float m_new = fmaxf(m_r[r2], mx[r2]);
                grow |= m_new > m_r[r2];
                mu[r2] = m_new == -INFINITY ? 0.f : m_new;
                alpha[r2] = fast_exp2(m_r[r2] - mu[r2]);
                m_r[r2] = m_new;
            }
            float ps[2] = {0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 2; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float pe = fast_exp2(s[j][e] - mu[e >> 1]);
                    s[j][e] = pe;
                    ps[e >> 1] += pe;
                }
            }
            l_r[0] = l_r[0] * alpha[0] + ps[0];
            l_r[1] = l_r[1] * alpha[1] + ps[1];
            if (__any_sync(0xffffffffu, grow)) {   // skip the rescale when no max grew
#pragma unroll
                for (int n = 0; n < D / 8; ++n) {
                    o[n][0] *= alpha[0];
                    o[n][1] *= alpha[0];
                    o[n][2] *= alpha[1];
                    o[n][3] *= alpha[1];
                }
            }
            uint32_t pa[4];
            pa[0] = Elem<MT>::pack2(s[0][0], s[0][1]);
            pa[1] = Elem<MT>::pack2(s[0][2], s[0][3]);
            pa[2] = Elem<MT>::pack2(s[1][0], s[1][1]);
            pa[3] = Elem<MT>::pack2(s[1][2], s[1][3]);
            if constexpr (FP8) {
                // b0 = V[2c][d], V[2c+1][d]; b1 = V[2c+8][d], V[2c+9][d] with
                // d = (D/8)*g + nn: byte nn of the lane's value segments, paired by row
#pragma unroll
                for (int w = 0; w < D / 32; ++w) {
                    uint32_t b0[4], b1[4];
                    e4m3x4_to_f16(prmt(vw[0][w], vw[1][w], 0x5140u), b0[0], b0[1]);
                    e4m3x4_to_f16(prmt(vw[0][w], vw[1][w], 0x7362u), b0[2], b0[3]);
                    e4m3x4_to_f16(prmt(vw[2][w], vw[3][w], 0x5140u), b1[0], b1[1]);
                    e4m3x4_to_f16(prmt(vw[2][w], vw[3][w], 0x7362u), b1[2], b1[3]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) mma16816<__half>(o[4 * w + i], pa, b0[i], b1[i]);
                }
            } else {
#pragma unroll
                for (int nn = 0; nn < D / 16; ++nn) {
                    uint32_t vb[4];
                    const int r = (mi & 1) * 8 + ri;
                    ldmatrix_x4_trans(vb, vtile + swz128(r, 2 * nn + (mi >> 1)));
                    mma16816<MT>(o[2 * nn], pa, vb[0], vb[1]);
                    mma16816<MT>(o[2 * nn + 1], pa, vb[2], vb[3]);
                }
            }
            if (!FP8) {
                __syncwarp();
                if (lane == 0) mbar_arrive(EMPTY(st));
            }
        }
        if constexpr (TP) {   // partial sums of heads 2c, 2c+1 over the 8 token lanes
#pragma unroll
            for (int o2 = 4; o2 < 32; o2 <<= 1) {
                l_r[0] += __shfl_xor_sync(0xffffffffu, l_r[0], o2);
                l_r[1] += __shfl_xor_sync(0xffffffffu, l_r[1], o2);
            }
        } else {
            l_r[0] += __shfl_xor_sync(0xffffffffu, l_r[0], 1);
            l_r[0] += __shfl_xor_sync(0xffffffffu, l_r[0], 2);
            l_r[1] += __shfl_xor_sync(0xffffffffu, l_r[1], 1);
            l_r[1] += __shfl_xor_sync(0xffffffffu, l_r[1], 2);
        }
    }

    // ---- merge the 4 consumer warps through shared memory (the ring is idle now) ----
    __syncthreads();
    float *so = reinterpret_cast<float *>(sgen);   // [4][16][D]
    float *sml = so + 4 * 16 * D;                  // [4][16][2]
    if (TP && warp < kConsumers) {
        // O^T m-tile n: output rows m = g (o[n][0..1]) and g + 8 (o[n][2..3]),
        // columns = heads 2c, 2c+1
#pragma unroll
        for (int n = 0; n < D / 16; ++n) {
            // e4m3: d = (D/16)*m + n; 16-bit: d = 16*n + m
            const int d0 = FP8 ? (D / 16) * g + n : 16 * n + g;
            const int d1 = FP8 ? d0 + D / 2 : d0 + 8;
            so[(warp * 16 + 2 * c) * D + d0] = o[n][0];
            so[(warp * 16 + 2 * c + 1) * D + d0] = o[n][1];
            so[(warp * 16 + 2 * c) * D + d1] = o[n][2];
            so[(warp * 16 + 2 * c + 1) * D + d1] = o[n][3];
        }
        if (g == 0) {
            sml[(warp * 16 + 2 * c) * 2 + 0] = m_r[0];
            sml[(warp * 16 + 2 * c) * 2 + 1] = l_r[0];
            sml[(warp * 16 + 2 * c + 1) * 2 + 0] = m_r[1];
            sml[(warp * 16 + 2 * c + 1) * 2 + 1] = l_r[1];
        }
    } else if (warp < kConsumers) {
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
            // output column of (n-tile n, MMA column 2c / 2c+1); FP8: d = (D/8)*col + n
            const int col0 = FP8 ? (D / 8) * (2 * c) + n : n * 8 + 2 * c;
            const int col1 = FP8 ? col0 + D / 8 : col0 + 1;
            so[(warp * 16 + g) * D + col0] = o[n][0];
            so[(warp * 16 + g) * D + col1] = o[n][1];
            so[(warp * 16 + g + 8) * D + col0] = o[n][2];
            so[(warp * 16 + g + 8) * D + col1] = o[n][3];
        }
        if (c == 0) {
            sml[(warp * 16 + g) * 2 + 0] = m_r[0];
            sml[(warp * 16 + g) * 2 + 1] = l_r[0];
            sml[(warp * 16 + g + 8) * 2 + 0] = m_r[1];
            sml[(warp * 16 + g + 8) * 2 + 1] = l_r[1];
        }
    }
    __syncthreads();

    const bool direct = n_split_b <= 1;
    for (int idx = tid; idx < rows * D; idx += kThreads) {
        const int r = idx / D;
        const int d = idx - r * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, sml[(w * 16 + r) * 2]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float f = fast_exp2(sml[(w * 16 + r) * 2] - Mu);
            L += sml[(w * 16 + r) * 2 + 1] * f;
            O += so[(w * 16 + r) * D + d] * f;
        }
        const float val = (L > 0.f ? O / L : 0.f) * (FP8 ? p.v_scale : 1.f);
        const int h = head0 + r;
        if (direct) {
            T *out = static_cast<T *>(p.out) + ((int64_t)qrow * p.num_heads + h) * D + d;
            *out = Elem<T>::from_float(val);
            if (p.lse != nullptr && d == 0)
                p.lse[(int64_t)h * p.total_q + qrow] =
                    L > 0.f ? (Mu + log2f(L)) * 0.6931471805599453f : -INFINITY;
        } else {
            const int64_t rec = ((int64_t)b * p.num_heads + h) * p.max_splits + split;
            p.part_o[rec * D + d] = val;
            if (d == 0) p.part_lse[rec] = L > 0.f ? Mu + log2f(L) : -INFINITY;
        }
    }
}

// Combine the split partials of every (sequence, q head) that used more than
// one split: out = sum_s 2^(lse_s - M) O_s / sum_s 2^(lse_s - M).
template <typename T, int D>
__global__ void __launch_bounds__(128) fa_decode_merge_kernel(DecodeParams p) {
    // one warp per (sequence, q head): lanes read the split log2-sum-exps in parallel,
    // reduce by shuffle, and each lane accumulates D/32 consecutive output columns
    constexpr int kPer = D / 32;
    const int lane = threadIdx.x & 31;
    // launched as a programmatic dependent of the split kernel: wait until that grid has
    // completed and its partial records are visible
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    const int rec_id = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (rec_id >= p.batch * p.num_heads) return;
    const int b = rec_id / p.num_heads;
    const int h = rec_id - b * p.num_heads;
    const int q_len = __ldg(p.q_seq_lens + b);
    const int kv_len = __ldg(p.kv_seq_lens + b);
    const int kv_lo = p.window_left >= 0 ? max(0, kv_len - 1 - p.window_left) : 0;
    const int ns =
        min((kv_len - (kv_lo & ~15) + p.split_tokens - 1) / p.split_tokens, p.max_splits);
    if (q_len <= 0 || ns <= 1) return;
    const int qrow = warp_seq_start(p.q_seq_lens, b);
    if (qrow >= p.total_q) return;
    const int64_t rec0 = ((int64_t)b * p.num_heads + h) * p.max_splits;
    float M = -INFINITY;
    for (int sp = lane; sp < ns; sp += 32) M = fmaxf(M, p.part_lse[rec0 + sp]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float Mu = M == -INFINITY ? 0.f : M;
    float W = 0.f, O[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) O[i] = 0.f;
    for (int s0 = 0; s0 < ns; s0 += 32) {
        const int sp = s0 + lane;
        const float wl = sp < ns ? fast_exp2(p.part_lse[rec0 + sp] - Mu) : 0.f;
        const int cnt = min(32, ns - s0);
        for (int t = 0; t < cnt; ++t) {
            const float w = __shfl_sync(0xffffffffu, wl, t);
            W += w;
            const float *src = p.part_o + (rec0 + s0 + t) * D + lane * kPer;
            if constexpr (kPer == 4) {
                const float4 v = *reinterpret_cast<const float4 *>(src);
                O[0] += w * v.x;
                O[1] += w * v.y;
                O[2] += w * v.z;
                O[3] += w * v.w;
            } else {
#pragma unroll
                for (int i = 0; i < kPer; ++i) O[i] += w * src[i];
            }
        }
    }
    const float inv = W > 0.f ? 1.f / W : 0.f;   // partials carry v_scale
    T *out = static_cast<T *>(p.out) + ((int64_t)qrow * p.num_heads + h) * D + lane * kPer;
#pragma unroll
    for (int i = 0; i < kPer; ++i) out[i] = Elem<T>::from_float(O[i] * inv);
    if (p.lse != nullptr && lane == 0)
        p.lse[(int64_t)h * p.total_q + qrow] =
            W > 0.f ? (Mu + log2f(W)) * 0.6931471805599453f : -INFINITY;
}

// ---- host side ------------------------------------------------------------------

bool decode_supported(int head_dim, int block_size, int group) {
    (void)group;
    return (head_dim == 64 || head_dim == 128) && block_size > 0 && (block_size % 16 == 0);
}

void decode_plan(int num_sms, int batch, int kv_heads, int group, int max_k, int *split_tokens,
                 int *max_splits, bool cache_fp8) {
    const int slices = (group + 15) / 16;
    const int64_t work = (int64_t)batch * kv_heads * slices * (int64_t)(max_k > 0 ? max_k : 1);
    // Many short CTAs even out the tail (splits end at different kv_len), but each CTA
    // pays a start-up and adds a merge record: ~64 waves of 2 CTAs per SM with at least
    // 1536 tokens per split measured best on both the B=64 (ctx <= 8k) and the B=256
    // (ctx <= 32k) decode workloads (8 waves / 256 tokens left 10 % on the table at B=256).
    const int64_t target = (int64_t)num_sms * 2 * 64;
    int64_t split = (work + target - 1) / target;
    split = ((split + 63) / 64) * 64;
    // (an e4m3 cache in the head-rows form, GQA group > 8: 3072 tokens per split measured
    // 4 % faster on the B=64 workload; the transposed form is best at 1536 like 16-bit)
    const int64_t smin = cache_fp8 && group > 8 ? 3072 : 1536;
    if (split < smin) split = smin;
    const int64_t cap = ((int64_t)(max_k > 0 ? max_k : 1) + 63) / 64 * 64;
    if (split > cap) split = cap < 64 ? 64 : cap;
    *split_tokens = (int)split;
    *max_splits = (int)(((max_k > 0 ? max_k : 1) + split - 1) / split);
}

size_t decode_workspace_bytes(int batch, int num_heads, int head_dim, int max_splits) {
    if (max_splits <= 1) return 0;
    const size_t recs = (size_t)batch * num_heads * max_splits;
    return recs * head_dim * sizeof(float) + recs * sizeof(float) + 256;
}

template <typename T, int D, bool FP8, bool TP>
static cudaError_t launch_decode_t(const DecodeParams &p, cudaStream_t stream) {
    const CacheElem ce = FP8 ? CacheElem::E4M3
                             : std::is_same<T, __half>::value ? CacheElem::F16 : CacheElem::BF16;
    CUtensorMap kmap, vmap;
    if (!encode_cache_map(&kmap, p.key_cache, ce, D, p.block_size, p.num_kv_heads, p.num_pages,
                          kChunk, p.kv_layout) ||
        !encode_cache_map(&vmap, p.value_cache, ce, D, p.block_size, p.num_kv_heads,
                          p.num_pages, kChunk, p.kv_layout))
        return cudaErrorInvalidValue;
    const int smem = DecodeSmem<D, FP8, TP>::kBytes;
    auto kfn = fa_decode_splitkv_kernel<T, D, FP8, TP>;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid(p.max_splits, p.num_kv_heads * p.num_slices, p.batch);
    kfn<<<grid, kThreads, smem, stream>>>(kmap, vmap, p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (p.max_splits > 1) {
        const int recs = p.batch * p.num_heads;
        // programmatic dependent launch: measured 1 % faster on the Llama-3-8B decode step
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((recs + 3) / 4);
        cfg.blockDim = dim3(128);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, fa_decode_merge_kernel<T, D>, p);
    }
    return e;
}

template <bool FP8, bool TP>
static cudaError_t launch_decode_f(const DecodeParams &p, bool bf16, cudaStream_t stream) {
    if (p.head_dim == 128) {
        return bf16 ? launch_decode_t<__nv_bfloat16, 128, FP8, TP>(p, stream)
                    : launch_decode_t<__half, 128, FP8, TP>(p, stream);
    }
    if (p.head_dim == 64) {
        return bf16 ? launch_decode_t<__nv_bfloat16, 64, FP8, TP>(p, stream)
                    : launch_decode_t<__half, 64, FP8, TP>(p, stream);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_decode(const DecodeParams &p, bool bf16, cudaStream_t stream) {
    if (p.cache_fp8 && p.new_key != nullptr) return cudaErrorInvalidValue;
    // a GQA group of at most 8 heads: the transposed (tokens x heads) form
    if (p.group <= 8)
        return p.cache_fp8 ? launch_decode_f<true, true>(p, bf16, stream)
                           : launch_decode_f<false, true>(p, bf16, stream);
    return p.cache_fp8 ? launch_decode_f<true, false>(p, bf16, stream)
                       : launch_decode_f<false, false>(p, bf16, stream);
}

}  // namespace kern
}  // namespace tecoops
