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
// B200 design.  One CTA owns two 128-row Q sub-tiles that read the same KV head:
// two heads of one GQA group over the same rows (group even), or two consecutive
// row tiles of one head (group odd).  K/V tiles are loaded once for both.
//   warps 0, 10 TMA producers (warp 0: both Q sub-tiles and the K ring; warp 10: the
//               V ring), K/V tiles of 128 tokens assembled
//               from 128/block_size page boxes of the 4-D cache tensor map (the page id
//               is a TMA coordinate; pages past kv_len use an out-of-range coordinate
//               so TMA zero-fills them); K ring of 2 stages released as soon as the S
//               MMAs reading a tile are done, V ring of 2 stages released after the
//               PV MMAs; 128-byte swizzle, 64-column boxes.  Warp 10 also clears V rows past
//               kv_len in the last tile.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer, fixed order
//               PV_0(j) S_0(j+1) | PV_1(j) S_1(j+1) | ... with every operand of a pair
//               awaited before its 16 MMAs go out back-to-back (the issue queue is
//               shallow, so gaps between groups idle the tensor pipe):
//                 S_X = Q_X K_j^T (SS form, M=128, N=128, K=D, fp32 in TMEM)
//                 O_X += P_X V_j  (TS form: P read from TMEM, V MN-major in smem)
//   warps 2-5   softmax of sub-tile 0, warps 6-9 of sub-tile 1: thread r owns
//               row r = TMEM lane r (r = 32*(warp%4) + lane); the 128-score row is
//               read from TMEM in one burst, max by 3-input max trees, exp2 on the
//               MUFU unit (scale and sums in packed f32x2 arithmetic), 16-bit P written over
//               the S columns it came from, lazy O rescale (only when the running max
//               grows by more than 2^8), epilogue O / l -> global: each warp stages
//               its 32 rows in shared memory, 64 columns at a time, and writes them with
//               one TMA store per half (row-per-thread global stores touch 32 lines per
//               instruction and measured ~2,300 cycles per epilogue; the staged form
//               frees the warp for the next unit's first tile).
// TMEM columns: S_0 [0,128) S_1 [128,256) O_0 [256,256+D) O_1 [384,384+D).
// Persistent: one CTA per SM walks work units (a Q row block of the two sub-tiles of
// one sequence), heaviest first, drawn from a global counter; Q of the next unit is
// loaded as soon as the current unit's last S MMAs have read Q, and its first PV
// waits only for the previous epilogue to have read O out of TMEM, so consecutive
// units overlap.  The counters live in the handle's device word block and are reset
// by the last CTA to finish.
// Every mbarrier wait is bounded (~2 s); a wait that gives up records its site in
// the device error word and the CTA drains its MMAs, frees TMEM and exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <type_traits>

#include "ual/kernels/common.cuh"
#include "ual/kernels/launchers.h"
#include "ual/kernels/sm100_primitives.cuh"
#include "ual/kernels/tensor_map.h"

namespace tecoops {
namespace kern {

using namespace sm100;

namespace {

constexpr int kBM = 128;        // Q rows per sub-tile
constexpr int kBN = 128;        // KV tokens per tile
constexpr int kThreads = 352;   // warp 0 Q/K producer, warp 1 MMA, warps 2-5 / 6-9 softmax
                                // of sub-tile 0 / 1, warp 10 V producer
constexpr uint32_t kTmemCols = 512;
// TMEM columns: S_X at 128*X (P_X aliased on its first 64 columns), O_X at 256 + 128*X
constexpr uint32_t kColS = 0;
constexpr uint32_t kColO = 256;

constexpr int kKStages = 2, kVStages = 2;
constexpr int kStageRowBytes = 128;   // epilogue staging: one 64-column bf16/f16 half-row

template <int D>
struct PrefillSmem {
    static constexpr int kHalves = D / 64;
    static constexpr int kHalfBytes = 128 * 128;              // 128 rows x 128 B
    static constexpr int kTileBytes = kHalves * kHalfBytes;   // one Q sub-tile, K or V tile
    static constexpr int kQ0 = 0;                              // Q sub-tiles 0 and 1
    static constexpr int kK0 = 2 * kTileBytes;                 // K stages
    static constexpr int kV0 = kK0 + kKStages * kTileBytes;    // V stages 0, 1
    // epilogue staging: per softmax warp 32 rows x 64 columns (one half of its rows)
    static constexpr int kO0 = kV0 + kVStages * kTileBytes;
    static constexpr int kOWarpBytes = 32 * kStageRowBytes;
    static constexpr int kBytes = kO0 + 8 * kOWarpBytes;
    static constexpr int kAlloc = kBytes + 1024;               // 1024-byte alignment slack
};

struct PrefillParams {
    const int *q_seq_lens;
    const int *kv_seq_lens;
    const int *block_table;
    void *out;
    int *dev_error;
    int *sched;         // [0] unit counter, [1] finished-CTA counter (zero at launch)
    int num_heads;
    int num_kv_heads;
    int group;
    int pair_heads;     // 1: sub-tiles are heads 2i, 2i+1 of one GQA group (same rows)
                        // 0: sub-tiles are row tiles 2i, 2i+1 of one head
    int block_size;
    int rows_per_box;   // min(block_size, 128)
    int block_table_dim;
    int num_pages;
    int num_units;      // per sequence: q-tiles (pair_heads) or q-tile pairs
    int batch;
    int total_q;
    float scale_log2;
    int causal;         // key bounds of row i (off = kv_len - q_len): j < kv_len and
    int window_left;    //   j <= off + i (causal) / off + i + window_right (non-causal,
    int window_right;   //   right >= 0); j >= off + i - window_left (left >= 0)
    float *lse;         // optional [Hq, total_q] natural-log log-sum-exp
    int out_al32;       // out is 32-byte aligned: rows are written with 256-bit stores
    int out_tma;        // out is 16-byte aligned: full 32-row warp tiles leave by TMA store
    int late_draw;      // draw each CTA's next unit late (few units per CTA)
};

// eight 32-bit words to a 32-byte aligned global address in one instruction
__device__ __forceinline__ void st_global_v8(void *ptr, const uint32_t *w) {
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"l"(ptr), "r"(w[0]),
                 "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
}

enum WaitSite : int {
    kSiteQ = 0x100, kSiteK = 0x200, kSiteV = 0x300, kSiteEmpty = 0x400, kSiteS = 0x500,
    kSiteP = 0x600, kSiteO = 0x700, kSiteDrain = 0x800, kSiteVz = 0x900, kSiteSched = 0xa00
};
// caller error the scheduler detects: a q_seq_lens entry above max_seqlen_q (the work
// units are planned from max_seqlen_q; rows past the plan are not computed)
constexpr int kErrQBeyondPlan = 0xb00;

// barrier slots
constexpr int Q_FULL = 0, K_FULL = 1, K_EMPTY = 4, V_FULL = 7, V_EMPTY = 9, S_FULL = 11,
              P_FULL = 13, O_DONE = 15, V_ZERO = 17, DRAIN = 18, Q_EMPTY = 19, O_FREE = 20,
              SCHED_FULL = 22, SCHED_EMPTY = 26, NUM_BARS = 30;
// roles that take each work unit from the scheduler ring: the V producer, the MMA
// thread and the 8 softmax warps (the Q/K producer is the scheduler)
constexpr int kSchedConsumers = 10;

// max of 32 scores (u) and acc; when MASKED only columns in [lo, nv) count
template <bool MASKED>
__device__ __forceinline__ float chunk_max(const uint32_t (&u)[32], int lo, int nv, float acc) {
    float m[4] = {acc, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
        float x0 = __uint_as_float(u[e]), x1 = __uint_as_float(u[e + 1]);
        if (MASKED) {
            // lo <= e < nv as one unsigned compare (an empty range masks everything)
            const unsigned w = nv > lo ? (unsigned)(nv - lo) : 0u;
            x0 = (unsigned)(e - lo) < w ? x0 : -INFINITY;
            x1 = (unsigned)(e + 1 - lo) < w ? x1 : -INFINITY;
        }
        m[(e >> 1) & 3] = fmax3(m[(e >> 1) & 3], x0, x1);
    }
    return fmax3(m[0], fmax3(m[1], m[2], m[3]), -INFINITY);
}

// p = 2^(s*scale - m) for 32 scores, packed to 16-bit pairs; row sum accumulated
// in two packed fp32 accumulators
template <typename T, bool MASKED>
__device__ __forceinline__ void chunk_exp(const uint32_t (&u)[32], int lo, int nv, uint64_t sl2x2,
                                          uint64_t negm2, uint64_t (&sum)[2],
                                          uint32_t (&pk)[16]) {
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
        float x0 = __uint_as_float(u[e]), x1 = __uint_as_float(u[e + 1]);
        if (MASKED) {
            // lo <= e < nv as one unsigned compare (an empty range masks everything)
            const unsigned w = nv > lo ? (unsigned)(nv - lo) : 0u;
            x0 = (unsigned)(e - lo) < w ? x0 : -INFINITY;
            x1 = (unsigned)(e + 1 - lo) < w ? x1 : -INFINITY;
        }
        float t0, t1;
        f2unpack(ffma2(f2pack(x0, x1), sl2x2, negm2), t0, t1);
        // every exp2 on the MUFU unit: moving a share of them to a polynomial on the
        // FMA pipe measured slower here (the softmax chain is latency-bound)
        const float p0 = fast_exp2(t0), p1 = fast_exp2(t1);
        sum[(e >> 1) & 1] = fadd2(sum[(e >> 1) & 1], f2pack(p0, p1));
        pk[e >> 1] = Elem<T>::pack2(p0, p1);
    }
}

}  // namespace

template <typename T, int D, bool kWindow>   // kWindow: a left window bounds the keys
__global__ void __launch_bounds__(kThreads, 1)
    fa_prefill_sm100_kernel(const __grid_constant__ CUtensorMap qmap,
                            const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap,
                            const __grid_constant__ CUtensorMap omap, PrefillParams p) {
    using Sm = PrefillSmem<D>;
    constexpr bool kBF16 = !std::is_same<T, __half>::value;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[NUM_BARS];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    // scheduler ring: {unit index, q_len, kv_len, first query row of the sequence}
    __shared__ int4 sched_slot[4];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t sbase = (raw_base + 1023u) & ~1023u;
    uint8_t *sgen = smem_raw + (sbase - raw_base);
    const uint32_t bar0 = smem_u32(&bars[0]);
    auto BAR = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int i = 0; i < NUM_BARS; ++i) {
            const bool wg = i == P_FULL || i == P_FULL + 1 || i == O_FREE || i == O_FREE + 1;
            const bool sched = i >= SCHED_EMPTY && i < SCHED_EMPTY + 4;
            mbar_init(BAR(i), wg ? 128 : (sched ? kSchedConsumers : 1));
        }
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

    // Work units, heaviest first: index = ((u_from_top * batch) + b) * units_per_row + hp.
    // CTA c starts on unit c; further units are handed out dynamically from
    // gridDim.x + a global counter (p.sched[0]).  The Q/K producer warp draws them, skips
    // empty units and publishes each with its sequence's lengths and first row through
    // a 4-slot shared-memory ring (index -1 ends it); every other role takes the same
    // sequence from the ring, so all barrier phases stay in step and only the producer
    // reads the length arrays.
    const int HP = p.pair_heads ? p.num_heads / 2 : p.num_heads;
    const int total = p.num_units * p.batch * HP;
    struct Unit {
        int b, L, S, qs, off, kvh, N, J0;   // KV tiles [J0, N) of the unit
        int hX[2], q0X[2], rowsX[2], nX[2];
    };
    auto read_slot = [&](int k) -> int4 {
        const volatile int *v = reinterpret_cast<volatile int *>(&sched_slot[k & 3]);
        return make_int4(v[0], v[1], v[2], v[3]);
    };
    // k-th unit of this CTA for a whole-warp consumer (lane 0 releases the slot)
    auto take_unit_warp = [&](int k) -> int4 {
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(BAR(SCHED_FULL + (k & 3)), (k >> 2) & 1,
                                                       abortp, p.dev_error, kSiteSched)))
            return make_int4(-1, 0, 0, 0);
        const int4 e = read_slot(k);
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(SCHED_EMPTY + (k & 3)));
        return e;
    };
    // e = {index, q_len, kv_len, first row}
    auto decode_unit = [&](int4 e, Unit &u) -> bool {
        const int idx = e.x;
        const int hp = idx % HP;
        const int t = idx / HP;
        u.b = t % p.batch;
        const int unit = p.num_units - 1 - t / p.batch;
        u.L = e.y;
        u.S = e.z;
        u.qs = e.w;
        u.off = u.S - u.L;   // bottom-right causal: row i attends keys <= off + i
#pragma unroll
        for (int X = 0; X < 2; ++X) {
            if (p.pair_heads) {
                u.hX[X] = 2 * hp + X;
                u.q0X[X] = unit * kBM;
            } else {
                u.hX[X] = hp;
                u.q0X[X] = unit * 2 * kBM + X * kBM;
            }
            u.rowsX[X] = min(kBM, u.L - u.q0X[X]);
            // one past the last admissible key of the sub-tile's last row
            const int last = u.off + u.q0X[X] + u.rowsX[X] - 1;
            const int kv_hi =
                u.rowsX[X] > 0
                    ? min(u.S, p.causal ? last + 1
                                        : (p.window_right >= 0 ? last + p.window_right + 1 : u.S))
                    : 0;
            u.nX[X] = (u.rowsX[X] > 0 && kv_hi > 0) ? (kv_hi + kBN - 1) / kBN : 0;
        }
        u.N = max(u.nX[0], u.nX[1]);
        // first KV tile: the left window of the unit's first row (sub-tile 0's rows
        // come first); every active sub-tile has tiles past it
        u.J0 = kWindow ? max(0, u.off + u.q0X[0] - p.window_left) / kBN : 0;
        if (u.J0 >= u.N) u.J0 = 0;
        u.kvh = u.hX[0] / p.group;
        return u.rowsX[0] > 0 || u.rowsX[1] > 0;
    };

    if (warp == 0 || warp == 10) {
        // ===================== TMA producers: warp 0 -> Q and K, warp 10 -> V ==============
        // Separate warps so that a K tile never waits behind the V ring (K stages free up
        // after the S MMAs, V stages only after the PV MMAs).  Page ids of the next tile
        // are fetched while the current tile's stage is awaited.  Q of the next unit is
        // loaded as soon as the last S MMA of the current unit has read Q.
        const bool isV = warp == 10;
        if (lane == 0) tma_prefetch_desc(isV ? &vmap : &kmap);
        if (!isV && lane == 0) tma_prefetch_desc(&qmap);
        const CUtensorMap *map = isV ? &vmap : &kmap;
        const int nst = isV ? kVStages : kKStages;
        const int full0 = isV ? V_FULL : K_FULL;
        const int empty0 = isV ? V_EMPTY : K_EMPTY;
        const uint32_t ring = sbase + (isV ? Sm::kV0 : Sm::kK0);
        const int rpb = p.rows_per_box;
        const int nbox = kBN / rpb;
        int t_glob = 0;   // K or V tiles issued in this CTA
        int units = 0;    // units with work seen so far
        int zeroed = 0;   // last-tile clears done (V warp)
        bool ok = true;
        int next = blockIdx.x;   // next candidate unit (scheduler warp)
        for (int k = 0; ok; ++k) {
            int4 e;
            if (!isV) {
                // ===== scheduler: find the next non-empty unit and publish it =====
                if (k >= 4)
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait_bounded(BAR(SCHED_EMPTY + (k & 3)),
                                                      ((k >> 2) - 1) & 1, abortp, p.dev_error,
                                                      kSiteSched));
                e = make_int4(-1, 0, 0, 0);
                for (int c = next; ok && c < total;) {
                    const int b = (c / HP) % p.batch;
                    const int L = __ldg(p.q_seq_lens + b);
                    const int unit = p.num_units - 1 - c / (HP * p.batch);
                    if (unit == p.num_units - 1 && lane == 0 &&
                        L > p.num_units * (p.pair_heads ? kBM : 2 * kBM))
                        atomicCAS(p.dev_error, 0, kErrQBeyondPlan);
                    if (unit * (p.pair_heads ? kBM : 2 * kBM) < L) {
                        e = make_int4(c, L, __ldg(p.kv_seq_lens + b),
                                      warp_seq_start(p.q_seq_lens, b));
                        break;
                    }
                    int d = 0;   // empty unit: draw another
                    if (lane == 0) d = atomicAdd(p.sched, 1);
                    c = (int)gridDim.x + __shfl_sync(0xffffffffu, d, 0);
                }
                if (lane == 0) {
                    sched_slot[k & 3] = e;
                    mbar_arrive(BAR(SCHED_FULL + (k & 3)));
                    // many units per CTA: the next draw is in flight while this unit's
                    // tiles are issued (see draw_next for the few-units case)
                    if (e.x >= 0 && !p.late_draw) next = (int)gridDim.x + atomicAdd(p.sched, 1);
                }
                next = __shfl_sync(0xffffffffu, next, 0);
            } else {
                e = take_unit_warp(k);
            }
            if (e.x < 0) break;
            // few units per CTA (p.late_draw): the next unit is drawn once this unit's last
            // K tile is issued (about two tiles before it ends), so the choice follows the
            // CTAs' actual progress -- longest-first list scheduling, which evens out the
            // end of the kernel; with many units per CTA the early draw measured faster
            bool drawn = !p.late_draw;
            auto draw_next = [&]() {
                if (!isV && !drawn) {
                    if (lane == 0) next = (int)gridDim.x + atomicAdd(p.sched, 1);
                    next = __shfl_sync(0xffffffffu, next, 0);
                    drawn = true;
                }
            };
            Unit u;
            if (!decode_unit(e, u) || u.N == 0) {
                draw_next();
                continue;
            }
            const int qs = u.qs;
            if (!isV && lane == 0) {
                // Q buffers are free once the previous unit's last S MMAs completed
                if (units > 0)
                    ok = mbar_wait_bounded(BAR(Q_EMPTY), (units - 1) & 1, abortp, p.dev_error,
                                           kSiteEmpty + 0xf0);
                if (ok) {
                    uint32_t qbytes = 0;
#pragma unroll
                    for (int X = 0; X < 2; ++X)
                        if (u.nX[X] > 0) qbytes += Sm::kTileBytes;
                    mbar_arrive_expect_tx(BAR(Q_FULL), qbytes);
#pragma unroll
                    for (int X = 0; X < 2; ++X) {
                        if (u.nX[X] == 0) continue;
#pragma unroll
                        for (int hh = 0; hh < Sm::kHalves; ++hh)
                            tma_load_3d(sbase + Sm::kQ0 + X * Sm::kTileBytes + hh * Sm::kHalfBytes,
                                        &qmap, BAR(Q_FULL), hh * 64, u.hX[X], qs + u.q0X[X]);
                    }
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            ++units;
            const int *bt = p.block_table + (int64_t)u.b * p.block_table_dim;
            auto page_of = [&](int j, int &row) {
                int blk = p.num_pages;
                row = 0;
                if (lane < nbox) {
                    const int tok = j * kBN + lane * rpb;
                    const int pi = tok / p.block_size;
                    row = tok - pi * p.block_size;
                    if (tok < u.S && pi < p.block_table_dim) blk = __ldg(bt + pi);
                }
                return blk;
            };
            int row_next = 0;
            int blk_next = page_of(u.J0, row_next);
            for (int j = u.J0; ok && j < u.N; ++j, ++t_glob) {
                int blk = blk_next, row = row_next;
                if (j + 1 < u.N) blk_next = page_of(j + 1, row_next);  // in flight during wait
                if (blk < 0 || blk >= p.num_pages) blk = p.num_pages;   // out of range -> zeros
                const int st = t_glob % nst;
                if (t_glob >= nst)
                    ok = mbar_wait_bounded(BAR(empty0 + st), ((t_glob / nst) - 1) & 1, abortp,
                                           p.dev_error, kSiteEmpty + (isV ? 0x80 : 0));
                if (!ok) break;
                if (lane == 0) mbar_arrive_expect_tx(BAR(full0 + st), Sm::kTileBytes);
                __syncwarp();
                if (lane < nbox) {
                    const uint32_t dst = ring + st * Sm::kTileBytes + lane * rpb * 128;
#pragma unroll
                    for (int hh = 0; hh < Sm::kHalves; ++hh)
                        tma_load_4d(dst + hh * Sm::kHalfBytes, map, BAR(full0 + st), hh * 64,
                                    row, u.kvh, blk);
                }
            }
            draw_next();
            // V rows of the unit's last tile past kv_len may hold arbitrary bits
            // (unwritten cache slots): clear them before the PV MMAs of that tile
            if (ok && isV && u.N * kBN > u.S) {
                const int tl = t_glob - 1;
                const int vs = tl % kVStages;
                ok = mbar_wait_bounded(BAR(V_FULL + vs), (tl / kVStages) & 1, abortp,
                                       p.dev_error, kSiteVz);
                if (ok) {
                    const int first = u.S - (u.N - 1) * kBN;
                    uint8_t *vt = sgen + Sm::kV0 + vs * Sm::kTileBytes;
                    for (int r = first + lane; r < kBN; r += 32) {
#pragma unroll
                        for (int hh = 0; hh < Sm::kHalves; ++hh) {
                            uint4 *q4 =
                                reinterpret_cast<uint4 *>(vt + hh * Sm::kHalfBytes + r * 128);
#pragma unroll
                            for (int e = 0; e < 8; ++e) q4[e] = make_uint4(0, 0, 0, 0);
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(BAR(V_ZERO));
                    ++zeroed;
                }
            }
        }
        // on abort: let this warp's own copies in flight land before the CTA exits
        if (*abortp && lane == 0) {
            for (int t = t_glob - nst < 0 ? 0 : t_glob - nst; t < t_glob; ++t)
                mbar_wait_bounded(BAR(full0 + t % nst), (t / nst) & 1, nullptr, nullptr, 0,
                                  100000000ull);
        }
        (void)zeroed;
    } else if (warp == 1) {
        // ===================== MMA issuer (one thread) =====================
        // Fixed issue order, one (PV_X(j), S_X(j+1)) pair per sub-tile and tile:
        //   PV_A(j) S_A(j+1) | PV_B(j) S_B(j+1) | ...
        // Every operand of a pair is waited for first, then its 16 MMAs go out
        // back-to-back: the tcgen05 issue queue is only a few MMAs deep, so any
        // bookkeeping between groups would leave the tensor pipe idle.
        // S_X(j+1) must follow PV_X(j): P_X(j) lives in S_X's TMEM columns and the
        // MMAs of one thread execute in order.
        if (lane == 0) {
            const uint32_t idesc_qk = idesc_f16(kBF16, false, kBM, kBN);
            const uint32_t idesc_pv = idesc_f16(kBF16, true, kBM, D);
            // Descriptors are built once; per MMA only the start-address field (bits
            // 0-13, address >> 4) advances by a compile-time offset.  Shared-memory
            // addresses stay below 2^18 bytes, so the add never carries out of the field.
            const uint64_t dq0 = smem_desc_sw128(sbase + Sm::kQ0, 16, 1024);
            const uint64_t dk0 = smem_desc_sw128(sbase + Sm::kK0, 16, 1024);
            const uint64_t dv0 = smem_desc_sw128(sbase + Sm::kV0, Sm::kHalfBytes, 1024);
            const uint32_t tS0 = tmem + kColS, tO0 = tmem + kColO;
            auto issue_s = [&](int X, int kt) {
                const uint64_t dq = dq0 + (uint64_t)((X * Sm::kTileBytes) >> 4);
                const uint64_t dk = dk0 + (uint64_t)(((kt % kKStages) * Sm::kTileBytes) >> 4);
                const uint32_t d = tS0 + X * 128;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    constexpr int kHalfShift = Sm::kHalfBytes >> 4;
                    const uint64_t off = (uint64_t)((kk >> 2) * kHalfShift + (kk & 3) * 2);
                    tc_mma_ss(d, dq + off, dk + off, idesc_qk, kk > 0 ? 1u : 0u);
                }
            };
            auto issue_pv = [&](int X, int vt, bool first) {
                const uint64_t dv = dv0 + (uint64_t)(((vt % kVStages) * Sm::kTileBytes) >> 4);
                const uint32_t d = tO0 + X * 128, a = tS0 + X * 128;
#pragma unroll
                for (int t = 0; t < kBN / 16; ++t)
                    tc_mma_ts(d, a + t * 8, dv + (uint64_t)(t * 16 * 128 / 16), idesc_pv,
                              (!first || t > 0) ? 1u : 0u);
            };
            auto wait_k = [&](int kt) {
                return mbar_wait_bounded(BAR(K_FULL + kt % kKStages), (kt / kKStages) & 1, abortp,
                                         p.dev_error, kSiteK);
            };
            int kt = 0, vt = 0, units = 0, zeroed = 0;
            int pcount[2] = {0, 0};   // P_X hand-offs consumed
            int ounits[2] = {0, 0};   // units in which sub-tile X was active
            bool ok = true;
            for (int k = 0; ok; ++k) {
                // k-th unit of this CTA (single-thread consumer of the scheduler ring)
                if (!mbar_wait_bounded(BAR(SCHED_FULL + (k & 3)), (k >> 2) & 1, abortp,
                                       p.dev_error, kSiteSched))
                    break;
                const int4 e = read_slot(k);
                mbar_arrive(BAR(SCHED_EMPTY + (k & 3)));
                if (e.x < 0) break;
                Unit u;
                if (!decode_unit(e, u) || u.N == 0) continue;
                const bool partial = u.N * kBN > u.S;
                ok = mbar_wait_bounded(BAR(Q_FULL), units & 1, abortp, p.dev_error, kSiteQ) &&
                     wait_k(kt);
                ++units;
                if (!ok) break;
                tc_fence_after();
                // prologue: S_A(0), S_B(0)
#pragma unroll
                for (int X = 0; X < 2; ++X) {
                    if (u.nX[X] == 0) continue;
                    issue_s(X, kt);
                    tc_commit(BAR(S_FULL + X));
                }
                tc_commit(BAR(K_EMPTY + kt % kKStages));
                if (u.N - u.J0 == 1) tc_commit(BAR(Q_EMPTY));
                for (int j = u.J0; ok && j < u.N; ++j) {
                    const int vj = vt + (j - u.J0);       // V ring tile of unit tile j
                    const int kn = kt + (j - u.J0) + 1;   // K ring tile of unit tile j+1
                    ok = mbar_wait_bounded(BAR(V_FULL + vj % kVStages), (vj / kVStages) & 1,
                                           abortp, p.dev_error, kSiteV);
                    if (ok && j == u.N - 1 && partial) {
                        ok = mbar_wait_bounded(BAR(V_ZERO), zeroed & 1, abortp, p.dev_error,
                                               kSiteVz);
                        ++zeroed;
                    }
                    if (ok && j + 1 < u.N) ok = wait_k(kn);
                    if (!ok) break;
#pragma unroll
                    for (int X = 0; X < 2; ++X) {
                        const int n = u.nX[X];
                        if (j >= n) continue;
                        ok = mbar_wait_bounded(BAR(P_FULL + X), pcount[X] & 1, abortp,
                                               p.dev_error, kSiteP);
                        ++pcount[X];
                        // the previous unit's epilogue must have read O_X before it is reset
                        if (ok && j == u.J0 && ounits[X] > 0)
                            ok = mbar_wait_bounded(BAR(O_FREE + X), (ounits[X] - 1) & 1, abortp,
                                                   p.dev_error, kSiteO);
                        if (!ok) break;
                        tc_fence_after();
                        issue_pv(X, vj, j == u.J0);
                        if (j + 1 < n) {
                            issue_s(X, kn);
                            tc_commit(BAR(S_FULL + X));
                        } else {
                            tc_commit(BAR(O_DONE + X));
                        }
                    }
                    if (!ok) break;
                    tc_commit(BAR(V_EMPTY + vj % kVStages));
                    if (j + 1 < u.N) {
                        tc_commit(BAR(K_EMPTY + kn % kKStages));
                        if (j + 2 == u.N) tc_commit(BAR(Q_EMPTY));   // last S of the unit
                    }
                }
#pragma unroll
                for (int X = 0; X < 2; ++X)
                    if (u.nX[X] > 0) ++ounits[X];
                kt += u.N - u.J0;
                vt += u.N - u.J0;
            }
            // drain: every MMA issued by this thread has completed before TMEM is freed
            tc_commit(BAR(DRAIN));
            mbar_wait_bounded(BAR(DRAIN), 0, nullptr, p.dev_error, kSiteDrain);
        }
        __syncwarp();
    } else {
        // ===================== softmax + epilogue (one row per thread) =====================
        // warps 2-5 serve sub-tile 0 and warps 6-9 sub-tile 1; a warp may only touch
        // TMEM lanes 32*(warp%4) .. +31, so row r = 32*(warp%4) + lane
        const int X = (warp - 2) >> 2;
        const int r = 32 * (warp & 3) + lane;
        const uint32_t lane_addr = (uint32_t)(32 * (warp & 3)) << 16;
        const uint32_t tS = tmem + lane_addr + kColS + X * 128;
        const uint32_t tO = tmem + lane_addr + kColO + X * 128;
        const float sl2 = p.scale_log2;
        int scount = 0, ocount = 0;
        bool ok = true;
        for (int k = 0; ok; ++k) {
            const int4 e = take_unit_warp(k);
            if (e.x < 0) break;
            Unit u;
            if (!decode_unit(e, u)) continue;
            const int n = X ? u.nX[1] : u.nX[0];
            const int rows = X ? u.rowsX[1] : u.rowsX[0];
            const int hx = X ? u.hX[1] : u.hX[0];
            const int qi = (X ? u.q0X[1] : u.q0X[0]) + r;
            const int qs = u.qs;
            if (n == 0) {
                // rows with no admissible key (q_len > kv_len) are written as zeros
                if (r < rows && qs + qi < p.total_q) {
                    T *o = static_cast<T *>(p.out) + ((int64_t)(qs + qi) * p.num_heads + hx) * D;
                    for (int d = 0; d < D; ++d) o[d] = Elem<T>::from_float(0.f);
                    if (p.lse != nullptr) p.lse[(int64_t)hx * p.total_q + qs + qi] = -INFINITY;
                }
                continue;
            }
            // admissible keys of this row: [klo, klim]
            const int klim = min(p.causal ? u.off + qi
                                          : (p.window_right >= 0 ? u.off + qi + p.window_right
                                                                 : u.S - 1),
                                 u.S - 1);
            const int klo = kWindow ? max(0, u.off + qi - p.window_left) : 0;
            float m_s = -INFINITY;   // running max, scaled (log2) units
            float l = 0.f;
            for (int j = u.J0; j < n; ++j) {
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(BAR(S_FULL + X), scount & 1,
                                                               abortp, p.dev_error, kSiteS))) {
                    ok = false;
                    break;
                }
                ++scount;
                tc_fence_after();
                const int kbase = j * kBN;
                // columns c outside [nlo, nvalid) are masked (causal / window / kv_len tail)
                const int nvalid = klim - kbase + 1;
                const int nlo = kWindow ? klo - kbase : -kBN;
                const bool masked = __any_sync(0xffffffffu, nvalid < kBN || (kWindow && nlo > 0));
                // the whole 128-score row in registers: four loads, one wait
                uint32_t uu[4][32];
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c) tmem_ld32(tS + c * 32, uu[c]);
                tmem_ld_wait();
                float mx = -INFINITY;
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c)
                    mx = masked ? chunk_max<true>(uu[c], nlo - c * 32, nvalid - c * 32, mx)
                                : chunk_max<false>(uu[c], 0, 32, mx);
                const float m_new = fmaxf(m_s, mx * sl2);
                const bool need = (j == u.J0) || (m_new > m_s + 8.0f);
                const bool warp_need = __any_sync(0xffffffffu, need);
                float alpha = 1.f;
                if (warp_need) {
                    alpha = (m_s == -INFINITY) ? 0.f : fast_exp2(m_s - m_new);
                    m_s = m_new;
                }
                const float m_use = (m_s == -INFINITY) ? 0.f : m_s;
                // p = 2^(s*scale - m), row sum, P (16-bit) written over the S columns
                const uint64_t sl2x2 = f2pack(sl2, sl2);
                const uint64_t negm2 = f2pack(-m_use, -m_use);
                uint64_t sum2[2] = {f2pack(0.f, 0.f), f2pack(0.f, 0.f)};
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c) {
                    uint32_t pk[16];
                    // a chunk masked for every row of the warp (the upper triangle of the
                    // diagonal tile, keys past kv_len, keys before a window) needs no exp2
                    if (masked && __all_sync(0xffffffffu, nvalid - c * 32 <= 0 ||
                                                              nlo - c * 32 >= 32)) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) pk[e] = 0u;
                    } else if (masked)
                        chunk_exp<T, true>(uu[c], nlo - c * 32, nvalid - c * 32, sl2x2, negm2,
                                           sum2, pk);
                    else
                        chunk_exp<T, false>(uu[c], 0, 32, sl2x2, negm2, sum2, pk);
                    tmem_st16(tS + c * 16, pk);
                }
                float s0, s1, s2, s3;
                f2unpack(sum2[0], s0, s1);
                f2unpack(sum2[1], s2, s3);
                l = l * alpha + ((s0 + s1) + (s2 + s3));
                // O rescale: PV_X(j-1) has completed (S_X(j), issued after it, has)
                if (j > u.J0 && warp_need) {
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t v[32];
                        tmem_ld32(tO + c * 32, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
                        tmem_st32(tO + c * 32, v);
                    }
                }
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(BAR(P_FULL + X));
            }
            if (!ok) break;
            // epilogue; then hand O_X back for the next unit's first PV
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(BAR(O_DONE + X), ocount & 1, abortp,
                                                           p.dev_error, kSiteO))) {
                ok = false;
                break;
            }
            ++ocount;
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            const bool store = r < rows && qs + qi < p.total_q;
            if (store && p.lse != nullptr)
                p.lse[(int64_t)hx * p.total_q + qs + qi] =
                    l > 0.f ? (m_s + log2f(l)) * 0.6931471805599453f : -INFINITY;
            T *orow = static_cast<T *>(p.out) + ((int64_t)(qs + qi) * p.num_heads + hx) * D;
            uint32_t ov[D / 32][32];
#pragma unroll
            for (int c = 0; c < D / 32; ++c) tmem_ld32(tO + c * 32, ov[c]);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(BAR(O_FREE + X));
            // warps whose 32 rows all belong to the sequence stage their rows in shared
            // memory (128-byte swizzle, conflict-free) one 64-column half at a time and
            // write them with one TMA store per half, instead of 32 scattered lines per
            // store instruction
            const int wrow0 = 32 * (warp & 3);
            const bool via_tma = p.out_tma && wrow0 + 32 <= rows &&
                                 qs + (X ? u.q0X[1] : u.q0X[0]) + wrow0 + 32 <= p.total_q;
            if (via_tma) {
                const uint32_t stg = sbase + Sm::kO0 + (warp - 2) * Sm::kOWarpBytes;
#pragma unroll
                for (int hh = 0; hh < D / 64; ++hh) {
                    if (lane == 0) bulk_wait_read_all();   // the buffer's last store has read it
                    __syncwarp();
#pragma unroll
                    for (int c2 = 0; c2 < 2; ++c2) {
                        const int c = hh * 2 + c2;
                        uint32_t pkd[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            pkd[e] = Elem<T>::pack2(__uint_as_float(ov[c][2 * e]) * inv,
                                                    __uint_as_float(ov[c][2 * e + 1]) * inv);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int ch = c2 * 4 + e;   // 16-byte chunk of the 128-byte half-row
                            st_shared_v4(stg + lane * kStageRowBytes + ((ch ^ (lane & 7)) << 4),
                                         pkd[4 * e], pkd[4 * e + 1], pkd[4 * e + 2],
                                         pkd[4 * e + 3]);
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_3d(&omap, stg, hh * 64, hx,
                                     qs + (X ? u.q0X[1] : u.q0X[0]) + wrow0);
                        bulk_commit_group();
                    }
                }
            } else if (store) {
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t pkd[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        pkd[e] = Elem<T>::pack2(__uint_as_float(ov[c][2 * e]) * inv,
                                                __uint_as_float(ov[c][2 * e + 1]) * inv);
                    if (p.out_al32) {
                        // 256-bit stores: each covers one whole 32-byte sector of the row
#pragma unroll
                        for (int e = 0; e < 2; ++e)
                            st_global_v8(orow + c * 32 + 16 * e, &pkd[8 * e]);
                    } else {
                        uint4 *dst = reinterpret_cast<uint4 *>(orow + c * 32);
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            dst[e] = make_uint4(pkd[4 * e], pkd[4 * e + 1], pkd[4 * e + 2],
                                                pkd[4 * e + 3]);
                    }
                }
            }
        }
    }

    // the epilogue's TMA stores have finished before the CTA's shared memory goes away
    if (warp >= 2 && warp < 10 && lane == 0) bulk_wait_all();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    // the last CTA to finish resets the scheduler counters for the next launch
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
            atomicExch(p.sched, 0);
            atomicExch(p.sched + 1, 0);
        }
    }
}

// ---- host side ------------------------------------------------------------------------

bool prefill_supported(int head_dim, int block_size, int group) {
    (void)group;
    if (head_dim != 64 && head_dim != 128) return false;
    if (block_size <= 0) return false;
    if (block_size <= 128) return block_size >= 8 && (128 % block_size) == 0;
    return (block_size % 128) == 0;
}

size_t prefill_workspace_bytes(const AttnShape &) { return 0; }

template <typename T, int D>
static cudaError_t launch_prefill_t(const AttnShape &s, int *dev_error, int num_sms,
                                   cudaStream_t stream) {
    if (dev_error == nullptr) return cudaErrorInvalidValue;   // holds the scheduler counters
    PFN_encodeTiled enc = get_encode_fn();
    if (!enc) return cudaErrorNotSupported;
    const CUtensorMapDataType dt =
        std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap qmap, kmap, vmap, omap;
    memset(&omap, 0, sizeof(omap));
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
        const CacheElem ce = std::is_same<T, __half>::value ? CacheElem::F16 : CacheElem::BF16;
        if (!encode_cache_map(&kmap, s.key_cache, ce, D, s.block_size, s.num_kv_heads,
                              s.num_pages, rpb, s.kv_layout) ||
            !encode_cache_map(&vmap, s.value_cache, ce, D, s.block_size, s.num_kv_heads,
                              s.num_pages, rpb, s.kv_layout))
            return cudaErrorInvalidValue;
    }
    PrefillParams p;
    p.q_seq_lens = s.q_seq_lens;
    p.kv_seq_lens = s.kv_seq_lens;
    p.block_table = s.block_table;
    p.out = s.out;
    p.dev_error = dev_error;
    p.sched = dev_error + 1;
    p.num_heads = s.num_heads;
    p.num_kv_heads = s.num_kv_heads;
    p.group = s.num_heads / s.num_kv_heads;
    p.pair_heads = (p.group % 2 == 0) ? 1 : 0;
    p.block_size = s.block_size;
    p.rows_per_box = rpb;
    p.block_table_dim = s.block_table_dim;
    p.num_pages = s.num_pages;
    const int nqt = (s.max_q + kBM - 1) / kBM;
    p.num_units = p.pair_heads ? nqt : (nqt + 1) / 2;
    p.total_q = s.total_q;
    p.batch = s.batch;
    p.scale_log2 = s.scale_log2;
    p.causal = s.causal;
    p.window_left = s.window_left;
    p.window_right = s.window_right;
    p.lse = s.lse;
    p.out_al32 = (reinterpret_cast<uintptr_t>(s.out) & 31u) == 0 ? 1 : 0;
    p.out_tma = 0;
    if ((reinterpret_cast<uintptr_t>(s.out) & 15u) == 0) {
        cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)s.num_heads, (cuuint64_t)s.total_q};
        cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)s.num_heads * D * 2};
        cuuint32_t box[3] = {64, 1, 32};
        cuuint32_t es[3] = {1, 1, 1};
        if (enc(&omap, dt, 3, s.out, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
            p.out_tma = 1;
    }
    if (p.num_units <= 0 || s.batch <= 0) return cudaSuccess;

    auto kfn = s.window_left >= 0 ? fa_prefill_sm100_kernel<T, D, true>
                                  : fa_prefill_sm100_kernel<T, D, false>;
    const int smem = PrefillSmem<D>::kAlloc;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const int units_total =
        p.num_units * s.batch * (p.pair_heads ? s.num_heads / 2 : s.num_heads);
    // persistent: one CTA per SM, units handed out by the in-kernel scheduler
    dim3 grid(units_total < num_sms ? units_total : num_sms);
    p.late_draw = units_total < 12 * (int)grid.x ? 1 : 0;   // fewer than ~12 per CTA
    kfn<<<grid, kThreads, smem, stream>>>(qmap, kmap, vmap, omap, p);
    return cudaGetLastError();
}

cudaError_t launch_prefill(const AttnShape &s, bool bf16, void *workspace, int *dev_error,
                           int num_sms, cudaStream_t stream) {
    (void)workspace;
    const uintptr_t a = reinterpret_cast<uintptr_t>(s.q) | reinterpret_cast<uintptr_t>(s.key_cache) |
                        reinterpret_cast<uintptr_t>(s.value_cache);
    if (a & 15u) return cudaErrorMisalignedAddress;
    if (s.head_dim == 128)
        return bf16 ? launch_prefill_t<__nv_bfloat16, 128>(s, dev_error, num_sms, stream)
                    : launch_prefill_t<__half, 128>(s, dev_error, num_sms, stream);
    if (s.head_dim == 64)
        return bf16 ? launch_prefill_t<__nv_bfloat16, 64>(s, dev_error, num_sms, stream)
                    : launch_prefill_t<__half, 64>(s, dev_error, num_sms, stream);
    return cudaErrorInvalidValue;
}

}  // namespace kern
}  // namespace tecoops
